// Host-side launch parameters of the tcgen05 attention kernels.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace sisa {

struct FwdParams {
  CUtensorMap tm_q;    // (64, L, H, B) bf16/fp16, box (64, 128), 128B swizzle
  CUtensorMap tm_k;    // box (64, 64)
  CUtensorMap tm_v;    // box (64, 64)
  CUtensorMap tm_c;    // (32, L, H, B), box (32, 128), 64B swizzle
  CUtensorMap tm_b;    // box (32, 64)
  CUtensorMap tm_pos;  // (L, 4, B*H) fp32 planes, box (64, 4, 1)
  CUtensorMap tm_ost;  // o, (64, L, H, B) view, box (64, 128), 128B swizzle (bulk-tensor store)
  CUtensorMap tm_o32;  // o'', (64, L, B*H) fp32, box (32, 128, 1), 128B swizzle (bulk-tensor store)
  const float* pos;    // (B*H, 4, Lp) planes {g, F, rowf, colf}
  const float* lam;
  char* o;
  int64_t o_sb, o_sh, o_sl;
  float* lse;
  float* o32;
  int B, H, L, Lp, ntq;
  int32_t* status;
};

struct BwdParams {
  // dq kernel (query-tile owner): Q, dO, C resident (box rows 128); K, V, B streamed (box rows 64)
  CUtensorMap tm_q128, tm_do128, tm_c128, tm_k64, tm_v64, tm_b64;
  // dkv kernel (key-tile owner): K, V, B resident (box rows 128); Q, dO, C streamed (box rows 64)
  CUtensorMap tm_k128, tm_v128, tm_b128, tm_q64, tm_do64, tm_c64;
  CUtensorMap tm_pos;    // (L, 4, B*H) fp32 planes, box (64, 4, 1)
  CUtensorMap tm_rstat;  // (L, 4, B*H) fp32 planes, box (64, 4, 1)
  // dq kernel: o'' as (64, L, B*H) fp32, box (32, 128, 1), 128B swizzle; or, without o'', o as a
  // (64, L, H, B) view, box (64, 128). dq (64, L, H, B) and dc (32, L, H, B) fp32, box rows 128,
  // 128B swizzle, for the epilogue's bulk-tensor stores.
  CUtensorMap tm_o, tm_dq, tm_dc;
  // dkv kernel: dk, dv (64, L, H, B) and db (32, L, H, B) fp32, box rows 128, 128B swizzle (stores)
  CUtensorMap tm_dk, tm_dv, tm_db;
  const float* pos;      // (B*H, 4, Lp) planes {g, F, rowf, colf}
  const float* lam;
  const char* q;  int64_t q_sb, q_sh, q_sl;
  const char* k;  int64_t k_sb, k_sh, k_sl;
  const char* bm; int64_t b_sb, b_sh, b_sl;
  const char* o;  int64_t o_sb, o_sh, o_sl;
  const char* dout; int64_t do_sb, do_sh, do_sl;
  const float* lse;
  const float* o32;
  char* dq; int64_t dq_sb, dq_sh, dq_sl;
  char* dk; int64_t dk_sb, dk_sh, dk_sl;
  char* dv; int64_t dv_sb, dv_sh, dv_sl;
  float* dc; int64_t dc_sb, dc_sh, dc_sl;
  float* db; int64_t db_sb, db_sh, db_sl;
  float* dg;
  float* dF;
  float* rstat;    // (B*H, 4, Lp) planes {F log2e - lse, -delta, -(T^ - delta), dS_tt} per query row
  float* rg;       // (B*H, L) row part of dg (times lambda)
  float* rf;       // row part of dF
  float* rl;       // per-row dlambda
  float* dlam;
  int B, H, L, Lp, ntq128, ntq64;
  int has_f;
  int32_t* status;
};

static_assert(sizeof(BwdParams) <= 4096, "kernel parameter block");

cudaError_t launch_attn_fwd(const FwdParams& p, int dtype, cudaStream_t st);
cudaError_t launch_attn_bwd(const BwdParams& p, int dtype, cudaStream_t st);

}  // namespace sisa
