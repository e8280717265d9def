// gemm.cu - persistent GEMM C (+)= A B^T on CTA pairs with the 5th-generation tensor cores
// (tcgen05 with cta_group::2): the linear-CE logits (with the online log-sum-exp in the epilogue,
// src/sisa/kernels/linear_ce.py:60-89) and its gradients dX = G W and dW += G^T X, and the plain
// GEMMs of the model's projections.
//
// A cluster of two CTAs computes 256 x 256 (narrow) or 256 x 512 (wide) tiles of C: each CTA loads
// its own 128 rows of A and its own half of the tile's B rows per 64-wide K stage with plain TMA tile
// loads that fill only the issuing CTA's shared memory, and the UMMAs of M = 256, N = 256, K = 16
// issued by the leader CTA read both CTAs' shared memory, so every B byte is loaded once per pair
// instead of once per CTA. Each CTA's
// tensor memory holds its 128 rows of the fp32 accumulator (512 columns: two 256-column buffers, or
// the two halves of one wide tile).
//
// Roles: E = 16 (narrow) or 8 (wide) epilogue warps (warp w reads TMEM lanes 32 (w % 4) .. + 31, the
// rows of its lane quarter, and 1024 / E columns of each 256-column part from (w / 4) 1024 / E), then
// the TMA producer warp, then the owner of the tensor memory and, in the leader CTA, the UMMA issuer.
// Barriers (same offsets in both CTAs):
//   full[s]      leader only: the leader's producer arrives with the stage's byte count of both CTAs,
//                and both CTAs' TMA loads complete on it;
//   empty[s]     both: the leader's UMMA commit arrives on both CTAs' copies when the stage is read;
//   acc_full[b]  both: the leader's commit after a tile's last K stage;
//   acc_empty[p] leader only: the epilogue warps of each CTA arrive when they have drained part p.
// Launched in clusters of two CTAs (cudaLaunchKernelEx). Every wait is bounded (SISA_ST_TIMEOUT); all
// warps of both CTAs meet at the final cluster barrier before the tensor memory is freed, so neither
// CTA leaves while the leader's UMMAs use its memory.
#include <cuda_runtime.h>

#include <cstdint>

#include "attn_common.cuh"
#include "gemm.h"

namespace sisa {
namespace gemm {

constexpr int BMC = 128;                   // rows of A per CTA (the pair tile has 256)
constexpr int BK = 64;
constexpr uint32_t SZ_HALF = 128 * BK * 2;                 // one CTA's 128 x 64 operand block: 16 KB
constexpr uint32_t TMEM_COLS = 512;


// Two tile shapes. Narrow: 256 x 256 pair tiles, five 32 KB stages, the accumulator double buffered
// (2 x 256 columns), so that a tile's epilogue runs under the next tile's UMMAs, and 16 epilogue warps
// (64 columns each): for short K, where the epilogue must keep up with the UMMAs. Wide: 256 x 512 pair
// tiles (two N = 256 UMMAs per K step into the two 256-column halves of one accumulator), four 48 KB
// stages and 8 epilogue warps (128 columns each): a quarter fewer operand bytes per flop from L2, for
// long K, where the epilogue (which the next tile's UMMAs into each half wait for) is a small part of a
// tile.
template <bool kWide, int EPI = EPI_STORE>
struct Cfg {
  static constexpr int BN = kWide ? 512 : 256;             // columns of the pair tile
  static constexpr int NST = kWide || EPI == EPI_SWIGLU ? 4 : 5;
  static constexpr int NBUF = kWide ? 1 : 2;               // accumulator buffers
  static constexpr int NHALF = kWide ? 2 : 1;              // 256-column parts per buffer
  static constexpr int NEPI = kWide ? 8 : 16;              // epilogue warps
  static constexpr int CW = 256 / (NEPI / 4);              // columns of a part per epilogue warp
  static constexpr int NTHREADS = 32 * (NEPI + 2);
  static constexpr int NBOX = 1;                           // staging boxes per epilogue warp
  static constexpr uint32_t SZ_B = NHALF * SZ_HALF;
  static constexpr uint32_t SZ_STAGE = SZ_HALF + SZ_B;     // A | B
  static constexpr uint32_t OFF_EPI = NST * SZ_STAGE;      // 160 / 192 KB of stages
  static constexpr uint32_t SZ_EPI = 4096;                 // one staging box: 32 rows x 128 bytes
  static constexpr uint32_t SZ_EPI2 = EPI == EPI_SWIGLU ? 2048 : 0;   // SwiGLU: a box of 32 rows x 64 bytes
  static constexpr uint32_t OFF_EPI2 = OFF_EPI + NEPI * NBOX * SZ_EPI;
  static constexpr uint32_t OFF_BAR = OFF_EPI2 + NEPI * SZ_EPI2;
  static_assert(NTHREADS * (kWide ? 168 : 112) <= 65536, "register budget of one CTA per SM");
  static constexpr int B_FULL = 0, B_EMPTY = NST, B_ACCF = 2 * NST, B_ACCE = 2 * NST + 2;
  // EPI_LCE: per row quarter and tile parity, "the other column groups' (max, sum) are in tensor memory"
  static constexpr int B_REC = 2 * NST + 4;
  static constexpr uint32_t TMEM_SLOT = 192;               // byte offset of the TMEM address in the barrier area
  static constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 + 1024;
  static_assert(SMEM_BYTES <= 232448, "fits the 227 KB shared-memory limit");
  static_assert((B_REC + 8) * 8 <= (int)TMEM_SLOT, "barriers end below the TMEM slot");
  static_assert(NBUF * NHALF * 256 == (int)TMEM_COLS, "the accumulators fill the tensor memory");
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The shared::cluster address of `saddr` (a shared::cta address of this CTA) in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Tile load into this CTA's shared memory that completes on an mbarrier of either CTA of the pair.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void* map, uint32_t bar_cluster, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
      ::"r"(dst), "l"(map), "r"(bar_cluster), "r"(c0), "r"(c1) : "memory");
}
__device__ __forceinline__ void umma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// Arrive once, when the UMMAs issued so far complete, on the barrier at this offset in both CTAs.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  const uint16_t both = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
      ::"r"(bar), "h"(both) : "memory");
}
// Store (or, for the accumulating fp32 output, add with a reduction in L2) one staged box of C.
__device__ __forceinline__ void tma_store_2d(const void* map, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"(map), "r"(src), "r"(c0), "r"(c1) : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const void* map, uint32_t src, int c0, int c1) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"(map), "r"(src), "r"(c0), "r"(c1) : "memory");
}
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Split-K: every K slice of a tile writes its fp32 partial of a warp's 32 rows x 64 columns to its own
// workspace slot (element i of lane l at slot[i * 32 + l]: each warp store is one coalesced 128-byte
// line) and counts itself in; the slice that arrives last sums the slots in slice order (a fixed
// order whoever arrives last: deterministic) and stores C. Slots are read past L1 (other SMs wrote them).
__device__ __forceinline__ void write_partial(float* slot, const float* v, int lane) {
#pragma unroll
  for (int i = 0; i < 64; ++i) __stcg(slot + i * 32 + lane, v[i]);
}
__device__ __forceinline__ bool arrive_last(uint32_t* counter, int ns, int lane) {
  __syncwarp();
  uint32_t old = 0;
  if (lane == 0) {
    __threadfence();
    old = atomicAdd(counter, 1u);
    __threadfence();
  }
  old = __shfl_sync(0xffffffffu, old, 0);
  return old + 1 == (uint32_t)ns;
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Tile t -> (pair-tile row mb, column nb). Tiles run in groups of GROUP_M tile rows, column by column
// within a group, so that the pairs resident at one time cover a near-square block of C and the A and
// B rows they stream stay in L2 together (each operand byte comes from DRAM about once per block).
constexpr int GROUP_M = 8;
__device__ __forceinline__ void tile_coords(const GemmParams& p, int t, int& mb, int& nb) {
  const int per_group = GROUP_M * p.num_n;
  const int g = t / per_group, r = t - g * per_group;
  const int rows = min(GROUP_M, p.num_m - g * GROUP_M);
  mb = g * GROUP_M + r % rows;
  nb = r / rows;
}

// Staging: a warp's 32 rows x 128 bytes of C go into a 128-byte-swizzled box (row r's 16-byte chunk q
// at r * 128 + ((q ^ (r & 7)) << 4): one st.shared.v4 per chunk and thread, no bank conflicts beyond
// the 4 wavefronts a 512-byte warp store needs), then one TMA store of the box (rows and columns
// beyond C are clipped by the tensor map). With NBOX boxes per warp, a box is rewritten only after
// the store issued from it NBOX steps earlier has read it.
template <int NBOX>
__device__ __forceinline__ uint32_t stage_and_store(const GemmParams& p, const uint32_t* w, uint32_t boxes, int lane,
                                                    int col, int row0, int& nbox, bool reduce) {
  const uint32_t box = boxes + (uint32_t)(nbox % NBOX) * 4096u;
  if (lane == 0 && nbox >= NBOX) {
    if constexpr (NBOX == 1) bulk_wait_read0(); else bulk_wait_read1();
  }
  __syncwarp();
#pragma unroll
  for (int q = 0; q < 8; ++q)
    st_shared_v4(box + sw128_off((uint32_t)lane, (uint32_t)q), w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (reduce) tma_reduce_add_2d(&p.tm_c, box, col, row0);
    else tma_store_2d(&p.tm_c, box, col, row0);
    bulk_commit();
  }
  ++nbox;
  return box;
}

// The bias of columns col .. col + 7 as fp32: bias[c - bias_c0] inside [bias_c0, bias_c1), 0 outside; the
// same address in every lane (a broadcast load). The type is branched on once per call, not per value.
template <bool kRoundHalf>
__device__ __forceinline__ void load_bias8(const GemmParams& p, int col, float* b) {
  const int i0 = col - p.bias_c0;
  if (p.bias_vec && i0 >= 0 && col + 8 <= p.bias_c1) {
    if (p.bias_dtype == 2) {
      const float4 a = reinterpret_cast<const float4*>(p.bias)[i0 / 4], c = reinterpret_cast<const float4*>(p.bias)[i0 / 4 + 1];
      b[0] = a.x; b[1] = a.y; b[2] = a.z; b[3] = a.w; b[4] = c.x; b[5] = c.y; b[6] = c.z; b[7] = c.w;
    } else {
      const uint4 u = reinterpret_cast<const uint4*>(p.bias)[i0 / 8];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
      if (p.bias_dtype == 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i) { b[2 * i] = unpack_lo<true>(w[i]); b[2 * i + 1] = unpack_hi<true>(w[i]); }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) { b[2 * i] = unpack_lo<false>(w[i]); b[2 * i + 1] = unpack_hi<false>(w[i]); }
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = col + i;
      b[i] = c < p.bias_c0 || c >= p.bias_c1 ? 0.f
             : p.bias_dtype == 2 ? static_cast<const float*>(p.bias)[c - p.bias_c0]
             : p.bias_dtype == 1 ? __half2float(static_cast<const __half*>(p.bias)[c - p.bias_c0])
                                 : __bfloat162float(static_cast<const __nv_bfloat16*>(p.bias)[c - p.bias_c0]);
    }
  }
  if (p.bias_round) {
#pragma unroll
    for (int i = 0; i < 8; ++i) b[i] = round_lp<kRoundHalf>(b[i]);
  }
}

// Whether the n columns from col meet the bias's columns (boxes outside them skip the bias).
__device__ __forceinline__ bool bias_meets(const GemmParams& p, int col, int n) {
  return col < p.bias_c1 && col + n > p.bias_c0;
}

// Epilogue EPI_STORE of 32 fp32 values per thread already in registers (the summed split-K slices).
template <int NBOX>
__device__ __forceinline__ void epilogue_store_values(const GemmParams& p, const float* vin, uint32_t boxes, int lane,
                                                      int col, int row0, int& nbox, bool reduce, bool add_bias) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = vin[i];
  if (add_bias && bias_meets(p, col, 32)) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      float b[8];
      load_bias8<false>(p, col + j, b);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[j + i] += b[i];
    }
  }
  uint32_t w[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(v[i]);
  stage_and_store<NBOX>(p, w, boxes, lane, col, row0, nbox, reduce);
}

// Epilogue EPI_STORE: one 128-byte box (32 fp32 or 64 bf16/fp16 columns) of the warp's 32 rows, plus
// the bias when given; `reduce` adds the box into C (fp32) instead of storing it.
template <int OUT, int NBOX>
__device__ __forceinline__ void epilogue_store(const GemmParams& p, uint32_t taddr, uint32_t boxes, int lane, int col,
                                               int row0, int& nbox, bool reduce, bool add_bias) {
  constexpr int NV = OUT == GEMM_OUT_F32 ? 32 : 64;
  float v[NV];
  tmem_ld32(taddr, v);
  if constexpr (NV == 64) tmem_ld32(taddr + 32u, v + 32);
  tmem_wait_ld();
  if (add_bias && bias_meets(p, col, NV)) {
#pragma unroll
    for (int j = 0; j < NV; j += 8) {
      float b[8];
      load_bias8<OUT == GEMM_OUT_F16>(p, col + j, b);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[j + i] += b[i];
    }
  }
  uint32_t w[32];
  if constexpr (OUT == GEMM_OUT_F32) {
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(v[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = pack2<OUT == GEMM_OUT_F16>(v[2 * i], v[2 * i + 1]);
  }
  stage_and_store<NBOX>(p, w, boxes, lane, col, row0, nbox, reduce);
}

// Maximum of two packed pairs of bf16 / fp16 values, lane by lane, NaN if either is NaN.
template <bool kHalf>
__device__ __forceinline__ uint32_t max2_nan(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (kHalf) asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  else asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Epilogue EPI_LCE (the linear-CE logits, C = X W^T in the compute dtype): the warp's one 64-column box
// of its 32 rows, stored like EPI_STORE, and folded into the thread's running maximum m (log2 units) /
// sum s of 2^(x log2 e - m) over the rounded logits x of the real vocabulary columns (col < V; a NaN
// logit makes both NaN), and the label's logit when it lies in the box. The maximum is taken on the
// packed rounded values (exact), and the sum in four independent chains.
template <bool kHalf, int NBOX>
__device__ __forceinline__ void epilogue_lce(const GemmParams& p, uint32_t taddr, uint32_t boxes, int lane, int col,
                                             int row0, int& nbox, int64_t lab, float& m, float& s, float& tgt,
                                             bool& has_tgt) {
  constexpr float kLog2e = 1.4426950408889634f;
  uint32_t w[32];
  {
    float v[64];
    tmem_ld32(taddr, v);
    tmem_ld32(taddr + 32u, v + 32);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = pack2<kHalf>(v[2 * i], v[2 * i + 1]);
  }
  const uint32_t box = stage_and_store<NBOX>(p, w, boxes, lane, col, row0, nbox, false);
  const int64_t d = lab - col;
  if (d >= 0 && d < 64) {
    // the label's rounded logit, read back from this thread's row of the staging box
    uint16_t h;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h)
                 : "r"(box + sw128_off((uint32_t)lane, (uint32_t)(d >> 3)) + 2u * (uint32_t)(d & 7)));
    tgt = unpack_lo<kHalf>((uint32_t)h);
    has_tgt = true;
  }
  float mc;
  const bool full = col + 64 <= p.V;
  if (full) {
    uint32_t q[4] = {w[0], w[1], w[2], w[3]};
#pragma unroll
    for (int i = 4; i < 32; ++i) q[i & 3] = max2_nan<kHalf>(q[i & 3], w[i]);
    const uint32_t qq = max2_nan<kHalf>(max2_nan<kHalf>(q[0], q[1]), max2_nan<kHalf>(q[2], q[3]));
    mc = max_nan(unpack_lo<kHalf>(qq), unpack_hi<kHalf>(qq)) * kLog2e;
  } else {
    mc = -INFINITY;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const float x = (i & 1) ? unpack_hi<kHalf>(w[i >> 1]) : unpack_lo<kHalf>(w[i >> 1]);
      if (col + i < p.V) mc = max_nan(mc, x * kLog2e);
    }
  }
  const float mn = max_nan(m, mc);
  if (mn != -INFINITY) {
    float a[4] = {(m == -INFINITY) ? 0.f : s * ex2_approx(m - mn), 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float lo = unpack_lo<kHalf>(w[i]), hi = unpack_hi<kHalf>(w[i]);
      const float elo = ex2_approx(fmaf(lo, kLog2e, -mn)), ehi = ex2_approx(fmaf(hi, kLog2e, -mn));
      a[i & 3] += (full || col + 2 * i < p.V ? elo : 0.f) + (full || col + 2 * i + 1 < p.V ? ehi : 0.f);
    }
    s = (a[0] + a[1]) + (a[2] + a[3]);
  }
  m = mn;
}

// Epilogue EPI_SWIGLU (the gate and up projections of the SwiGLU MLP, W's rows interleaved in blocks
// of 8: gate rows 8b .. 8b + 7, then up rows 8b .. 8b + 7, for feature block b): the warp's 64 columns
// hold 32 features. They are stored (C: g and u in that interleaved order, in the compute dtype, as the
// backward reads them), and a = silu(g) u is computed in fp32 from the rounded g and u (the arithmetic
// of the separate SwiGLU kernel, one rounding) and stored to the second output, 32 features x 32 rows
// through a 64-byte-swizzled box.
template <bool kHalf, int NBOX>
__device__ __forceinline__ void epilogue_swiglu(const GemmParams& p, uint32_t taddr, uint32_t boxes, uint32_t box2,
                                                int lane, int col, int row0, int& nbox) {
  float v[64];
  tmem_ld32(taddr, v);
  tmem_ld32(taddr + 32u, v + 32);
  tmem_wait_ld();
  uint32_t w[32], a2[16];
#pragma unroll
  for (int i = 0; i < 32; ++i) w[i] = pack2<kHalf>(v[2 * i], v[2 * i + 1]);
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    float a[8];
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      const uint32_t gw = w[8 * b + j / 2], uw = w[8 * b + 4 + j / 2];
      const float g0 = unpack_lo<kHalf>(gw), g1 = unpack_hi<kHalf>(gw);
      const float u0 = unpack_lo<kHalf>(uw), u1 = unpack_hi<kHalf>(uw);
      a[j] = g0 * (1.f / (1.f + __expf(-g0))) * u0;
      a[j + 1] = g1 * (1.f / (1.f + __expf(-g1))) * u1;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) a2[4 * b + j] = pack2<kHalf>(a[2 * j], a[2 * j + 1]);
  }
  const uint32_t box = boxes + (uint32_t)(nbox % NBOX) * 4096u;
  if (lane == 0 && nbox >= NBOX) bulk_wait_read0();
  __syncwarp();
  if (!p.skip_c) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      st_shared_v4(box + sw128_off((uint32_t)lane, (uint32_t)q), w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
  }
#pragma unroll
  for (int q = 0; q < 4; ++q)
    st_shared_v4(box2 + sw64_off((uint32_t)lane, (uint32_t)q), a2[4 * q], a2[4 * q + 1], a2[4 * q + 2], a2[4 * q + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (!p.skip_c) tma_store_2d(&p.tm_c, box, col, row0);
    tma_store_2d(&p.tm_c2, box2, col / 2, row0);
    bulk_commit();
  }
  ++nbox;
}

template <int EPI, int OUT, bool kHalf, bool A_MN, bool B_MN, bool kWide>
__global__ void __launch_bounds__(Cfg<kWide>::NTHREADS, 1) gemm_pair_kernel(const __grid_constant__ GemmParams p) {
  using C = Cfg<kWide, EPI>;
  constexpr int NST = C::NST, BN = C::BN, NBUF = C::NBUF, NHALF = C::NHALF, NBOX = C::NBOX, NEPI = C::NEPI;
  constexpr int CW = C::CW;
  constexpr int WP = NEPI, WM = NEPI + 1;                  // producer and UMMA warps
  extern __shared__ uint8_t smem_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + C::OFF_BAR + C::TMEM_SLOT);
#define BAR(i) (bar0 + 8u * (uint32_t)(i))
  if (tid == 0) {
    for (int s = 0; s < NST; ++s) { mbar_init(BAR(C::B_FULL + s), 1); mbar_init(BAR(C::B_EMPTY + s), 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(BAR(C::B_ACCF + b), 1); mbar_init(BAR(C::B_ACCE + b), 2 * NEPI); }
    if constexpr (EPI == EPI_LCE)
      for (int b = 0; b < 8; ++b) mbar_init(BAR(C::B_REC + b), NEPI / 4 - 1);
    fence_barrier_init();
  }
  if (warp == WM) { tmem_alloc_pair(smem_u32(tmem_slot), TMEM_COLS); tmem_relinquish_pair(); }
  if (warp == WP && lane == 0) {
    tma_prefetch_desc(&p.tm_a); tma_prefetch_desc(&p.tm_b); tma_prefetch_desc(&p.tm_c);
    if constexpr (EPI == EPI_SWIGLU) tma_prefetch_desc(&p.tm_c2);
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();          // the leader's barriers exist before the peer's loads and arrivals reach them
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  // work item w: tile w / k_split, K slice w % k_split (k-blocks [slice kb_split, + kb_split) of nk)
  const int ns = p.k_split;
  const int nwork = p.num_m * p.num_n * ns;
  const int cid = (int)blockIdx.x >> 1, ncl = (int)gridDim.x >> 1;
  const int nk = (p.K + BK - 1) / BK;
  auto kblocks = [&](int w, int& kb0) {
    kb0 = (w % ns) * p.kb_split;
    const int kb1 = kb0 + p.kb_split < nk ? kb0 + p.kb_split : nk;
    return kb1 - kb0;
  };

  if (warp == WP) {
    // ---------------------------------------------------------------- TMA producer (both CTAs)
    if (lane == 0) {
      const uint32_t full_leader = map_rank(BAR(C::B_FULL), 0);
      int it = 0;
      bool ok = true;
      for (int w = cid; ok && w < nwork; w += ncl) {
        int mb, nb, kb0;
        tile_coords(p, w / ns, mb, nb);
        const int nl = kblocks(w, kb0);
        const int kb1 = kb0 + nl;
        // this CTA's rows: A rows m0 .. m0 + 127; B rows n0 + 256 h .. + 127 for each half h
        const int m0 = mb * 2 * BMC + (int)rank * BMC, n0 = nb * BN + (int)rank * 128;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % NST;
          if (it >= NST && !mbar_wait<true>(BAR(C::B_EMPTY + s), ((it / NST) - 1) & 1, p.status)) { ok = false; break; }
          if (leader) mbar_expect_tx(BAR(C::B_FULL + s), 2 * C::SZ_STAGE);
          const uint32_t st = sbase + (uint32_t)s * C::SZ_STAGE, fb = full_leader + 8u * (uint32_t)s;
          if constexpr (A_MN) {
            tma_load_2d_pair(st, &p.tm_a, fb, m0, kb * BK);
            tma_load_2d_pair(st + SZ_HALF / 2, &p.tm_a, fb, m0 + 64, kb * BK);
          } else {
            tma_load_2d_pair(st, &p.tm_a, fb, kb * BK, m0);
          }
#pragma unroll
          for (int h = 0; h < NHALF; ++h) {
            const uint32_t sb = st + SZ_HALF * (1 + h);
            if constexpr (B_MN) {
              tma_load_2d_pair(sb, &p.tm_b, fb, n0 + 256 * h, kb * BK);
              tma_load_2d_pair(sb + SZ_HALF / 2, &p.tm_b, fb, n0 + 256 * h + 64, kb * BK);
            } else {
              tma_load_2d_pair(sb, &p.tm_b, fb, kb * BK, n0 + 256 * h);
            }
          }
        }
      }
      // Tail: the leader's last UMMA commits still arrive on this CTA's empty barriers; see them land
      // before the CTA can leave.
      for (int i = it - NST < 0 ? 0 : it - NST; ok && i < it; ++i)
        ok = mbar_wait<true>(BAR(C::B_EMPTY + i % NST), (i / NST) & 1, p.status);
    }
  } else if (warp == WM) {
    // ---------------------------------------------------------------- UMMA issuer (leader CTA)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = make_idesc(2 * BMC, 256, kHalf ? 0 : 1, A_MN ? 1 : 0, B_MN ? 1 : 0);
      // The four K = 16 UMMAs of one stage into one 256-column part of the accumulator.
      auto issue = [&](uint32_t acc, int s, int h, bool first) {
        const uint32_t sa = sbase + (uint32_t)s * C::SZ_STAGE, sb = sa + SZ_HALF * (1 + h);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k) {
          const uint64_t da = A_MN ? make_sdesc(sa + k * 2048, 8192, 1024, SW_128B) : make_sdesc(sa + k * 32, 16, 1024, SW_128B);
          const uint64_t db = B_MN ? make_sdesc(sb + k * 2048, 8192, 1024, SW_128B) : make_sdesc(sb + k * 32, 16, 1024, SW_128B);
          umma_ss_pair(acc, da, db, idesc, (first && k == 0) ? 0u : 1u);
        }
      };
      auto wait_full = [&](int i) {
        const bool r = mbar_wait<true>(BAR(C::B_FULL + i % NST), (i / NST) & 1, p.status);
        tc_fence_after();
        return r;
      };
      auto wait_drained = [&](int part, int round) {
        const bool r = round == 0 || mbar_wait<true>(BAR(C::B_ACCE + part), (round - 1) & 1, p.status);
        tc_fence_after();
        return r;
      };
      int it = 0, tl = 0;
      bool ok = true;
      for (int w = cid; ok && w < nwork; w += ncl, ++tl) {
        const int buf = tl % NBUF, round = tl / NBUF;
        const uint32_t acc = tbase + (uint32_t)(buf * NHALF * 256);
        int kb0;
        const int nloc = kblocks(w, kb0);
        int kb = 0;
        if constexpr (kWide) {
          // Half 0 runs ahead over the stages already loaded while the epilogue still drains half 1 of
          // the previous tile; the stages are released once half 1 has read them too.
          const int S = nloc < NST ? nloc : NST;
          ok = wait_drained(0, round);
          for (int j = 0; ok && j < S; ++j) {
            if (!(ok = wait_full(it + j))) break;
            issue(acc, (it + j) % NST, 0, j == 0);
          }
          ok = ok && wait_drained(1, round);
          for (int j = 0; ok && j < S; ++j) {
            issue(acc + 256, (it + j) % NST, 1, j == 0);
            umma_commit_pair(BAR(C::B_EMPTY + (it + j) % NST));
          }
          it += S;
          kb = S;
        } else {
          ok = wait_drained(buf, round);
        }
        for (; ok && kb < nloc; ++kb, ++it) {
          if (!(ok = wait_full(it))) break;
#pragma unroll
          for (int h = 0; h < NHALF; ++h) issue(acc + 256 * h, it % NST, h, kb == 0);
          umma_commit_pair(BAR(C::B_EMPTY + it % NST));
        }
        if (!ok) break;
        umma_commit_pair(BAR(C::B_ACCF + buf));
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue warps (both CTAs)
    constexpr int COLS = (EPI == EPI_STORE && OUT == GEMM_OUT_F32) ? 32 : 64;   // columns per 128-byte box row
    static_assert(EPI == EPI_STORE || CW == 64, "the linear-CE and SwiGLU epilogues take one 64-column box per warp");
    const int quarter = warp & 3, cgroup = warp >> 2;
    const uint32_t acce_leader = map_rank(BAR(C::B_ACCE), 0);
    const uint32_t boxes = sbase + C::OFF_EPI + (uint32_t)warp * NBOX * C::SZ_EPI;
    int tl = 0, nbox = 0;
    for (int w = cid; w < nwork; w += ncl, ++tl) {
      int mb, nb;
      const int t = w / ns, slice = w % ns;
      tile_coords(p, t, mb, nb);
      const int buf = tl % NBUF;
      const int wslot = (t * 2 + (int)rank) * NEPI + warp;      // this warp's rows and columns of tile t
      const int row0 = mb * 2 * BMC + (int)rank * BMC + quarter * 32;
      int64_t lab = -1;
      if constexpr (EPI == EPI_LCE) {
        if (row0 + lane < p.M) lab = p.labels[row0 + lane];   // in flight during the wait below
      }
      // the epilogue warps sleep through the main loop (suspend-time hint), leaving issue slots to the
      // producer and UMMA threads on their sub-partitions
      if (!warp_wait<true>(BAR(C::B_ACCF + buf), (tl / NBUF) & 1, p.status)) break;
      tc_fence_after();
      const uint32_t tlane = tbase + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
      for (int h = 0; h < NHALF; ++h) {
        // columns 256 h + 128 r + j of the tile come from CTA r's B rows n0 + 256 h + j; this warp
        // takes the CW columns from 256 h + CW cgroup
        const int cbase = nb * BN + 256 * h + CW * cgroup;
        const uint32_t tcol = (uint32_t)((buf * NHALF + h) * 256 + CW * cgroup);
        if constexpr (EPI == EPI_SWIGLU) {
          static_assert(CW == 64, "the SwiGLU epilogue takes one 64-column box per warp");
          if (row0 < p.M && cbase < p.N)
            epilogue_swiglu<kHalf, NBOX>(p, tlane + tcol, boxes, sbase + C::OFF_EPI2 + (uint32_t)warp * C::SZ_EPI2, lane,
                                         cbase, row0, nbox);
        } else if constexpr (EPI == EPI_LCE) {
          // One (max, sum) record per row and 256-column tile: the column groups 1..3 of a row quarter
          // leave theirs in the first two of their own accumulator columns (read already, and not
          // rewritten before this tile's accumulator-empty barrier, which the merging warp arrives on
          // last), and column group 0 merges the four in column order.
          static_assert(NHALF == 1 && CW == 64, "the linear-CE epilogue runs on the narrow tile");
          const int row = row0 + lane;
          float m = -INFINITY, sum = 0.f, tgt = 0.f;
          bool has_tgt = false;
          if (row0 < p.M && cbase < p.N)
            epilogue_lce<kHalf, NBOX>(p, tlane + tcol, boxes, lane, cbase, row0, nbox, lab, m, sum, tgt, has_tgt);
          if (has_tgt && row < p.M) p.tgt[row] = tgt;
          const uint32_t rec = BAR(C::B_REC + 2 * quarter + (tl & 1));
          if (cgroup > 0) {
            tmem_st2(tlane + tcol, make_float2(m, sum));
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(rec);
          } else {
            // (a wait that runs out has set the status word's timeout bit; the record is then this
            // group's alone and the call fails on the host)
            const bool got = warp_wait(rec, (tl >> 1) & 1, p.status);
            tc_fence_after();
            float2 q[NEPI / 4 - 1];
#pragma unroll
            for (int c = 1; c < NEPI / 4; ++c) tmem_ld2(tlane + tcol + (uint32_t)(CW * c), q[c - 1]);
            tmem_wait_ld();
#pragma unroll
            for (int c = 1; c < NEPI / 4; ++c) {
              if (!got) break;
              const float mc = q[c - 1].x, sc = q[c - 1].y;
              const float mn = max_nan(m, mc);
              if (mn != -INFINITY)
                sum = (m == -INFINITY ? 0.f : sum * ex2_approx(m - mn)) + (mc == -INFINITY ? 0.f : sc * ex2_approx(mc - mn));
              m = mn;
            }
            if (row < p.M) p.part[(int64_t)row * p.n_part + nb * (BN / 256)] = make_float2(m, sum);
          }
        } else {
          bool split_done = false;
          if constexpr (OUT == GEMM_OUT_F32 && !kWide) {
            if (ns > 1) {
              // a K slice: partial to the workspace; the last slice to arrive sums them and stores C
              float v[64];
              tmem_ld32(tlane + tcol, v);
              tmem_ld32(tlane + tcol + 32u, v + 32);
              tmem_wait_ld();
              float* slots = p.partials + (size_t)wslot * ns * 2048;
              write_partial(slots + (size_t)slice * 2048, v, lane);
              if (arrive_last(p.sema + wslot, ns, lane)) {
#pragma unroll
                for (int i = 0; i < 64; ++i) v[i] = 0.f;
                for (int k = 0; k < ns; ++k) {
                  const float* sl = slots + (size_t)k * 2048;
#pragma unroll
                  for (int i = 0; i < 64; ++i) v[i] += __ldcg(sl + i * 32 + lane);
                }
#pragma unroll
                for (int c0 = 0; c0 < 64; c0 += 32)
                  if (row0 < p.M && cbase + c0 < p.N)
                    epilogue_store_values<NBOX>(p, v + c0, boxes, lane, cbase + c0, row0, nbox, p.accumulate != 0,
                                                p.bias != nullptr);
              }
              split_done = true;
            }
          }
          if (!split_done) {
#pragma unroll 1
            for (int c0 = 0; c0 < CW; c0 += COLS)
              if (row0 < p.M && cbase + c0 < p.N)
                epilogue_store<OUT, NBOX>(p, tlane + tcol + (uint32_t)c0, boxes, lane, cbase + c0, row0, nbox,
                                          OUT == GEMM_OUT_F32 && p.accumulate, p.bias != nullptr);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(acce_leader + 8u * (uint32_t)(buf * NHALF + h));
      }
    }
    if (lane == 0) bulk_wait_all();          // the stores have landed before the kernel ends
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();          // neither CTA frees its memory while the pair's UMMAs may still use it
  if (warp == WM) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, TMEM_COLS);
  }
#undef BAR
}

}  // namespace gemm

// CTA pairs of the GEMM kernels that can be resident at once on the current device (one CTA per SM,
// clusters of two; not every GPC holds an even number of SMs), asked once per device.
static int resident_pairs(int num_sms) {
  static int cache[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
  using namespace gemm;
  auto kernel = gemm_pair_kernel<EPI_STORE, GEMM_OUT_F32, false, false, false, false>;
  int pairs = 0;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<false>::SMEM_BYTES) ==
      cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2; attr[0].val.clusterDim.y = 1; attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(Cfg<false>::NTHREADS);
    cfg.gridDim = dim3(2 * (num_sms / 2));
    cfg.dynamicSmemBytes = Cfg<false>::SMEM_BYTES;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&pairs, kernel, &cfg) != cudaSuccess) pairs = 0;
  }
  cudaGetLastError();
  if (pairs < 1) pairs = num_sms / 2;
  if (dev >= 0 && dev < 64) cache[dev] = pairs;
  return pairs;
}

// One launch of a persistent grid: min(resident pairs, work items) clusters of two CTAs.
template <int EPI, int OUT, bool H, bool W>
static cudaError_t launch_majors(const GemmParams& p, int a_mn, int b_mn, int pairs, cudaStream_t st) {
  using namespace gemm;
  auto run = [&](auto kernel) {
    const uint32_t smem = Cfg<W, EPI>::SMEM_BYTES;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    const int nwork = p.num_m * p.num_n * p.k_split;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2; attr[0].val.clusterDim.y = 1; attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(Cfg<W, EPI>::NTHREADS);
    cfg.gridDim = dim3(2 * (pairs < nwork ? pairs : nwork));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, p);
  };
  if constexpr (EPI != EPI_STORE) {
    return run(gemm_pair_kernel<EPI, OUT, H, false, false, W>);     // X and W rows are K-major
  } else {
    if (a_mn && b_mn) return run(gemm_pair_kernel<EPI, OUT, H, true, true, W>);
    if (a_mn) return run(gemm_pair_kernel<EPI, OUT, H, true, false, W>);
    if (b_mn) return run(gemm_pair_kernel<EPI, OUT, H, false, true, W>);
    return run(gemm_pair_kernel<EPI, OUT, H, false, false, W>);
  }
}

// Tile shape and K split from a cost model in units of one narrow tile's 64-wide K block (one round of
// work items takes its longest item's K blocks plus ~3 of pipeline fill and epilogue; a wide tile's K
// block costs 1.8 narrow ones: it moves a quarter fewer operand bytes). A split (narrow tiles, fp32
// output, at most 4 rounds of work items) is taken only where the tiles fill less than one wave of CTA
// pairs and it saves at least 10 %.
static void choose_shape(int64_t M, int64_t N, int64_t K, int out, int pairs, int tile, bool can_split, int& wide,
                         int& ns) {
  const int nk = (int)((K + 63) / 64);
  const int num_m = (int)((M + 255) / 256);
  wide = tile > 0 ? 1 : 0;
  ns = 1;
  if (tile >= 0) return;
  double best = 1e300;
  for (int w = 0; w < 2; ++w) {
    const int nt = num_m * (int)((N + (w ? 511 : 255)) / (w ? 512 : 256));
    const double unit = w ? 1.8 : 1.0;
    const double base = (double)((nt + pairs - 1) / pairs) * (nk + 3.0) * unit;
    if (base < best) { best = base; wide = w; ns = 1; }
    if (w || out != GEMM_OUT_F32 || !can_split || nt >= pairs) continue;
    for (int k = 2; k <= 16 && nk / k >= 4 && nt * k <= 4 * pairs; ++k) {
      const int kbs = (nk + k - 1) / k;
      if ((nk + kbs - 1) / kbs != k) continue;           // the same split as a smaller k
      const double cost = (double)((nt * k + pairs - 1) / pairs) * (kbs + 3.0) * unit;
      if (cost < 0.9 * base && cost < best) { best = cost; wide = w; ns = k; }
    }
  }
}

// Workspace of a split: counters (one per epilogue warp of each CTA of each tile), then the slots.
static int64_t split_bytes(int64_t M, int64_t N, int ns) {
  const int64_t nt = ((M + 255) / 256) * ((N + 255) / 256);
  const int64_t warps = nt * 2 * gemm::Cfg<false>::NEPI;
  const int64_t head = ((warps * 4 + 255) / 256) * 256;
  return ns > 1 ? head + warps * ns * 2048 * 4 : 0;
}

int64_t gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int out, int num_sms) {
  int wide, ns;
  choose_shape(M, N, K, out, resident_pairs(num_sms), -1, true, wide, ns);
  return split_bytes(M, N, ns);
}

template <int OUT, bool H>
static cudaError_t launch_shape(const GemmParams& p, int a_mn, int b_mn, int wide, int pairs, cudaStream_t st) {
  return wide ? launch_majors<EPI_STORE, OUT, H, true>(p, a_mn, b_mn, pairs, st)
              : launch_majors<EPI_STORE, OUT, H, false>(p, a_mn, b_mn, pairs, st);
}

cudaError_t launch_gemm(const GemmParams& p0, int in_dtype, int a_mn, int b_mn, int out, int tile, int num_sms,
                        cudaStream_t st) {
  GemmParams p = p0;
  const int pairs = resident_pairs(num_sms);
  int wide, ns;
  choose_shape(p.M, p.N, p.K, out, pairs, tile, true, wide, ns);
  if (ns > 1 && (p.sema == nullptr || p.ws_bytes < split_bytes(p.M, p.N, ns))) ns = 1;
  const int nk = (p.K + 63) / 64;
  p.num_n = (p.N + (wide ? 511 : 255)) / (wide ? 512 : 256);
  p.k_split = ns;
  p.kb_split = (nk + ns - 1) / ns;
  if (ns > 1) {
    const int64_t warps = (int64_t)p.num_m * p.num_n * 2 * gemm::Cfg<false>::NEPI;
    p.partials = reinterpret_cast<float*>(reinterpret_cast<char*>(p.sema) + ((warps * 4 + 255) / 256) * 256);
    cudaError_t e = cudaMemsetAsync(p.sema, 0, (size_t)warps * 4, st);
    if (e != cudaSuccess) return e;
  }
  const bool h = in_dtype == 1;
  if (out == GEMM_OUT_F32) return h ? launch_shape<GEMM_OUT_F32, true>(p, a_mn, b_mn, wide, pairs, st)
                                    : launch_shape<GEMM_OUT_F32, false>(p, a_mn, b_mn, wide, pairs, st);
  if (out == GEMM_OUT_BF16) return h ? launch_shape<GEMM_OUT_BF16, true>(p, a_mn, b_mn, wide, pairs, st)
                                     : launch_shape<GEMM_OUT_BF16, false>(p, a_mn, b_mn, wide, pairs, st);
  return h ? launch_shape<GEMM_OUT_F16, true>(p, a_mn, b_mn, wide, pairs, st)
           : launch_shape<GEMM_OUT_F16, false>(p, a_mn, b_mn, wide, pairs, st);
}

cudaError_t launch_gemm_swiglu(const GemmParams& p0, int in_dtype, int num_sms, cudaStream_t st) {
  GemmParams p = p0;
  p.num_n = (p.N + 255) / 256;
  p.k_split = 1;
  p.kb_split = (p.K + 63) / 64;
  const int pairs = resident_pairs(num_sms);
  return in_dtype == 1 ? launch_majors<EPI_SWIGLU, GEMM_OUT_F16, true, false>(p, 0, 0, pairs, st)
                       : launch_majors<EPI_SWIGLU, GEMM_OUT_BF16, false, false>(p, 0, 0, pairs, st);
}

cudaError_t launch_lce_logits_gemm(const GemmParams& p0, int in_dtype, int num_sms, cudaStream_t st) {
  GemmParams p = p0;
  p.num_n = (p.N + 255) / 256;
  p.k_split = 1;
  p.kb_split = (p.K + 63) / 64;
  const int pairs = resident_pairs(num_sms);
  return in_dtype == 1 ? launch_majors<EPI_LCE, GEMM_OUT_F16, true, false>(p, 0, 0, pairs, st)
                       : launch_majors<EPI_LCE, GEMM_OUT_BF16, false, false>(p, 0, 0, pairs, st);
}

}  // namespace sisa
