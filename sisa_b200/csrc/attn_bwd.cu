// attn_bwd.cu - exact-delta SISA attention backward on Blackwell tensor cores.
//
// Reference semantics: src/sisa/kernels/attention.py:28-78 (numerics (D), (E)), 300-491 (_bwd_dq),
// 495-663 (_bwd_dkv) and 781-783 (fp64 d lambda). Two kernels, no atomics on data (deterministic):
//
//  dq kernel (query-tile owner, 128 rows): recomputes S = QK^T, U = CB~^T, dP = dO V^T per 64-key tile,
//    P = 2^(x - lse), the FlashAttention-standard dS^ = P (dP - delta'') with delta'' = do.o'' (the
//    self-normalised fp32 forward output), and accumulates dQ += dS^ K and dC += (dS^ * colf mid) B~ in
//    TMEM. It also accumulates the row sums of the exact-delta scheme (Z, D, P_tt, dP_tt, the
//    u-weighted sums) and finishes every row: T^, the delta-free diagonal dS_tt, the row parts of
//    dg, dF and d lambda, and the per-row statistics {-lse, -delta, -(T^-delta), dS_tt} read by the dkv
//    kernel (negated so that kernel adds them).
//  dkv kernel (key-tile owner, 128 rows): recomputes S^T, U^T, dP^T per 64-query tile, uses
//    dS = dS^' - P'(T^ - delta) for dK and the column sums of dg and dF, dS^' for dB (the same delta as
//    dC, so the Phi_i - Phi_j cancellation of d theta holds), and the dq kernel's dS_tt on the diagonal.
//
// Both kernels: 16 compute warps (four warpgroups splitting each tile's 64 columns 16/16/16/16; thread =
// TMEM lane = owned row, four compute warps per SM sub-partition), one TMA producer warp and two UMMA
// warps. Per tile the compute warps pull S, U, dP into registers and release TMEM at once, so the next
// tile's GEMMs overlap their math; the gradient GEMMs read the bf16 operands (dS, P^T, ...) the compute
// warps stored into tensor memory (A from TMEM), so the tensor core fetches only the B tiles from
// shared memory.
//
// Waits: the UMMA issuers and the TMA thread sleep on their mbarriers (suspend-time hint) so that
// they do not spin through issue slots the compute warps need; the compute warps poll, because a
// suspended warp resumes later and their hand-offs are on the critical path (measured: issuers
// sleeping -1.0 % attn_bwd, compute warps sleeping +1.1 %).
//
// UMMA issue is split over two single-thread issuers on different SM sub-partitions: one issues the
// score GEMMs (S, U, dP) and waits only on the stage-full and scores-consumed barriers, the other
// issues the gradient GEMMs and waits only on the operands-full barrier. An mbarrier wait costs the
// issuing thread some 150 cycles even when the phase has already completed, and a compute warp that can
// issue every cycle starves a same-sub-partition issuer several-fold, so one issuer doing both chains
// serialises ~6 waits per tile; two issuers keep the tensor pipe fed while either one waits. A tile's
// score GEMMs have completed before its operands exist, so the gradient issuer's commit alone releases
// the stage.
#include <cuda_runtime.h>
#include <cooperative_groups.h>
#include <type_traits>

#include "attn_common.cuh"
#include "attn.h"

namespace sisa {
namespace bwd {

constexpr int NST = 4;           // key (dq) / query (dkv) tile stages
constexpr int NWG = 4;           // compute warpgroups; each owns 64 / NWG columns of every tile
constexpr int NCOL = 64 / NWG;   // 16
constexpr int NCW = 4 * NWG;     // compute warps
constexpr int NTHREADS = 32 * NCW + 96;    // + one TMA warp + two UMMA issuer warps
constexpr int WARP_TMA = NCW, WARP_MMA = NCW + 1, WARP_GRAD = NCW + 2;   // sub-partitions 0, 1, 2
constexpr int NCT = 32 * NCW;    // compute threads
// barrier area: up to 32 mbarriers, then the TMEM address slot
constexpr uint32_t kTmemSlot = 256, kBarBytes = 512;

// ----------------------------------------------------------------------------- dq kernel layout
namespace dqk {
constexpr uint32_t SZ_Q = 128 * 128, SZ_DO = 128 * 128, SZ_C = 128 * 64;
constexpr uint32_t SZ_K = 64 * 128, SZ_V = 64 * 128, SZ_B = 64 * 64, SZ_POS = 64 * 16;
constexpr uint32_t SZ_STAGE = SZ_K + SZ_V + SZ_B + SZ_POS;   // 21504
constexpr uint32_t OFF_Q = 0, OFF_DO = OFF_Q + SZ_Q, OFF_C = OFF_DO + SZ_DO, OFF_ST = OFF_C + SZ_C;
constexpr uint32_t OFF_RED = OFF_ST + NST * SZ_STAGE;          // [8 values][NWG][128 rows] floats
// o'' of the tile for delta'' (two 128-byte-swizzled boxes of 32 fp32 columns; o itself, when the
// forward kept no o'', is one 64-column low-precision box)
constexpr uint32_t SZ_OB = 128 * 128, OFF_O = OFF_RED + 128 * NWG * 8 * 4;
// the tile's own key and B~ rows (k_t, b_t) for the diagonal terms of the epilogue
constexpr uint32_t OFF_KR = OFF_O + 2 * SZ_OB, OFF_BR = OFF_KR + 128 * 128;
constexpr uint32_t OFF_BAR = OFF_BR + 128 * 64;
constexpr uint32_t SMEM_BYTES = OFF_BAR + kBarBytes + 1024;
// The epilogue stages dq (low precision, 128-byte rows) in the Q region and dc (fp32, 128-byte rows)
// in the dO region for bulk-tensor stores; both are free once the last gradient UMMA has completed.
// TMEM: S, U, dP per tile; dQ, dC_off, dC_diag accumulators; the bf16 operands dS and dS*cf of the
// gradient UMMAs (two buffers of 2 x 32 columns, written by the compute warps, read as A from TMEM)
constexpr int COL_S = 0, COL_U = 64, COL_DP = 128, COL_DQ = 192, COL_DCO = 256, COL_DCD = 288, COL_OPS = 320;
constexpr int B_KVF = 0, B_KVE = NST, B_Q = 2 * NST, B_SUF = B_Q + 1, B_SUE = B_Q + 2, B_OPF = B_Q + 3,
              B_OPE = B_Q + 5, B_ACC = B_Q + 7, B_O = B_Q + 8, B_KR = B_Q + 9;
static_assert(OFF_ST % 1024 == 0 && OFF_O % 1024 == 0 && OFF_KR % 1024 == 0 && OFF_BR % 1024 == 0 &&
                  SZ_STAGE % 1024 == 0, "swizzled tiles need 1024-byte alignment");
static_assert(SMEM_BYTES <= 232448, "shared memory per block");
static_assert(B_KR * 8 < kTmemSlot, "barriers end below the TMEM slot");
}  // namespace dqk

// ----------------------------------------------------------------------------- dkv kernel layout
namespace dkv {
constexpr uint32_t SZ_K = 128 * 128, SZ_V = 128 * 128, SZ_B = 128 * 64;
constexpr uint32_t SZ_Q = 64 * 128, SZ_DO = 64 * 128, SZ_C = 64 * 64, SZ_POS = 64 * 16, SZ_RST = 64 * 16;
constexpr uint32_t SZ_STAGE = SZ_Q + SZ_DO + SZ_C + SZ_POS + SZ_RST;   // 22528
constexpr uint32_t OFF_K = 0, OFF_V = OFF_K + SZ_K, OFF_B = OFF_V + SZ_V, OFF_ST = OFF_B + SZ_B;
constexpr uint32_t OFF_RED = OFF_ST + NST * SZ_STAGE;                  // [2 values][NWG][128 rows] floats
constexpr uint32_t SZ_DSB = 128 * 128;                                 // (dS^' rq)^T operand: 128 keys x 64 queries
constexpr uint32_t OFF_DSB = OFF_RED + 128 * NWG * 2 * 4;              // two buffers, K-major, 128-byte swizzle
constexpr uint32_t OFF_BAR = OFF_DSB + 2 * SZ_DSB;
constexpr uint32_t SMEM_BYTES = OFF_BAR + kBarBytes + 1024;
// TMEM: S^T, U^T, dP^T per tile; dV, dK, dB_diag, dB_off accumulators; the bf16 operands P^T and dS^T
// (two buffers of 2 x 32 columns, A operands read from TMEM). The third operand, (dS^' rq)^T, goes
// through shared memory (two buffers), so the compute warps store tile n while the gradient UMMAs of
// tile n-1 still read theirs.
constexpr int COL_S = 0, COL_U = 64, COL_DP = 128, COL_DV = 192, COL_DK = 256, COL_DBD = 320, COL_DBO = 352,
              COL_OPS = 384;
static_assert(OFF_DSB % 1024 == 0, "swizzled operand tiles need 1024-byte alignment");
constexpr int B_KVF = 0, B_KVE = NST, B_K = 2 * NST, B_SUF = B_K + 1, B_SUE = B_K + 2, B_OPF = B_K + 3,
              B_OPE = B_K + 5, B_ACC = B_K + 7;
static_assert(B_ACC * 8 < kTmemSlot, "barriers end below the TMEM slot");
static_assert(OFF_ST % 1024 == 0 && SZ_STAGE % 1024 == 0, "alignment");
}  // namespace dkv

constexpr uint32_t TMEM_COLS = 512;

// Store this thread's NCOL low-precision operand values (NCOL/2 packed pairs) into its lane of a
// 32-column TMEM operand tile: warpgroup wg owns columns [wg * NCOL/2, (wg + 1) * NCOL/2).
__device__ __forceinline__ void st_op_tmem(uint32_t tbase, int quarter, int col, int wg, const uint32_t* w) {
  static_assert(NCOL == 16, "one x8 store per operand");
  tmem_st8(tmem_addr(tbase, quarter, col + wg * (NCOL / 2)), w);
}

template <bool kHalf>
__device__ __forceinline__ float ld_lp_g(const char* base, int64_t i) {
  if constexpr (kHalf) return __half2float(reinterpret_cast<const __half*>(base)[i]);
  else return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
}

// =============================================================================================
// dq kernel
// =============================================================================================
template <bool kHalf>
__global__ void __launch_bounds__(NTHREADS, 1) attn_bwd_dq_kernel(const __grid_constant__ BwdParams p) {
  using namespace dqk;
  extern __shared__ uint8_t smem_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int bh, rank;
  tile_order(p.ntq128, p.B * p.H, bh, rank);
  const int qt = p.ntq128 - 1 - rank;                // heaviest query tiles first
  const int b = bh / p.H, h = bh % p.H;
  const int L = p.L;
  const int m0 = qt * 128;
  const int ndiag = (m0 + 64 < L) ? 2 : 1;
  const int ntiles = ndiag + m0 / 64;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);
  const uint32_t bar0 = sbase + OFF_BAR;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_BAR + kTmemSlot);
#define BAR(i) (bar0 + 8u * (uint32_t)(i))
  auto key0 = [&](int n) { return n < ndiag ? m0 + n * 64 : (n - ndiag) * 64; };
  auto stage_addr = [&](int s) { return sbase + OFF_ST + (uint32_t)s * SZ_STAGE; };
  // The TMA thread initialises the barriers and issues the resident tiles and the first NST key tiles
  // before the block-wide sync (which also waits for the TMEM allocation): nothing else touches those
  // barriers or buffers until after it, and the loads' latency starts that much earlier.
  const int npre = ntiles < NST ? ntiles : NST;
  auto issue_stage = [&](int n) {
    const int s = n % NST;
    const int j0 = key0(n);
    const uint32_t st = stage_addr(s);
    mbar_expect_tx(BAR(B_KVF + s), SZ_STAGE);
    tma_load_4d(st, &p.tm_k64, BAR(B_KVF + s), 0, j0, h, b);
    tma_load_4d(st + SZ_K, &p.tm_v64, BAR(B_KVF + s), 0, j0, h, b);
    tma_load_4d(st + SZ_K + SZ_V, &p.tm_b64, BAR(B_KVF + s), 0, j0, h, b);
    tma_load_3d(st + SZ_K + SZ_V + SZ_B, &p.tm_pos, BAR(B_KVF + s), j0, 0, bh);
    if (n == 0) {
      // o'' for delta'', behind the first key tile (the score GEMMs need that first)
      if (p.o32) {
        mbar_expect_tx(BAR(B_O), 2 * SZ_OB);
        tma_load_3d(sbase + OFF_O, &p.tm_o, BAR(B_O), 0, m0, bh);
        tma_load_3d(sbase + OFF_O + SZ_OB, &p.tm_o, BAR(B_O), 32, m0, bh);
      } else {
        mbar_expect_tx(BAR(B_O), SZ_OB);
        tma_load_4d(sbase + OFF_O, &p.tm_o, BAR(B_O), 0, m0, h, b);
      }
    }
  };
  if (warp == WARP_TMA && lane == 0) {
    for (int s = 0; s < NST; ++s) { mbar_init(BAR(B_KVF + s), 1); mbar_init(BAR(B_KVE + s), 1); }
    mbar_init(BAR(B_Q), 1);
    mbar_init(BAR(B_SUF), 1);
    mbar_init(BAR(B_SUE), NCT);
    for (int i = 0; i < 2; ++i) { mbar_init(BAR(B_OPF + i), NCT); mbar_init(BAR(B_OPE + i), 1); }
    mbar_init(BAR(B_ACC), 1);
    mbar_init(BAR(B_O), 1);
    mbar_init(BAR(B_KR), 1);
    fence_barrier_init();
    fence_proxy_async_smem();
    mbar_expect_tx(BAR(B_Q), SZ_Q + SZ_DO + SZ_C);
    tma_load_4d(sbase + OFF_Q, &p.tm_q128, BAR(B_Q), 0, m0, h, b);
    tma_load_4d(sbase + OFF_DO, &p.tm_do128, BAR(B_Q), 0, m0, h, b);
    tma_load_4d(sbase + OFF_C, &p.tm_c128, BAR(B_Q), 0, m0, h, b);
    for (int n = 0; n < npre; ++n) issue_stage(n);
  }
  if (warp == WARP_MMA) { tmem_alloc(smem_u32(tmem_slot), TMEM_COLS); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == WARP_TMA) {
    if (lane == 0) {
      for (int n = npre; n < ntiles; ++n) {
        const int s = n % NST;
        if (!mbar_wait<true>(BAR(B_KVE + s), ((n / NST) - 1) & 1, p.status)) break;
        issue_stage(n);
      }
      // the tile's own key and B~ rows, needed only by the epilogue
      mbar_expect_tx(BAR(B_KR), 128 * 128 + 128 * 64);
      tma_load_4d(sbase + OFF_KR, &p.tm_k128, BAR(B_KR), 0, m0, h, b);
      tma_load_4d(sbase + OFF_BR, &p.tm_b128, BAR(B_KR), 0, m0, h, b);
    }
  } else if (warp == WARP_MMA) {
    // score GEMMs S = Q K^T, U = C B~^T, dP = dO V^T of every key tile
    if (lane == 0) {
      constexpr uint32_t fmt = kHalf ? 0 : 1;
      constexpr uint32_t id_s = make_idesc(128, 64, fmt, 0, 0);
      const uint32_t sQ = sbase + OFF_Q, sDO = sbase + OFF_DO, sC = sbase + OFF_C;
      bool ok = mbar_wait<true>(BAR(B_Q), 0, p.status);
      for (int n = 0; ok && n < ntiles; ++n) {
        const int s = n % NST;
        if (!mbar_wait<true>(BAR(B_KVF + s), (n / NST) & 1, p.status)) { ok = false; break; }
        if (n > 0 && !mbar_wait<true>(BAR(B_SUE), (n - 1) & 1, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t st = stage_addr(s);
#pragma unroll
        for (int k = 0; k < 4; ++k) umma_ss(tbase + COL_S, desc_k128(sQ + k * 32), desc_k128(st + k * 32), id_s, k > 0);
#pragma unroll
        for (int k = 0; k < 2; ++k)
          umma_ss(tbase + COL_U, desc_k64(sC + k * 32), desc_k64(st + SZ_K + SZ_V + k * 32), id_s, k > 0);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_ss(tbase + COL_DP, desc_k128(sDO + k * 32), desc_k128(st + SZ_K + k * 32), id_s, k > 0);
        umma_commit(BAR(B_SUF));
      }
    }
  } else if (warp == WARP_GRAD) {
    // gradient GEMMs dQ += dS^ K, dC += (dS^ colf mid) B~ from the operands in TMEM; releases the stage
    if (lane == 0) {
      constexpr uint32_t fmt = kHalf ? 0 : 1;
      constexpr uint32_t id_dq = make_idesc(128, 64, fmt, 0, 1);
      constexpr uint32_t id_dc = make_idesc(128, 32, fmt, 0, 1);
      int ndco = 0, ndcd = 0;   // GEMMs issued into dC_off / dC_diag so far
      for (int m = 0; m < ntiles; ++m) {
        const int buf = m & 1, s = m % NST;
        if (!mbar_wait<true>(BAR(B_OPF + buf), (m >> 1) & 1, p.status)) break;
        tc_fence_after();
        const uint32_t tDS = tbase + COL_OPS + (uint32_t)buf * 64, tDSC = tDS + 32;
        const uint32_t st = stage_addr(s);
        const bool dg = m < ndiag;
        const uint32_t tdc = tbase + (dg ? COL_DCD : COL_DCO);
        int& cnt = dg ? ndcd : ndco;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_ts(tbase + COL_DQ, tDS + k * 8, desc_mn128(st + k * 2048), id_dq, (m > 0 || k > 0));
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_ts(tdc, tDSC + k * 8, desc_mn64(st + SZ_K + SZ_V + k * 1024), id_dc, (cnt > 0 || k > 0));
        ++cnt;
        umma_commit(BAR(B_OPE + buf));
        umma_commit(BAR(B_KVE + s));
      }
      // The accumulator of a region that received no GEMM is never read (see the epilogue).
      umma_commit(BAR(B_ACC));
    }
  } else {
    // ------------------------------------------------------------------ compute warps
    const int wg = warp >> 2, quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int row = m0 + r;
    const bool vrow = row < L;
    const int64_t rb = (int64_t)bh * L;
    const float* posbh = p.pos + (int64_t)bh * 4 * p.Lp;   // planes g, F, rowf, colf
    const int rr = vrow ? row : L - 1;
    const float gi = posbh[rr], fi = posbh[p.Lp + rr];
    const float ga = posbh[m0];
    const float lam = p.lam[h];
    const float rowf = exp2f(fmin_nan((gi - ga) * kLOG2E, 0.f));
    const float rs = lam * rowf;
    const float rs2 = rs * kLOG2E;
    const float lam2 = lam * kLOG2E;
    const float c1 = kScale * kLOG2E;
    const float lse = vrow ? p.lse[rb + row] : INFINITY;
    float* red = reinterpret_cast<float*>(gbase + OFF_RED);
    // delta'' = do . o'' over this warpgroup's NCOL head dims, combined across the warpgroups. o'' comes
    // from the forward already snapped to the rounded output (attention.py:341-350); without it, o'' = o.
    // Both arrive by TMA (o'' as two 128-byte-swizzled boxes of 32 fp32 columns), so the compute warps
    // hold no registers on global loads while they wait.
    static_assert(NCOL == 16, "two 16-byte chunks of dO / o, four of o''");
    bool ok = warp_wait(BAR(B_Q), 0, p.status);
    ok = ok && warp_wait(BAR(B_O), 0, p.status);
    float dh = 0.f;
    if (ok) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int chunk = wg * 2 + q;
        const uint4 dv = *reinterpret_cast<const uint4*>(gbase + OFF_DO + sw128_off(r, chunk));
        const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
        float o[8];
        if (p.o32) {
          // fp32 columns 8 chunk .. 8 chunk + 7: box chunk / 4, 16-byte chunks 2 (chunk % 4) and + 1
          const uint8_t* ob = gbase + OFF_O + (chunk >> 2) * SZ_OB;
          const float4 o0 = *reinterpret_cast<const float4*>(ob + sw128_off(r, 2 * (chunk & 3)));
          const float4 o1 = *reinterpret_cast<const float4*>(ob + sw128_off(r, 2 * (chunk & 3) + 1));
          o[0] = o0.x; o[1] = o0.y; o[2] = o0.z; o[3] = o0.w; o[4] = o1.x; o[5] = o1.y; o[6] = o1.z; o[7] = o1.w;
        } else {
          const uint4 ov = *reinterpret_cast<const uint4*>(gbase + OFF_O + sw128_off(r, chunk));
          const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) { o[2 * i] = unpack_lo<kHalf>(ow[i]); o[2 * i + 1] = unpack_hi<kHalf>(ow[i]); }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          dh = fmaf(o[2 * i], unpack_lo<kHalf>(dw[i]), dh);
          dh = fmaf(o[2 * i + 1], unpack_hi<kHalf>(dw[i]), dh);
        }
      }
    }
    // partial sums of the other warpgroups go to wg 0, which forms delta'' (fixed order) and hands it back
    // row exchange slots, [value][warpgroup][row]: a warp's 32 rows are one 128-byte line
    auto rx = [&](int k, int w) -> float& { return red[(k * NWG + w) * 128 + r]; };
    if (wg > 0) rx(7, wg) = dh;
    named_bar_sync(1, NCT);
    float dl = 0.f;
    if (wg == 0) {
      dl = dh;
#pragma unroll
      for (int w = 1; w < NWG; ++w) dl += rx(7, w);
      rx(6, 0) = dl;
    }
    named_bar_sync(1, NCT);
    if (wg > 0) dl = rx(6, 0);
    const uint32_t tS = tmem_addr(tbase, quarter, COL_S + wg * NCOL);
    const uint32_t tU = tmem_addr(tbase, quarter, COL_U + wg * NCOL);
    const uint32_t tP = tmem_addr(tbase, quarter, COL_DP + wg * NCOL);
    float za = 0.f, ya = 0.f, wa = 0.f, xa = 0.f, ptt = 0.f, dptt = 0.f, xd = 0.f;
    // (F_i - F_j) log2e - lse = fma(F_j, -log2e, F_i log2e - lse): one packed FMA per column pair
    const float filse = fi * kLOG2E - lse;
    const float2 c1v = bcast2(c1), nl2e = bcast2(-kLOG2E), filse2 = bcast2(filse);
    const float2 ndl2 = bcast2(-dl), rs2v = bcast2(rs2);
    float2 xo2 = bcast2(0.f), yo2 = bcast2(0.f), za2 = bcast2(0.f), wa2 = bcast2(0.f);
    float2 xd2 = bcast2(0.f), yd2 = bcast2(0.f);   // u-weighted sums of diagonal tiles (u fully decayed)
    for (int n = 0; ok && n < ntiles; ++n) {
      const int s = n % NST;
      const int j0 = key0(n) + wg * NCOL;
      if (!warp_wait(BAR(B_SUF), n & 1, p.status)) { ok = false; break; }
      tc_fence_after();
      float sv[NCOL], uv[NCOL], pv[NCOL];
      tmem_ld16(tS, sv);
      tmem_ld16(tU, uv);
      tmem_ld16(tP, pv);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(BAR(B_SUE));
      // key position planes of this tile ([4][64] floats {g, F, rowf, colf}), this warpgroup's columns
      const float* kpos = reinterpret_cast<const float*>(gbase + OFF_ST + s * SZ_STAGE + SZ_K + SZ_V + SZ_B);
      const float4* kg4 = reinterpret_cast<const float4*>(kpos + wg * NCOL);
      const float4* kf4 = reinterpret_cast<const float4*>(kpos + 64 + wg * NCOL);
      const float4* kc4 = reinterpret_cast<const float4*>(kpos + 192 + wg * NCOL);
      uint32_t wds[NCOL / 2], wdc[NCOL / 2];
      if (n < ndiag) {
        // Diagonal tile (keys jt .. jt+63). The class of this warp's 32 rows is uniform:
        //  after  - every row lies past the key tile: exp(g_i - g_j) = exp(g_i - ge) colf_j with both
        //           factors <= 1 (ge = g at the key tile's end), packed like the off-diagonal path;
        //  before - every row precedes the key tile: nothing is valid;
        //  across - the diagonal crosses these rows: pairwise exp(min(g_i - g_j, 0)), causal mask, and
        //           the diagonal element itself kept apart (the exact-delta terms).
        const int jt = key0(n), r0 = m0 + quarter * 32;
        if (r0 > jt + 63) {
          const float rowe = ex2_approx(fmin_nan((gi - kpos[63]) * kLOG2E, 0.f));
          const float2 rowe2 = bcast2(rowe), lamv = bcast2(lam), lam2v = bcast2(lam2);
#pragma unroll
          for (int c = 0; c < NCOL; c += 2) {
            const float4 f4 = kf4[c / 4], c4 = kc4[c / 4];
            const float2 fj = (c & 2) ? make_float2(f4.z, f4.w) : make_float2(f4.x, f4.y);
            const float2 cj = (c & 2) ? make_float2(c4.z, c4.w) : make_float2(c4.x, c4.y);
            const float2 dec = mul2(cj, rowe2);
            const float2 u = mul2(make_float2(uv[c], uv[c + 1]), dec);
            const float2 y = fma2(u, lam2v, fma2(fj, nl2e, filse2));
            const float2 x = fma2(make_float2(sv[c], sv[c + 1]), c1v, y);
            const float2 pr = make_float2(ex2_approx(x.x), ex2_approx(x.y));
            const float2 ds = mul2(pr, add2(make_float2(pv[c], pv[c + 1]), ndl2));
            xd2 = fma2(ds, u, xd2);
            yd2 = fma2(pr, u, yd2);
            za2 = add2(za2, pr);
            wa2 = add2(wa2, ds);
            const float2 dsc = mul2(ds, mul2(dec, lamv));
            wds[c / 2] = pack2<kHalf>(ds.x, ds.y);
            wdc[c / 2] = pack2<kHalf>(dsc.x, dsc.y);
          }
        } else if (r0 + 31 < jt) {
#pragma unroll
          for (int c = 0; c < NCOL / 2; ++c) { wds[c] = 0u; wdc[c] = 0u; }
        } else {
          const float gil = gi * kLOG2E;
#pragma unroll
          for (int c = 0; c < NCOL; c += 2) {
            const float4 g4 = kg4[c / 4], f4 = kf4[c / 4];
            float dsv[2], dcv[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int cc = c + e;
              const float gj = (c & 2) ? (e ? g4.w : g4.z) : (e ? g4.y : g4.x);
              const float fj = (c & 2) ? (e ? f4.w : f4.z) : (e ? f4.y : f4.x);
              const int j = j0 + cc;
              const bool valid = (j <= row) && (j < L);
              const float dec = valid ? ex2_approx(fmin_nan(fmaf(gj, -kLOG2E, gil), 0.f)) : 0.f;
              const float u = dec * uv[cc];
              const float x = fmaf(sv[cc], c1, fmaf(fj, -kLOG2E, fmaf(lam2, u, filse)));   // x - lse (log2)
              const float pr = valid ? ex2_approx(x) : 0.f;
              const float ds = pr * (pv[cc] - dl);
              const bool eye = (j == row);
              const float dso = eye ? 0.f : ds;
              if (eye) { ptt += pr; dptt += pv[cc]; xd += uv[cc]; }
              const float po = eye ? 0.f : pr;
              za += po;
              ya = fmaf(po, u, ya);
              wa += dso;
              xa = fmaf(dso, u, xa);
              dsv[e] = dso;
              dcv[e] = dso * (lam * dec);
            }
            wds[c / 2] = pack2<kHalf>(dsv[0], dsv[1]);
            wdc[c / 2] = pack2<kHalf>(dcv[0], dcv[1]);
          }
        }
      } else {
        const float ge = kpos[63];
        const float2 mid2 = bcast2(exp2f(fmin_nan((ga - ge) * kLOG2E, 0.f)));
#pragma unroll
        for (int c = 0; c < NCOL; c += 2) {
          const float4 f4 = kf4[c / 4], c4 = kc4[c / 4];
          const float2 fj = (c & 2) ? make_float2(f4.z, f4.w) : make_float2(f4.x, f4.y);
          const float2 cj = (c & 2) ? make_float2(c4.z, c4.w) : make_float2(c4.x, c4.y);
          const float2 cf = mul2(cj, mid2);                                         // colf mid
          const float2 uc = mul2(make_float2(uv[c], uv[c + 1]), cf);
          const float2 y = fma2(uc, rs2v, fma2(fj, nl2e, filse2));
          const float2 x = fma2(make_float2(sv[c], sv[c + 1]), c1v, y);          // x - lse (log2)
          const float2 pr = make_float2(ex2_approx(x.x), ex2_approx(x.y));
          const float2 ds = mul2(pr, add2(make_float2(pv[c], pv[c + 1]), ndl2));  // P (dP - delta'')
          xo2 = fma2(ds, uc, xo2);
          yo2 = fma2(pr, uc, yo2);
          za2 = add2(za2, pr);
          wa2 = add2(wa2, ds);
          const float2 dsc = mul2(ds, cf);
          wds[c / 2] = pack2<kHalf>(ds.x, ds.y);
          wdc[c / 2] = pack2<kHalf>(dsc.x, dsc.y);
        }
      }
      if (n >= 2 && !warp_wait(BAR(B_OPE + (n & 1)), ((n >> 1) - 1) & 1, p.status)) { ok = false; break; }
      st_op_tmem(tbase, quarter, COL_OPS + (n & 1) * 64, wg, wds);
      st_op_tmem(tbase, quarter, COL_OPS + (n & 1) * 64 + 32, wg, wdc);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(BAR(B_OPF + (n & 1)));
    }
    za += za2.x + za2.y;
    wa += wa2.x + wa2.y;
    xa = fmaf(rowf, xo2.x + xo2.y, xa) + (xd2.x + xd2.y);
    ya = fmaf(rowf, yo2.x + yo2.y, ya) + (yd2.x + yd2.y);
    // ---- combine the warpgroups' row sums (wg > 0 -> smem -> wg 0, fixed order)
    if (wg > 0) {
      rx(0, wg) = za; rx(1, wg) = ya; rx(2, wg) = wa; rx(3, wg) = xa;
      rx(4, wg) = ptt; rx(5, wg) = dptt; rx(6, wg) = xd;
    }
    named_bar_sync(1, NCT);
    if (wg == 0) {
#pragma unroll
      for (int w = 1; w < NWG; ++w) {
        za += rx(0, w); ya += rx(1, w); wa += rx(2, w); xa += rx(3, w);
        ptt += rx(4, w); dptt += rx(5, w); xd += rx(6, w);
      }
      // exact delta, delta-free diagonal (attention.py:449-480)
      float ssum = ptt + za;
      ssum = ssum > 0.f ? ssum : 1.f;
      const float x0 = dptt - dl;
      const float tt = dl + (ptt * x0 + wa) / ssum;
      const float dstt = ptt * (za * x0 - wa) / ssum;
      const float dl_row = xa + (dl - tt) * ya;
      const float dd = tt - dl;
      if (vrow) {
        // the dkv kernel's per-query records: F log2e - lse, and the negated delta terms it adds
        float* rst = p.rstat + (int64_t)bh * 4 * p.Lp + row;
        rst[0] = filse;
        rst[p.Lp] = -dl;
        rst[2 * p.Lp] = -dd;
        rst[3 * p.Lp] = dstt;
        p.rl[rb + row] = dl_row + dstt * xd;
        p.rg[rb + row] = lam * dl_row;
        p.rf[rb + row] = wa - za * dd;
      }
      rx(5, 0) = dstt;                        // handed to the other warpgroups for their column slices
    }
    named_bar_sync(1, NCT);
    const float dstt = rx(5, 0);
    if (ok && !warp_wait(BAR(B_ACC), 0, p.status)) ok = false;
    if (ok && !warp_wait(BAR(B_KR), 0, p.status)) ok = false;
    if (ok) {
      tc_fence_after();
      // every warpgroup drains its slice of the accumulators into the staging tiles:
      // dq = scale * (sum_{j<t} dS^ k_j + DT(dS_tt) k_t), columns [16 wg, 16 wg + 16)
      {
        float acc[16];
        tmem_ld16(tmem_addr(tbase, quarter, COL_DQ + 16 * wg), acc);
        tmem_wait_ld();
        const float dsr = round_lp<kHalf>(dstt);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint4 kv = *reinterpret_cast<const uint4*>(gbase + OFF_KR + sw128_off(r, 2 * wg + q));
          const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w};
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float a0 = fmaf(dsr, unpack_lo<kHalf>(kw[i]), acc[q * 8 + 2 * i]) * kScale;
            const float a1 = fmaf(dsr, unpack_hi<kHalf>(kw[i]), acc[q * 8 + 2 * i + 1]) * kScale;
            w[i] = pack2<kHalf>(a0, a1);
          }
          st_shared_v4(sbase + OFF_Q + sw128_off(r, 2 * wg + q), w[0], w[1], w[2], w[3]);
        }
      }
      // dc = dC_diag + lam rowf dC_off + DT(lam dS_tt) b_t (fp32), columns [8 wg, 8 wg + 8)
      {
        float dco[8], dcd[8];
        tmem_ld8(tmem_addr(tbase, quarter, COL_DCO + 8 * wg), dco);
        tmem_ld8(tmem_addr(tbase, quarter, COL_DCD + 8 * wg), dcd);
        tmem_wait_ld();
        const float dsl = round_lp<kHalf>(dstt * lam);
        const uint4 bv = *reinterpret_cast<const uint4*>(gbase + OFF_BR + sw64_off(r, wg));
        const uint32_t bw[4] = {bv.x, bv.y, bv.z, bv.w};
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float d0 = (ndiag > 0 ? dcd[2 * i] : 0.f) + (ntiles > ndiag ? rs * dco[2 * i] : 0.f);
          const float d1 = (ndiag > 0 ? dcd[2 * i + 1] : 0.f) + (ntiles > ndiag ? rs * dco[2 * i + 1] : 0.f);
          o[2 * i] = __float_as_uint(fmaf(dsl, unpack_lo<kHalf>(bw[i]), d0));
          o[2 * i + 1] = __float_as_uint(fmaf(dsl, unpack_hi<kHalf>(bw[i]), d1));
        }
        st_shared_v4(sbase + OFF_DO + sw128_off(r, 2 * wg), o[0], o[1], o[2], o[3]);
        st_shared_v4(sbase + OFF_DO + sw128_off(r, 2 * wg + 1), o[4], o[5], o[6], o[7]);
      }
      fence_proxy_async_smem();
    }
    // one thread stores both tiles (rows past L are clipped) and waits until they have been read
    named_bar_sync(1, NCT);
    if (tid == 0 && ok) {
      tma_store_4d(&p.tm_dq, sbase + OFF_Q, 0, m0, h, b);
      tma_store_4d(&p.tm_dc, sbase + OFF_DO, 0, m0, h, b);
      bulk_commit();
      bulk_wait_read0();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
#undef BAR
}

// =============================================================================================
// dkv kernel
// =============================================================================================
template <bool kHalf>
__global__ void __launch_bounds__(NTHREADS, 1) attn_bwd_dkv_kernel(const __grid_constant__ BwdParams p) {
  using namespace dkv;
  extern __shared__ uint8_t smem_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int bh, kt;
  tile_order(p.ntq128, p.B * p.H, bh, kt);           // early key tiles carry the most work
  const int b = bh / p.H, h = bh % p.H;
  const int L = p.L;
  const int n0 = kt * 128;
  const int ntiles = (L - n0 + 63) / 64;             // query tiles m0 = n0 + 64 n < L
  const int ndiag = ntiles < 2 ? ntiles : 2;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);
  const uint32_t bar0 = sbase + OFF_BAR;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_BAR + kTmemSlot);
#define BAR(i) (bar0 + 8u * (uint32_t)(i))
  auto stage_addr = [&](int s) { return sbase + OFF_ST + (uint32_t)s * SZ_STAGE; };
  auto issue_stage = [&](int n) {
    const int s = n % NST;
    const int m0 = n0 + 64 * n;
    const uint32_t st = stage_addr(s);
    mbar_expect_tx(BAR(B_KVF + s), SZ_STAGE);
    tma_load_4d(st, &p.tm_q64, BAR(B_KVF + s), 0, m0, h, b);
    tma_load_4d(st + SZ_Q, &p.tm_do64, BAR(B_KVF + s), 0, m0, h, b);
    tma_load_4d(st + SZ_Q + SZ_DO, &p.tm_c64, BAR(B_KVF + s), 0, m0, h, b);
    tma_load_3d(st + SZ_Q + SZ_DO + SZ_C, &p.tm_pos, BAR(B_KVF + s), m0, 0, bh);
    tma_load_3d(st + SZ_Q + SZ_DO + SZ_C + SZ_POS, &p.tm_rstat, BAR(B_KVF + s), m0, 0, bh);
  };
  // As in the dq kernel, the TMA thread initialises the barriers and issues the resident tiles and
  // the first NST query tiles before the block-wide sync.
  const int npre = ntiles < NST ? ntiles : NST;
  if (warp == WARP_TMA && lane == 0) {
    for (int s = 0; s < NST; ++s) { mbar_init(BAR(B_KVF + s), 1); mbar_init(BAR(B_KVE + s), 1); }
    mbar_init(BAR(B_K), 1);
    mbar_init(BAR(B_SUF), 1);
    mbar_init(BAR(B_SUE), NCT);
    for (int i = 0; i < 2; ++i) { mbar_init(BAR(B_OPF + i), NCT); mbar_init(BAR(B_OPE + i), 1); }
    mbar_init(BAR(B_ACC), 1);
    fence_barrier_init();
    fence_proxy_async_smem();
    mbar_expect_tx(BAR(B_K), SZ_K + SZ_V + SZ_B);
    tma_load_4d(sbase + OFF_K, &p.tm_k128, BAR(B_K), 0, n0, h, b);
    tma_load_4d(sbase + OFF_V, &p.tm_v128, BAR(B_K), 0, n0, h, b);
    tma_load_4d(sbase + OFF_B, &p.tm_b128, BAR(B_K), 0, n0, h, b);
    for (int n = 0; n < npre; ++n) issue_stage(n);
  }
  if (warp == WARP_MMA) { tmem_alloc(smem_u32(tmem_slot), TMEM_COLS); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == WARP_TMA) {
    if (lane == 0) {
      for (int n = npre; n < ntiles; ++n) {
        const int s = n % NST;
        if (!mbar_wait<true>(BAR(B_KVE + s), ((n / NST) - 1) & 1, p.status)) break;
        issue_stage(n);
      }
    }
  } else if (warp == WARP_MMA) {
    // score GEMMs S^T = K Q^T, U^T = B~ C^T, dP^T = V dO^T of every query tile
    if (lane == 0) {
      constexpr uint32_t fmt = kHalf ? 0 : 1;
      constexpr uint32_t id_s = make_idesc(128, 64, fmt, 0, 0);
      const uint32_t sK = sbase + OFF_K, sV = sbase + OFF_V, sB = sbase + OFF_B;
      bool ok = mbar_wait<true>(BAR(B_K), 0, p.status);
      for (int n = 0; ok && n < ntiles; ++n) {
        const int s = n % NST;
        if (!mbar_wait<true>(BAR(B_KVF + s), (n / NST) & 1, p.status)) { ok = false; break; }
        if (n > 0 && !mbar_wait<true>(BAR(B_SUE), (n - 1) & 1, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t st = stage_addr(s);
#pragma unroll
        for (int k = 0; k < 4; ++k) umma_ss(tbase + COL_S, desc_k128(sK + k * 32), desc_k128(st + k * 32), id_s, k > 0);
#pragma unroll
        for (int k = 0; k < 2; ++k)
          umma_ss(tbase + COL_U, desc_k64(sB + k * 32), desc_k64(st + SZ_Q + SZ_DO + k * 32), id_s, k > 0);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_ss(tbase + COL_DP, desc_k128(sV + k * 32), desc_k128(st + SZ_Q + k * 32), id_s, k > 0);
        umma_commit(BAR(B_SUF));
      }
    }
  } else if (warp == WARP_GRAD) {
    // gradient GEMMs dV += P^T dO, dK += dS^T Q, dB += dSb^T C from the operands in TMEM; releases the stage
    if (lane == 0) {
      constexpr uint32_t fmt = kHalf ? 0 : 1;
      constexpr uint32_t id_mn64 = make_idesc(128, 64, fmt, 0, 1);
      constexpr uint32_t id_mn32 = make_idesc(128, 32, fmt, 0, 1);
      int nbo = 0, nbd = 0;
      for (int m = 0; m < ntiles; ++m) {
        const int buf = m & 1, s = m % NST;
        if (!mbar_wait<true>(BAR(B_OPF + buf), (m >> 1) & 1, p.status)) break;
        tc_fence_after();
        const uint32_t tPT = tbase + COL_OPS + (uint32_t)buf * 64, tDST = tPT + 32;
        const uint32_t sDSB = sbase + OFF_DSB + (uint32_t)buf * SZ_DSB;
        const uint32_t st = stage_addr(s);
        const bool dg = m < ndiag;
        int& cnt = dg ? nbd : nbo;
        const uint32_t tdb = tbase + (dg ? COL_DBD : COL_DBO);
#pragma unroll
        for (int k = 0; k < 4; ++k)   // dV += P^T dO
          umma_ts(tbase + COL_DV, tPT + k * 8, desc_mn128(st + SZ_Q + k * 2048), id_mn64, (m > 0 || k > 0));
#pragma unroll
        for (int k = 0; k < 4; ++k)   // dK += dS^T Q
          umma_ts(tbase + COL_DK, tDST + k * 8, desc_mn128(st + k * 2048), id_mn64, (m > 0 || k > 0));
#pragma unroll
        for (int k = 0; k < 4; ++k)   // dB += dSb^T C
          umma_ss(tdb, desc_k128(sDSB + k * 32), desc_mn64(st + SZ_Q + SZ_DO + k * 1024), id_mn32, (cnt > 0 || k > 0));
        ++cnt;
        umma_commit(BAR(B_OPE + buf));
        umma_commit(BAR(B_KVE + s));
      }
      umma_commit(BAR(B_ACC));
    }
  } else {
    const int wg = warp >> 2, quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int j = n0 + r;                                // owned key row
    const bool vcol = j < L;
    const int64_t rb = (int64_t)bh * L;
    const float* posbh = p.pos + (int64_t)bh * 4 * p.Lp;   // planes g, F, rowf, colf
    const int jj = vcol ? j : L - 1;
    const float gj = posbh[jj], fj = posbh[p.Lp + jj];
    const float ge = posbh[min(n0 + 127, L - 1)];
    const float lam = p.lam[h];
    const float colf = exp2f(fmin_nan((ge - gj) * kLOG2E, 0.f));     // 128-row key-tile anchor
    const float rk = lam * colf;
    const float rk2 = rk * kLOG2E;
    const float lam2 = lam * kLOG2E;
    const float c1 = kScale * kLOG2E;
    const float dstt_j = vcol ? p.rstat[(int64_t)bh * 4 * p.Lp + 3 * p.Lp + j] : 0.f;
    float* red = reinterpret_cast<float*>(gbase + OFF_RED);
    const uint32_t tS = tmem_addr(tbase, quarter, COL_S + wg * NCOL);
    const uint32_t tU = tmem_addr(tbase, quarter, COL_U + wg * NCOL);
    const uint32_t tP = tmem_addr(tbase, quarter, COL_DP + wg * NCOL);
    float dgu = 0.f, dfs = 0.f;
    const float nfjl = -fj * kLOG2E;                              // x - lse_i = ... + (F_i log2e - lse_i) - F_j log2e
    const float2 c1v = bcast2(c1), nfjl2 = bcast2(nfjl), rk2v = bcast2(rk2);
    float2 dgo2 = bcast2(0.f), dfs2 = bcast2(0.f);
    float2 dgd2 = bcast2(0.f);   // u-weighted dS sum of diagonal tiles (u fully decayed)
    bool ok = true;
    for (int n = 0; ok && n < ntiles; ++n) {
      const int s = n % NST;
      const int i0 = n0 + 64 * n + wg * NCOL;          // first query column of this thread's part
      if (!warp_wait(BAR(B_SUF), n & 1, p.status)) { ok = false; break; }
      tc_fence_after();
      float sv[NCOL], uv[NCOL], pv[NCOL];
      tmem_ld16(tS, sv);
      tmem_ld16(tU, uv);
      tmem_ld16(tP, pv);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(BAR(B_SUE));
      const uint8_t* st = gbase + OFF_ST + s * SZ_STAGE;
      // query position planes {g, F, rowf, colf} and row-statistic planes {F log2e - lse, -delta,
      // -(T^ - delta), dS_tt} of this tile ([4][64] floats each), this warpgroup's columns
      const float* qpos = reinterpret_cast<const float*>(st + SZ_Q + SZ_DO + SZ_C);
      const float* qrst = reinterpret_cast<const float*>(st + SZ_Q + SZ_DO + SZ_C + SZ_POS);
      const float4* qg4 = reinterpret_cast<const float4*>(qpos + wg * NCOL);
      const float4* qr4 = reinterpret_cast<const float4*>(qpos + 128 + wg * NCOL);
      const float4* qG4 = reinterpret_cast<const float4*>(qrst + wg * NCOL);
      const float4* qD4 = reinterpret_cast<const float4*>(qrst + 64 + wg * NCOL);
      const float4* qT4 = reinterpret_cast<const float4*>(qrst + 128 + wg * NCOL);
      uint32_t wp[NCOL / 2], wk[NCOL / 2], wb[NCOL / 2];
      if (n < ndiag) {
        // Diagonal query tile (queries mt .. mt+63). The class of this warp's 32 keys is uniform:
        //  before - every key precedes the query tile: exp(g_i - g_j) = rowf_i exp(g_mt - g_j) with both
        //           factors <= 1 (rowf relative to the query block start mt), packed like the
        //           off-diagonal path; every pair is strictly causal;
        //  after  - every key follows the query tile: nothing is valid;
        //  across - the diagonal crosses these keys: pairwise decay, causal mask, diagonal element.
        const int mt = n0 + 64 * n, k0 = n0 + quarter * 32;
        if (k0 + 31 < mt) {
          const float ek = ex2_approx(fmin_nan((qpos[0] - gj) * kLOG2E, 0.f));   // exp(g_mt - g_j)
          const float2 ek2 = bcast2(ek), lamv = bcast2(lam), lam2v = bcast2(lam2);
          const bool tail = (mt + 64 > L);
#pragma unroll
          for (int c = 0; c < NCOL; c += 2) {
            const float4 r4 = qr4[c / 4], G4 = qG4[c / 4], D4 = qD4[c / 4], T4 = qT4[c / 4];
            const bool hi = (c & 2) != 0;
            const float2 rowf2 = hi ? make_float2(r4.z, r4.w) : make_float2(r4.x, r4.y);
            const float2 G2 = hi ? make_float2(G4.z, G4.w) : make_float2(G4.x, G4.y);
            const float2 nD2 = hi ? make_float2(D4.z, D4.w) : make_float2(D4.x, D4.y);
            const float2 nT2 = hi ? make_float2(T4.z, T4.w) : make_float2(T4.x, T4.y);
            const float2 dec = mul2(rowf2, ek2);
            const float2 u = mul2(make_float2(uv[c], uv[c + 1]), dec);
            const float2 y = fma2(u, lam2v, add2(G2, nfjl2));
            const float2 x = fma2(make_float2(sv[c], sv[c + 1]), c1v, y);
            float2 pr = make_float2(ex2_approx(x.x), ex2_approx(x.y));
            if (tail) {
              if (i0 + c >= L) pr.x = 0.f;
              if (i0 + c + 1 >= L) pr.y = 0.f;
            }
            const float2 dsh = mul2(pr, add2(make_float2(pv[c], pv[c + 1]), nD2));
            const float2 dsx = fma2(pr, nT2, dsh);
            dgd2 = fma2(dsx, u, dgd2);
            dfs2 = add2(dfs2, dsx);
            const float2 dsb = mul2(dsh, mul2(dec, lamv));
            wp[c / 2] = pack2<kHalf>(pr.x, pr.y);
            wk[c / 2] = pack2<kHalf>(dsx.x, dsx.y);
            wb[c / 2] = pack2<kHalf>(dsb.x, dsb.y);
          }
        } else if (k0 > mt + 63) {
#pragma unroll
          for (int c = 0; c < NCOL / 2; ++c) { wp[c] = 0u; wk[c] = 0u; wb[c] = 0u; }
        } else {
          const float gjl = gj * kLOG2E;
#pragma unroll
        for (int c = 0; c < NCOL; c += 2) {
          const float4 g4 = qg4[c / 4], G4 = qG4[c / 4], D4 = qD4[c / 4], T4 = qT4[c / 4];
          float pe[2], ke[2], be[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int cc = c + e;
            const int i = i0 + cc;
            const int sel = (c & 2) + e;
            const float gi = sel == 0 ? g4.x : sel == 1 ? g4.y : sel == 2 ? g4.z : g4.w;
            const float Gi = sel == 0 ? G4.x : sel == 1 ? G4.y : sel == 2 ? G4.z : G4.w;
            const float nDi = sel == 0 ? D4.x : sel == 1 ? D4.y : sel == 2 ? D4.z : D4.w;
            const float nTi = sel == 0 ? T4.x : sel == 1 ? T4.y : sel == 2 ? T4.z : T4.w;
            const bool valid = (i >= j) && (i < L);
            const bool strict = valid && (i > j);
            const bool eye = valid && (i == j);
            const float dec = valid ? ex2_approx(fmin_nan(fmaf(gi, kLOG2E, -gjl), 0.f)) : 0.f;
            const float u = dec * uv[cc];
            const float x = fmaf(sv[cc], c1, fmaf(lam2, u, Gi + nfjl));   // x - lse_i (log2)
            const float pr = valid ? ex2_approx(x) : 0.f;
            const float dsh = pr * (pv[cc] + nDi);
            const float dsx = fmaf(pr, nTi, dsh);
            const float dso = strict ? dsx : 0.f;
            dgu = fmaf(dso, u, dgu);
            dfs += dso;
            pe[e] = pr;
            ke[e] = eye ? dstt_j : dso;
            be[e] = (eye ? dstt_j : (strict ? dsh : 0.f)) * (lam * dec);
          }
          wp[c / 2] = pack2<kHalf>(pe[0], pe[1]);
          wk[c / 2] = pack2<kHalf>(ke[0], ke[1]);
          wb[c / 2] = pack2<kHalf>(be[0], be[1]);
        }
        }
      } else {
        const float gs = qpos[0];                                  // query block start
        const float2 mid2 = bcast2(exp2f(fmin_nan((gs - ge) * kLOG2E, 0.f)));
        // the last query tile of a sequence whose length is not a multiple of 64 masks its columns
        // past L; every other tile takes the loop without the mask (a tile-uniform branch)
        const uint32_t qa = sbase + OFF_ST + (uint32_t)s * SZ_STAGE + SZ_Q + SZ_DO + SZ_C + (uint32_t)wg * NCOL * 4;
        auto ldf4 = [](uint32_t a) {                     // four columns of one plane in one 16-byte load
          const uint4 v = ld_shared_v4(a);
          return make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w));
        };
        auto offdiag = [&](auto masked) {
          float4 r4, G4, D4, T4;
#pragma unroll
          for (int c = 0; c < NCOL; c += 2) {
            if ((c & 2) == 0) {
              r4 = ldf4(qa + 512 + c * 4);
              G4 = ldf4(qa + SZ_POS + c * 4);
              D4 = ldf4(qa + SZ_POS + 256 + c * 4);
              T4 = ldf4(qa + SZ_POS + 512 + c * 4);
            }
            const bool hi = (c & 2) != 0;
            const float2 rowf2 = hi ? make_float2(r4.z, r4.w) : make_float2(r4.x, r4.y);
            const float2 G2 = hi ? make_float2(G4.z, G4.w) : make_float2(G4.x, G4.y);
            const float2 nD2 = hi ? make_float2(D4.z, D4.w) : make_float2(D4.x, D4.y);
            const float2 nT2 = hi ? make_float2(T4.z, T4.w) : make_float2(T4.x, T4.y);
            const float2 rq = mul2(rowf2, mid2);                                      // rowf mid
            const float2 uc = mul2(make_float2(uv[c], uv[c + 1]), rq);
            const float2 y = fma2(uc, rk2v, add2(G2, nfjl2));                         // ... - lse_i
            const float2 x = fma2(make_float2(sv[c], sv[c + 1]), c1v, y);
            float2 pr = make_float2(ex2_approx(x.x), ex2_approx(x.y));
            if constexpr (decltype(masked)::value) {
              if (i0 + c >= L) pr.x = 0.f;
              if (i0 + c + 1 >= L) pr.y = 0.f;
            }
            const float2 dsh = mul2(pr, add2(make_float2(pv[c], pv[c + 1]), nD2));
            const float2 dsx = fma2(pr, nT2, dsh);                                    // exact dS
            dgo2 = fma2(dsx, uc, dgo2);
            dfs2 = add2(dfs2, dsx);
            const float2 dsb = mul2(dsh, rq);
            wp[c / 2] = pack2<kHalf>(pr.x, pr.y);
            wk[c / 2] = pack2<kHalf>(dsx.x, dsx.y);
            wb[c / 2] = pack2<kHalf>(dsb.x, dsb.y);
          }
        };
        if (n0 + 64 * n + 64 > L) offdiag(std::true_type{});
        else offdiag(std::false_type{});
      }
      // two operand buffers: the gradient UMMAs of tile n-2 must have read this one
      const int ob = n & 1;
      if (n >= 2 && !warp_wait(BAR(B_OPE + ob), ((n >> 1) - 1) & 1, p.status)) { ok = false; break; }
      st_op_tmem(tbase, quarter, COL_OPS + ob * 64, wg, wp);
      st_op_tmem(tbase, quarter, COL_OPS + ob * 64 + 32, wg, wk);
      {
        const uint32_t dsb = sbase + OFF_DSB + (uint32_t)ob * SZ_DSB;   // this thread's key row, 16 query columns
        st_shared_v4(dsb + sw128_off(r, 2 * wg), wb[0], wb[1], wb[2], wb[3]);
        st_shared_v4(dsb + sw128_off(r, 2 * wg + 1), wb[4], wb[5], wb[6], wb[7]);
      }
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(BAR(B_OPF + ob));
    }
    dfs += dfs2.x + dfs2.y;
    dgu = fmaf(colf, dgo2.x + dgo2.y, dgu) + (dgd2.x + dgd2.y);
    // row exchange slots, [value][warpgroup][row]: a warp's 32 rows are one 128-byte line
    auto rx = [&](int k, int w) -> float& { return red[(k * NWG + w) * 128 + r]; };
    if (wg > 0) { rx(0, wg) = dgu; rx(1, wg) = dfs; }
    named_bar_sync(1, NCT);
    if (ok && !warp_wait(BAR(B_ACC), 0, p.status)) ok = false;
    if (ok) {
      tc_fence_after();
      // every warpgroup drains its slice of the accumulators into the staging tiles (the resident K and
      // V tiles and the dSb buffers, all free once the last gradient UMMA has completed):
      // dK and dV columns [16 wg, 16 wg + 16), dB columns [8 wg, 8 wg + 8)
#pragma unroll 1
      for (int part = 0; part < 2; ++part) {
        float acc[16];
        tmem_ld16(tmem_addr(tbase, quarter, (part == 0 ? COL_DK : COL_DV) + 16 * wg), acc);
        tmem_wait_ld();
        const float sc = part == 0 ? kScale : 1.f;
        const uint32_t dst = sbase + (part == 0 ? OFF_K : OFF_V);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          uint32_t w4[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) w4[i] = pack2<kHalf>(acc[q * 8 + 2 * i] * sc, acc[q * 8 + 2 * i + 1] * sc);
          st_shared_v4(dst + sw128_off(r, 2 * wg + q), w4[0], w4[1], w4[2], w4[3]);
        }
      }
      {
        float dbo[8], dbd[8];
        tmem_ld8(tmem_addr(tbase, quarter, COL_DBO + 8 * wg), dbo);
        tmem_ld8(tmem_addr(tbase, quarter, COL_DBD + 8 * wg), dbd);
        tmem_wait_ld();
        const bool has_off = ntiles > ndiag;
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = __float_as_uint(dbd[i] + (has_off ? rk * dbo[i] : 0.f));
        st_shared_v4(sbase + OFF_DSB + sw128_off(r, 2 * wg), o[0], o[1], o[2], o[3]);
        st_shared_v4(sbase + OFF_DSB + sw128_off(r, 2 * wg + 1), o[4], o[5], o[6], o[7]);
      }
      fence_proxy_async_smem();
      if (wg == 0 && vcol) {
#pragma unroll
        for (int w = 1; w < NWG; ++w) { dgu += rx(0, w); dfs += rx(1, w); }
        p.dg[rb + j] = p.rg[rb + j] - lam * dgu;
        if (p.dF) p.dF[rb + j] = p.rf[rb + j] - dfs;
      }
    }
    // one thread stores the three tiles (rows past L are clipped) and waits until they have been read
    named_bar_sync(1, NCT);
    if (tid == 0 && ok) {
      tma_store_4d(&p.tm_dk, sbase + OFF_K, 0, n0, h, b);
      tma_store_4d(&p.tm_dv, sbase + OFF_V, 0, n0, h, b);
      tma_store_4d(&p.tm_db, sbase + OFF_DSB, 0, n0, h, b);
      bulk_commit();
      bulk_wait_read0();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == WARP_MMA) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
#undef BAR
}

// d lambda_h = sum over (b, t) of the per-row parts, in fp64 with a fixed reduction tree, rounded once
// (attention.py:781-783). One cluster of kDlamCluster CTAs per head: CTA rank q, thread i takes the
// elements (q kDlamThreads + i) + k kDlamThreads kDlamCluster of the head's B x L values (eight loads in
// flight per round), a tree over the CTA's threads, then rank 0 adds the CTAs' sums in rank order
// through distributed shared memory (deterministic, no atomics, no workspace).
constexpr int kDlamThreads = 512, kDlamCluster = 8;
__global__ void __cluster_dims__(kDlamCluster, 1, 1) __launch_bounds__(kDlamThreads)
    dlam_kernel(const float* rl, float* dlam, int B, int H, int L) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int h = blockIdx.y, rank = (int)cluster.block_rank();
  __shared__ double part[kDlamThreads];
  const int64_t n = (int64_t)B * L, stride = (int64_t)kDlamThreads * kDlamCluster;
  auto at = [&](int64_t e) {
    const int64_t bb = e / L;
    return __ldg(rl + (bb * H + h) * L + (e - bb * L));
  };
  double acc = 0.0;
  int64_t e = (int64_t)rank * kDlamThreads + threadIdx.x;
  for (; e + 7 * stride < n; e += 8 * stride) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = at(e + (int64_t)i * stride);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc += (double)v[i];
  }
  for (; e < n; e += stride) acc += (double)at(e);
  part[threadIdx.x] = acc;
  __syncthreads();
  for (int w = kDlamThreads / 2; w > 0; w >>= 1) {
    if ((int)threadIdx.x < w) part[threadIdx.x] += part[threadIdx.x + w];
    __syncthreads();
  }
  cluster.sync();                        // every CTA's part[0] is final
  if (rank == 0 && threadIdx.x == 0) {
    double t = 0.0;
    for (int q = 0; q < kDlamCluster; ++q) t += *cluster.map_shared_rank(&part[0], q);
    dlam[h] = (float)t;
  }
  cluster.sync();                        // the other CTAs' shared memory stays until rank 0 has read it
}

}  // namespace bwd

cudaError_t launch_attn_bwd(const BwdParams& p, int dtype, cudaStream_t st) {
  using namespace bwd;
  dim3 gq(p.ntq128, p.B * p.H);
  dim3 gk(p.ntq128, p.B * p.H);
  if (dtype == 1) {
    cudaFuncSetAttribute(attn_bwd_dq_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, dqk::SMEM_BYTES);
    cudaFuncSetAttribute(attn_bwd_dkv_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, dkv::SMEM_BYTES);
    attn_bwd_dq_kernel<true><<<gq, NTHREADS, dqk::SMEM_BYTES, st>>>(p);
    attn_bwd_dkv_kernel<true><<<gk, NTHREADS, dkv::SMEM_BYTES, st>>>(p);
  } else {
    cudaFuncSetAttribute(attn_bwd_dq_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, dqk::SMEM_BYTES);
    cudaFuncSetAttribute(attn_bwd_dkv_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, dkv::SMEM_BYTES);
    attn_bwd_dq_kernel<false><<<gq, NTHREADS, dqk::SMEM_BYTES, st>>>(p);
    attn_bwd_dkv_kernel<false><<<gk, NTHREADS, dkv::SMEM_BYTES, st>>>(p);
  }
  dlam_kernel<<<dim3(kDlamCluster, p.H), kDlamThreads, 0, st>>>(p.rl, p.dlam, p.B, p.H, p.L);
  return cudaGetLastError();
}

}  // namespace sisa
