// attn_fwd.cu - exact SISA attention forward on Blackwell tensor cores (tcgen05 + TMA + TMEM).
//
// Reference semantics: src/sisa/kernels/attention.py:177-296 (_fwd) and src/sisa/functional.py:69-103.
// Outputs: o = softmax(s) v (low precision), lse (log2 units), and the self-normalised fp32 output
// o'' = sum DT(p) v / sum DT(p) used by the exact-delta backward (attention.py:36-44, 286-293).
//
// CTA = one 128-row query tile of one (batch, head). Warp roles:
//   warps 0-3  softmax: thread r owns query row r = TMEM lane r (row reductions are thread-local),
//   warp 4     TMA producer: Q and C once, then K, V, B~ and the key position records per 64-key tile,
//   warp 5     UMMA issuer (one lane) and TMEM owner.
// Per key tile: S = Q K^T and U = C B~^T (M=128, N=64) land in TMEM; the softmax threads build
// x = s log2e and write P = 2^(x - m) as packed bf16 straight into tensor memory (one tcgen05.st
// per thread), from where the MMA warp accumulates O += P V with A read from TMEM - the tensor core
// reads only V from shared memory, which keeps these small-N UMMAs off the shared-memory bandwidth
// limit. The P V UMMA runs with N = 80 against V followed by a constant tile that is 1 in its first
// column, so O's column 64 accumulates sum_j DT(p_ij) (the denominator of the self-normalised output)
// on the tensor core instead of two unpacks and an add per column pair. The running maximum is
// rescaled lazily: O (in TMEM, its sum column included) and l are corrected only when a row's tile
// maximum exceeds the reference maximum by more than 2^8, so most tiles need no correction pass. The
// per-element arithmetic runs on packed fp32 pairs (FFMA2/FADD2/FMUL2) with tree reductions. Key
// tiles are visited diagonal first, then from the start of the sequence.
// TMEM: 240 of 256 columns (S 64 | U 64 | O 80 | P 32), so two CTAs share an SM and one CTA's MMAs
// overlap the other's softmax.
#include <cuda_runtime.h>

#include "attn_common.cuh"
#include "attn.h"

namespace sisa {
namespace fwd {

constexpr int BM = 128, BN = 64, NSTAGE = 3;
constexpr uint32_t SZ_Q = BM * 128, SZ_C = BM * 64;
constexpr uint32_t SZ_K = BN * 128, SZ_V = BN * 128, SZ_ONE = BN * 128, SZ_B = BN * 64, SZ_POS = BN * 16;
// Stage: K | V | ONE | B~ | pos. ONE is a constant tile (1 in the first column of every key row) that
// sits where the P V UMMA with N = 80 reads the second 64-wide slice of its V operand, so O's column 64
// accumulates sum_j DT(p_ij) on the tensor core.
constexpr uint32_t OFFS_V = SZ_K, OFFS_ONE = OFFS_V + SZ_V, OFFS_B = OFFS_ONE + SZ_ONE, OFFS_POS = OFFS_B + SZ_B;
constexpr uint32_t SZ_STAGE = OFFS_POS + SZ_POS;              // 29696 = 29 KiB
constexpr uint32_t OFF_Q = 0, OFF_C = OFF_Q + SZ_Q, OFF_ST = OFF_C + SZ_C;
constexpr uint32_t OFF_BAR = OFF_ST + NSTAGE * SZ_STAGE;
constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 + 1024;
static_assert(NSTAGE * SZ_STAGE >= 2 * BM * 128 && SZ_Q >= BM * 128, "epilogue staging fits");
constexpr uint32_t TMEM_COLS = 256;
constexpr int NO = 80;                                           // O columns: 64 head dims | sum DT(p) | 15 zero
constexpr int COL_S = 0, COL_U = 64, COL_O = 128, COL_P = COL_O + NO;   // P: one 32-column bf16x2 buffer
static_assert(COL_P + 32 <= (int)TMEM_COLS, "TMEM budget");
// barrier indices
constexpr int B_Q = 0, B_KVF = 1, B_KVE = 1 + NSTAGE, B_SUF = 1 + 2 * NSTAGE, B_SUE = B_SUF + 1, B_PF = B_SUF + 2,
              B_PE = B_SUF + 3, B_O = B_SUF + 4;
static_assert(B_O * 8 < 128, "barriers end below the TMEM slot");
// two CTAs per SM: 2 x (SMEM_BYTES + 1 KB reserved per block) within the SM's 228 KB
static_assert(2 * (OFF_ST + NSTAGE * SZ_STAGE + 256 + 1024 + 1024) <= 228 * 1024, "two CTAs per SM");

static_assert(OFF_ST % 1024 == 0 && SZ_STAGE % 1024 == 0, "swizzle alignment");

template <bool kHalf>
__global__ void __launch_bounds__(192, 2) attn_fwd_kernel(const __grid_constant__ FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  int bh, rank;
  tile_order(p.ntq, p.B * p.H, bh, rank);
  const int qt = p.ntq - 1 - rank;                 // heaviest query tiles first
  const int b = bh / p.H, h = bh % p.H;
  const int L = p.L;
  const int m0 = qt * BM;
  const int ndiag = (m0 + BN < L) ? 2 : 1;
  const int ntiles = ndiag + m0 / BN;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);
  const uint32_t sQ = sbase + OFF_Q, sC = sbase + OFF_C;
  const uint32_t bar0 = sbase + OFF_BAR;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_BAR + 128);
#define BAR(i) (bar0 + 8u * (uint32_t)(i))

  if (tid == 0) {
    mbar_init(BAR(B_Q), 1);
    for (int s = 0; s < NSTAGE; ++s) { mbar_init(BAR(B_KVF + s), 1); mbar_init(BAR(B_KVE + s), 1); }
    mbar_init(BAR(B_SUF), 1);
    mbar_init(BAR(B_SUE), 128);
    mbar_init(BAR(B_PF), 128);
    mbar_init(BAR(B_PE), 1);
    mbar_init(BAR(B_O), 1);
    fence_barrier_init();
  }
  if (warp == 5) { tmem_alloc(smem_u32(tmem_slot), TMEM_COLS); tmem_relinquish(); }
  if (tid < NSTAGE * BN) {
    // ONE tile row (128-byte swizzle, as TMA lays out V): element 0 of key row k lives in 16-byte chunk k % 8
    const int s = tid / BN, k = tid % BN;
    const uint32_t row = sbase + OFF_ST + (uint32_t)s * SZ_STAGE + OFFS_ONE + (uint32_t)k * 128;
    const uint32_t one = kHalf ? 0x3C00u : 0x3F80u;
#pragma unroll
    for (int c = 0; c < 8; ++c) st_shared_v4(row + (uint32_t)c * 16, c == (k & 7) ? one : 0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch_desc(&p.tm_q); tma_prefetch_desc(&p.tm_k); tma_prefetch_desc(&p.tm_v);
    tma_prefetch_desc(&p.tm_c); tma_prefetch_desc(&p.tm_b); tma_prefetch_desc(&p.tm_pos);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  auto key0 = [&](int n) { return n < ndiag ? m0 + n * BN : (n - ndiag) * BN; };
  auto stage_addr = [&](int s) { return sbase + OFF_ST + (uint32_t)s * SZ_STAGE; };

  if (warp == 4) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_expect_tx(BAR(B_Q), SZ_Q + SZ_C);
      tma_load_4d(sQ, &p.tm_q, BAR(B_Q), 0, m0, h, b);
      tma_load_4d(sC, &p.tm_c, BAR(B_Q), 0, m0, h, b);
      for (int n = 0; n < ntiles; ++n) {
        const int s = n % NSTAGE;
        if (n >= NSTAGE && !mbar_wait<true>(BAR(B_KVE + s), ((n / NSTAGE) - 1) & 1, p.status)) break;
        const int j0 = key0(n);
        const uint32_t st = stage_addr(s);
        mbar_expect_tx(BAR(B_KVF + s), SZ_K + SZ_V + SZ_B + SZ_POS);
        tma_load_4d(st, &p.tm_k, BAR(B_KVF + s), 0, j0, h, b);
        tma_load_4d(st + OFFS_V, &p.tm_v, BAR(B_KVF + s), 0, j0, h, b);
        tma_load_4d(st + OFFS_B, &p.tm_b, BAR(B_KVF + s), 0, j0, h, b);
        tma_load_3d(st + OFFS_POS, &p.tm_pos, BAR(B_KVF + s), j0, 0, bh);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      constexpr uint32_t id_qk = make_idesc(128, 64, kHalf ? 0 : 1, 0, 0);
      constexpr uint32_t id_pv = make_idesc(128, NO, kHalf ? 0 : 1, 0, 1);
      const uint32_t tS = tbase + COL_S, tU = tbase + COL_U, tO = tbase + COL_O;
      bool ok = mbar_wait<true>(BAR(B_Q), 0, p.status);
      auto issue_pv = [&](int m) -> bool {
        const int s = m % NSTAGE;
        if (!mbar_wait<true>(BAR(B_PF), m & 1, p.status)) return false;
        tc_fence_after();
        const uint32_t tP = tbase + COL_P;
        const uint32_t sV = stage_addr(s) + OFFS_V;     // N = 80: V, then the ONE tile 8192 bytes (LBO) on
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_ts(tO, tP + k * 8, desc_mn128(sV + k * 2048), id_pv, (m > 0 || k > 0) ? 1u : 0u);
        umma_commit(BAR(B_PE));
        umma_commit(BAR(B_KVE + s));
        return true;
      };
      for (int n = 0; ok && n < ntiles; ++n) {
        const int s = n % NSTAGE;
        if (!mbar_wait<true>(BAR(B_KVF + s), (n / NSTAGE) & 1, p.status)) { ok = false; break; }
        if (n > 0 && !mbar_wait<true>(BAR(B_SUE), (n - 1) & 1, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t st = stage_addr(s);
#pragma unroll
        for (int k = 0; k < 4; ++k) umma_ss(tS, desc_k128(sQ + k * 32), desc_k128(st + k * 32), id_qk, k > 0);
#pragma unroll
        for (int k = 0; k < 2; ++k)
          umma_ss(tU, desc_k64(sC + k * 32), desc_k64(st + OFFS_B + k * 32), id_qk, k > 0);
        umma_commit(BAR(B_SUF));
        if (n > 0 && !issue_pv(n - 1)) { ok = false; break; }
      }
      if (ok) issue_pv(ntiles - 1);
      umma_commit(BAR(B_O));
    }
  } else {
    // ------------------------------------------------------------------ softmax warps 0-3
    const int r = tid;
    const int row = m0 + r;
    const bool vrow = row < L;
    const float* posbh = p.pos + (int64_t)bh * 4 * p.Lp;        // planes g, F, rowf, colf
    const int rr = vrow ? row : L - 1;
    const float gi = posbh[rr], fi = posbh[p.Lp + rr];
    const float ga = posbh[m0];
    const float lam = p.lam[h];
    const float rs = lam * exp2f(fmin_nan((gi - ga) * kLOG2E, 0.f));   // lam * rowf (128-row anchor)
    const float lam2 = lam * kLOG2E;
    const float c1 = kScale * kLOG2E;
    const uint32_t tS = tmem_addr(tbase, warp, COL_S);
    const uint32_t tU = tmem_addr(tbase, warp, COL_U);
    const uint32_t tO = tmem_addr(tbase, warp, COL_O);
    // (F_i - F_j) log2e = fma(F_j, -log2e, F_i log2e): one packed FMA per column pair
    const float2 c1v = bcast2(c1), nl2e = bcast2(-kLOG2E), lam2v = bcast2(lam2);
    float m_ref = -INFINITY;
    float2 lacc[4] = {bcast2(0.f), bcast2(0.f), bcast2(0.f), bcast2(0.f)};   // l = sum of fp32 p
    // (sum of DT(p) is O's column 64, accumulated by the P V UMMA)
    bool ok = true;
    for (int n = 0; n < ntiles; ++n) {
      const int s = n % NSTAGE;
      const int j0 = key0(n);
      if (!warp_wait_tested<true>(BAR(B_SUF), n & 1, p.status)) { ok = false; break; }
      tc_fence_after();
      // key position planes of this tile: [4][64] floats {g, F, rowf, colf}
      const float* kpos = reinterpret_cast<const float*>(gbase + OFF_ST + s * SZ_STAGE + OFFS_POS);
      const float4* kg4 = reinterpret_cast<const float4*>(kpos);
      const float4* kf4 = reinterpret_cast<const float4*>(kpos + BN);
      const float4* kc4 = reinterpret_cast<const float4*>(kpos + 3 * BN);
      float sv[64], uv[64];
      tmem_ld32(tS, sv);
      tmem_ld32(tS + 32, sv + 32);
      tmem_ld32(tU, uv);
      tmem_ld32(tU + 32, uv + 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(BAR(B_SUE));            // S and U are in registers: the next tile's GEMMs may start
      float2* x2 = reinterpret_cast<float2*>(sv);     // x overwrites S in place, two columns per float2
      const float2* u2 = reinterpret_cast<const float2*>(uv);
      // The running reference max is folded into the row constant: the loops below produce
      // d = x - m_ref directly (m_ref = 0 before the first finite maximum).
      const float mbase = (m_ref == -INFINITY) ? 0.f : m_ref;
      const float2 film2 = bcast2(fi * kLOG2E - mbase);
      if (n < ndiag) {
        // diagonal tile: pairwise decay exp(min(g_i - g_j, 0)), causal mask and sequence end
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float4 g4 = kg4[q], f4 = kf4[q];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = 2 * q + e;
            const float gja = e ? g4.z : g4.x, gjb = e ? g4.w : g4.y;
            const float2 fj = e ? make_float2(f4.z, f4.w) : make_float2(f4.x, f4.y);
            const float da = exp2f(fmin_nan((gi - gja) * kLOG2E, 0.f));
            const float db = exp2f(fmin_nan((gi - gjb) * kLOG2E, 0.f));
            const float2 u = mul2(make_float2(da, db), u2[c]);
            const float2 y = fma2(u, lam2v, fma2(fj, nl2e, film2));
            float2 x = fma2(x2[c], c1v, y);
            const int j = j0 + 2 * c;
            if (!(j <= row && j < L)) x.x = -INFINITY;
            if (!(j + 1 <= row && j + 1 < L)) x.y = -INFINITY;
            x2[c] = x;
          }
        }
      } else {
        const float ge = kpos[BN - 1];
        const float2 rsm = bcast2(rs * exp2f(fmin_nan((ga - ge) * kLOG2E, 0.f)) * kLOG2E);   // lam rowf mid log2e
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const float4 f4 = kf4[q], c4 = kc4[q];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int c = 2 * q + e;
            const float2 fj = e ? make_float2(f4.z, f4.w) : make_float2(f4.x, f4.y);
            const float2 cf = e ? make_float2(c4.z, c4.w) : make_float2(c4.x, c4.y);
            const float2 w = mul2(u2[c], cf);                        // U colf
            const float2 y = fma2(w, rsm, fma2(fj, nl2e, film2));
            x2[c] = fma2(x2[c], c1v, y);
          }
        }
      }
      // tile maximum: 8 independent partial maxima over 8 columns each, three-input max
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        mx[i] = fmax3(sv[i], sv[i + 8], sv[i + 16]);
        mx[i] = fmax3(mx[i], sv[i + 24], sv[i + 32]);
        mx[i] = fmax3(mx[i], sv[i + 40], sv[i + 48]);
        mx[i] = fmaxf(mx[i], sv[i + 56]);
      }
      // mt: this tile's maximum of x - m_ref. The reference moves only when it is exceeded by more
      // than 2^8 (or on the first finite maximum); then O, l and sum DT(p) are scaled by 2^-(shift).
      const float mt = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
      const bool need = (m_ref == -INFINITY) ? (mt > -INFINITY) : (mt > 8.f);
      const float shift = need ? mt : 0.f;
      const float m_new = need ? mbase + mt : m_ref;
      const float corr = need ? ex2_approx(m_ref - m_new) : 1.f;
      const bool any_need = __any_sync(0xffffffffu, need);
      if (any_need && n > 0) {
        // lazy correction of O (including its DT(p) sum column): wait until the previous tile's UMMAs
        // have landed
        if (!warp_wait_tested<true>(BAR(B_PE), (n - 1) & 1, p.status)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int q = 0; q < 5; ++q) {
          float ov[16];
          tmem_ld16(tO + q * 16, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) ov[i] *= corr;
          tmem_st16(tO + q * 16, ov);
        }
        tmem_wait_st();
      }
      const float2 corr2 = bcast2(corr);
#pragma unroll
      for (int i = 0; i < 4; ++i) lacc[i] = mul2(lacc[i], corr2);
      m_ref = m_new;
      if (any_need) {
        // rows whose reference moved shift their exponents (warp-uniform branch, rare after the first tile)
        const float2 ns2 = bcast2(-shift);
#pragma unroll
        for (int c = 0; c < 32; ++c) x2[c] = add2(x2[c], ns2);
      }
      uint32_t w[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float2 pe = make_float2(ex2_approx(x2[c].x), ex2_approx(x2[c].y));
        lacc[c & 3] = add2(lacc[c & 3], pe);
        w[c] = pack2<kHalf>(pe.x, pe.y);
      }
      // one P buffer: the previous tile's P V UMMAs must have read it
      if (n >= 1 && !warp_wait_tested<true>(BAR(B_PE), (n - 1) & 1, p.status)) { ok = false; break; }
      tmem_st32u(tmem_addr(tbase, warp, COL_P), w);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(BAR(B_PF));
    }
    const float2 lsum = add2(add2(lacc[0], lacc[1]), add2(lacc[2], lacc[3]));
    const float l = lsum.x + lsum.y;
    if (ok && !warp_wait_tested<true>(BAR(B_O), 0, p.status)) ok = false;
    if (ok) {
      tc_fence_after();
      float ov[64], lb;
      tmem_ld32(tO, ov);
      tmem_ld32(tO + 32, ov + 32);
      tmem_ld1(tO + 64, lb);
      tmem_wait_ld();
      const float ls = (l == 0.f) ? 1.f : l;
      const float lbs = (lb == 0.f) ? 1.f : lb;
      const float rls = 1.f / ls, rlbs = 1.f / lbs;
      // The row is staged in shared memory that the finished GEMMs no longer read: o (low precision,
      // 128-byte rows) in the Q tile, o'' (fp32, two 32-column boxes) over the stages.
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = pack2<kHalf>(ov[q * 8 + 2 * i] * rls, ov[q * 8 + 2 * i + 1] * rls);
        st_shared_v4(sbase + OFF_Q + sw128_off(r, q), w[0], w[1], w[2], w[3]);
      }
      if (p.o32) {
        // o'' for the exact-delta backward: the self-normalised fp32 output, snapped to the rounded
        // output where the two agree to 2^-15 (attention.py:341-350 does this in the backward)
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          uint32_t o3[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float o32 = ov[4 * q + i] * rlbs, olp = round_lp<kHalf>(ov[4 * q + i] * rls);
            o3[i] = __float_as_uint((fabsf(o32 - olp) <= 3.0517578125e-05f * fabsf(olp)) ? olp : o32);
          }
          st_shared_v4(sbase + OFF_ST + (q >> 3) * (BM * 128) + sw128_off(r, q & 7), o3[0], o3[1], o3[2], o3[3]);
        }
      }
      fence_proxy_async_smem();
      if (vrow) {
        const float lse = ((m_ref == -INFINITY) ? 0.f : m_ref) + log2f(ls);
        p.lse[(int64_t)bh * L + row] = lse;
        if (!isfinite(lse) && p.status) atomicOr(p.status, SISA_ST_NONFINITE);
      }
    }
    // one thread stores the tiles (rows past L are clipped) and waits until they have been read
    named_bar_sync(1, 128);
    if (tid == 0 && ok) {
      tma_store_4d(&p.tm_ost, sbase + OFF_Q, 0, m0, h, b);
      if (p.o32) {
        tma_store_3d(&p.tm_o32, sbase + OFF_ST, 0, m0, bh);
        tma_store_3d(&p.tm_o32, sbase + OFF_ST + BM * 128, 32, m0, bh);
      }
      bulk_commit();
      bulk_wait_read0();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
#undef BAR
}

}  // namespace fwd

cudaError_t launch_attn_fwd(const FwdParams& p, int dtype, cudaStream_t st) {
  using namespace fwd;
  dim3 grid(p.ntq, p.B * p.H);
  if (dtype == 1) {
    cudaFuncSetAttribute(attn_fwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    attn_fwd_kernel<true><<<grid, 192, SMEM_BYTES, st>>>(p);
  } else {
    cudaFuncSetAttribute(attn_fwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    attn_fwd_kernel<false><<<grid, 192, SMEM_BYTES, st>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace sisa
