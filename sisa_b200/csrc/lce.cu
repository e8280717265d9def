// lce.cu - chunked linear + cross-entropy over the tied LM head (reference: src/sisa/kernels/linear_ce.py).
//
// Per chunk of R token rows:
//  1. lce_logits_kernel: persistent tcgen05 GEMM logits = X_c W_p^T (M=128 rows x N=256 vocab tiles,
//     K in 64-wide TMA stages, fp32 accumulators double-buffered in TMEM). Its epilogue rounds each
//     logit to the compute dtype (the autocast rounding point the reference's loss is defined on,
//     linear_ce.py:26-28), stores the bf16 chunk and emits per (row, vocab tile) the online
//     maximum / sum of 2^(x log2e - m) over the real vocabulary columns plus the target logit - the
//     first pass of the reference's row kernel (linear_ce.py:60-89) without re-reading the logits.
//  2. lce_grad_kernel: per row, merge the tile partials into lse, write loss_row = lse - x_label and
//     overwrite the row with G = (exp(x - lse) - onehot) * scale in the compute dtype (linear_ce.py:90-96).
//  dX = G W_p and dW += G^T X_c are plain GEMMs issued by the host (cuBLAS).
#include <cuda_runtime.h>
#include <cstdint>

#include "attn_common.cuh"
#include "lce.h"

namespace sisa {
namespace lce {

constexpr int BM = 128, BN = 256, BK = 64, NST = 4;
constexpr uint32_t SZ_A = BM * BK * 2, SZ_B = BN * BK * 2, SZ_STAGE = SZ_A + SZ_B;   // 48 KiB
constexpr uint32_t OFF_BAR = NST * SZ_STAGE;
constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 + 1024;
constexpr uint32_t TMEM_COLS = 512;       // two 128 x 256 fp32 accumulators
constexpr int B_FULL = 0, B_EMPTY = NST, B_ACCF = 2 * NST, B_ACCE = 2 * NST + 2;
constexpr float kLog2e = 1.4426950408889634f;

template <bool kHalf>
__global__ void __launch_bounds__(192, 1) lce_logits_kernel(const __grid_constant__ LceParams p) {
  extern __shared__ uint8_t smem_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sbase = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (sbase - raw);
  const uint32_t bar0 = sbase + OFF_BAR;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + OFF_BAR + 128);
#define BAR(i) (bar0 + 8u * (uint32_t)(i))
  if (tid == 0) {
    for (int s = 0; s < NST; ++s) { mbar_init(BAR(B_FULL + s), 1); mbar_init(BAR(B_EMPTY + s), 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(BAR(B_ACCF + i), 1); mbar_init(BAR(B_ACCE + i), 128); }
    fence_barrier_init();
  }
  if (warp == 5) { tmem_alloc(smem_u32(tmem_slot), TMEM_COLS); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const int ntiles = p.n_mblk * p.n_nblk;
  const int nk = p.D / BK;

  if (warp == 4) {
    if (lane == 0) {
      int it = 0;   // global k-stage counter
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const int mb = t % p.n_mblk, nb = t / p.n_mblk;
        bool ok = true;
        for (int k = 0; k < nk; ++k, ++it) {
          const int s = it % NST;
          if (it >= NST && !mbar_wait(BAR(B_EMPTY + s), ((it / NST) - 1) & 1, p.status)) { ok = false; break; }
          const uint32_t st = sbase + (uint32_t)s * SZ_STAGE;
          mbar_expect_tx(BAR(B_FULL + s), SZ_STAGE);
          tma_load_2d(st, &p.tm_x, BAR(B_FULL + s), k * BK, mb * BM);
          tma_load_2d(st + SZ_A, &p.tm_w, BAR(B_FULL + s), k * BK, nb * BN);
        }
        if (!ok) break;
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(BM, BN, kHalf ? 0 : 1, 0, 0);
      int it = 0, tl = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < ntiles; t += gridDim.x, ++tl) {
        const int buf = tl & 1;
        if (tl >= 2 && !mbar_wait(BAR(B_ACCE + buf), ((tl >> 1) - 1) & 1, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t acc = tbase + (uint32_t)buf * BN;
        for (int k = 0; k < nk; ++k, ++it) {
          const int s = it % NST;
          if (!mbar_wait(BAR(B_FULL + s), (it / NST) & 1, p.status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t st = sbase + (uint32_t)s * SZ_STAGE;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_ss(acc, desc_k128(st + kk * 32), desc_k128(st + SZ_A + kk * 32), idesc, (k > 0 || kk > 0));
          umma_commit(BAR(B_EMPTY + s));
        }
        if (!ok) break;
        umma_commit(BAR(B_ACCF + buf));
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue warps 0-3
    const int r = tid;
    int tl = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tl) {
      const int mb = t % p.n_mblk, nb = t / p.n_mblk;
      const int buf = tl & 1;
      if (!warp_wait(BAR(B_ACCF + buf), (tl >> 1) & 1, p.status)) break;
      tc_fence_after();
      const int row = mb * BM + r;
      const bool vrow = row < p.R;
      const int64_t lab = vrow ? p.labels[row] : -1;
      const int n0 = nb * BN;
      float m = -INFINITY, s = 0.f, tgt = 0.f;
      bool has_tgt = false;
      uint4* dst = reinterpret_cast<uint4*>(p.logits + 2 * ((int64_t)(vrow ? row : 0) * p.ld + n0));
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        tmem_ld32(tmem_addr(tbase, warp, buf * BN + c0), v);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) w[i] = pack2<kHalf>(v[2 * i], v[2 * i + 1]);
        if (vrow) {
#pragma unroll
          for (int q = 0; q < 4; ++q) dst[c0 / 8 + q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
        }
        // online max / sum-exp over the rounded logits of the real vocabulary columns (NaN propagates)
        float x2[32];
        float mc = -INFINITY;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float x = (i & 1) ? unpack_hi<kHalf>(w[i >> 1]) : unpack_lo<kHalf>(w[i >> 1]);
          const int col = n0 + c0 + i;
          x2[i] = (col < p.V) ? x * kLog2e : -INFINITY;
          mc = (x2[i] != x2[i]) ? x2[i] : fmaxf(mc, x2[i]);
          if (col == lab) { tgt = x; has_tgt = true; }
        }
        const float mn = (mc != mc || m != m) ? NAN : fmaxf(m, mc);
        if (mn != -INFINITY) {
          float acc = (m == -INFINITY) ? 0.f : s * ex2_approx(m - mn);
#pragma unroll
          for (int i = 0; i < 32; ++i) acc += ex2_approx(x2[i] - mn);
          s = acc;
        }
        m = mn;
      }
      tc_fence_before();
      mbar_arrive(BAR(B_ACCE + buf));
      if (vrow) {
        p.part[(int64_t)row * p.n_nblk + nb] = make_float2(m, s);
        if (has_tgt) p.tgt[row] = tgt;
      }
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

// One CTA (256 threads) per row: lse from the tile partials, loss_row, then G in place.
template <bool kHalf>
__global__ void __launch_bounds__(256) lce_grad_kernel(LceGradParams p) {
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  __shared__ float s_m[8], s_s[8];
  const int64_t lab = p.labels[row];
  const bool valid = lab != p.ignore_index;
  // merge partials (log2 domain)
  float m = -INFINITY, s = 0.f;
  for (int i = tid; i < p.n_nblk; i += 256) {
    const float2 q = p.part[(int64_t)row * p.n_nblk + i];
    const float mn = (q.x != q.x || m != m) ? NAN : fmaxf(m, q.x);
    if (mn != -INFINITY) s = (m == -INFINITY ? 0.f : s * exp2f(m - mn)) + (q.x == -INFINITY ? 0.f : q.y * exp2f(q.x - mn));
    m = mn;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float mn = (m2 != m2 || m != m) ? NAN : fmaxf(m, m2);
    if (mn != -INFINITY) s = (m == -INFINITY ? 0.f : s * exp2f(m - mn)) + (m2 == -INFINITY ? 0.f : s2 * exp2f(m2 - mn));
    m = mn;
  }
  if ((tid & 31) == 0) { s_m[tid >> 5] = m; s_s[tid >> 5] = s; }
  __syncthreads();
  m = s_m[0]; s = s_s[0];
  for (int w = 1; w < 8; ++w) {
    const float m2 = s_m[w], s2 = s_s[w];
    const float mn = (m2 != m2 || m != m) ? NAN : fmaxf(m, m2);
    if (mn != -INFINITY) s = (m == -INFINITY ? 0.f : s * exp2f(m - mn)) + (m2 == -INFINITY ? 0.f : s2 * exp2f(m2 - mn));
    m = mn;
  }
  const float lse = (m + log2f(s)) * 0.6931471805599453f;   // natural log
  if (tid == 0) {
    p.loss_rows[row] = valid ? lse - p.tgt[row] : 0.f;
    if (valid && !isfinite(lse) && p.status) atomicOr(p.status, SISA_ST_NONFINITE);
  }
  if (!p.compute_grad) return;
  const float scale = valid ? p.inv_n[0] * p.gscale : 0.f;
  uint4* rowp = reinterpret_cast<uint4*>(p.logits + 2 * (int64_t)row * p.ld);
  const int nvec = p.Vp / 8;
  for (int i = tid; i < nvec; i += 256) {
    const uint4 v = rowp[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float g2[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int col = i * 8 + 2 * e + h;
        const float x = h ? unpack_hi<kHalf>(w[e]) : unpack_lo<kHalf>(w[e]);
        g2[h] = (col < p.V) ? (expf(x - lse) - (col == lab ? 1.f : 0.f)) * scale : 0.f;
      }
      o[e] = pack2<kHalf>(g2[0], g2[1]);
    }
    rowp[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace lce

cudaError_t launch_lce_logits(const LceParams& p, int dtype, int num_sms, cudaStream_t st) {
  using namespace lce;
  const int ntiles = p.n_mblk * p.n_nblk;
  const int grid = ntiles < num_sms ? ntiles : num_sms;
  if (dtype == 1) {
    cudaFuncSetAttribute(lce_logits_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    lce_logits_kernel<true><<<grid, 192, SMEM_BYTES, st>>>(p);
  } else {
    cudaFuncSetAttribute(lce_logits_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    lce_logits_kernel<false><<<grid, 192, SMEM_BYTES, st>>>(p);
  }
  return cudaGetLastError();
}

cudaError_t launch_lce_grad(const LceGradParams& p, int dtype, cudaStream_t st) {
  if (p.R == 0) return cudaSuccess;
  if (dtype == 1) lce::lce_grad_kernel<true><<<p.R, 256, 0, st>>>(p);
  else lce::lce_grad_kernel<false><<<p.R, 256, 0, st>>>(p);
  return cudaGetLastError();
}

}  // namespace sisa
