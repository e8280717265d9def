// lce.cu - chunked linear + cross-entropy over the tied LM head (reference: src/sisa/kernels/linear_ce.py).
//
// Per chunk of R token rows:
//  1. the logits: the CTA-pair tcgen05 GEMM of gemm.cu with its linear-CE epilogue, logits = X_c W_p^T
//     rounded to the compute dtype (the autocast rounding point the reference's loss is defined on,
//     linear_ce.py:26-28), stored as the chunk, with per (row, 256-column tile) the online maximum /
//     sum of 2^(x log2e - m) over the real vocabulary columns plus the target logit - the first pass of
//     the reference's row kernel (linear_ce.py:60-89) without re-reading the logits.
//  2. lce_grad_kernel (here): per row, merge the segment partials into lse, write loss_row = lse - x_label
//     and overwrite the row with G = (exp(x - lse) - onehot) * scale in the compute dtype
//     (linear_ce.py:90-96).
//  3. dX = G W_p and dW += G^T X_c: the same GEMM with the plain epilogue, issued by the host.
//  4. seed_scale_kernel (here): the backward's multiplication of dX / dW by the seed.
#include <cuda_runtime.h>
#include <cstdint>

#include "attn_common.cuh"
#include "lce.h"

namespace sisa {
namespace lce {

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
  const float lse2 = lse * 1.4426950408889634f;             // exp(x - lse) = 2^(x log2 e - lse log2 e)
  uint4* rowp = reinterpret_cast<uint4*>(p.logits + 2 * (int64_t)row * p.ld);
  const int nvec = p.Vp / 8;
  // Four 16-byte loads in flight per thread before any is rewritten: the pass is bound by HBM
  // latency x bytes in flight, not by its arithmetic.
  constexpr int U = 4;
  for (int i0 = tid; i0 < nvec; i0 += 256 * U) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i0 + 256 * u < nvec) v[u] = rowp[i0 + 256 * u];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + 256 * u;
      if (i >= nvec) break;
      const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float g2[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int col = i * 8 + 2 * e + h;
          const float x = h ? unpack_hi<kHalf>(w[e]) : unpack_lo<kHalf>(w[e]);
          const float e2 = ex2_approx(fmaf(x, 1.4426950408889634f, -lse2));
          g2[h] = (col < p.V) ? (e2 - (col == lab ? 1.f : 0.f)) * scale : 0.f;
        }
        o[e] = pack2<kHalf>(g2[0], g2[1]);
      }
      rowp[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// x (n fp32) times the backward seed *seed, written to out in out_dtype, or in place when out is
// null. With out null and a seed of exactly 1 nothing is written (each block reads the seed and
// leaves), so the common loss.backward() costs one short launch instead of a pass over dW.
template <int OUT>
__global__ void __launch_bounds__(256) seed_scale_kernel(float* x, int64_t n, const float* seed, void* out) {
  const float sd = *seed;
  if (OUT == 2 && out == nullptr && sd == 1.f) return;
  const int64_t n4 = n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 v = reinterpret_cast<const float4*>(x)[i];
    v.x *= sd; v.y *= sd; v.z *= sd; v.w *= sd;
    if constexpr (OUT == 2) {
      reinterpret_cast<float4*>(out ? out : x)[i] = v;
    } else {
      const uint32_t a = pack2<OUT == 1>(v.x, v.y), b = pack2<OUT == 1>(v.z, v.w);
      reinterpret_cast<uint2*>(out)[i] = make_uint2(a, b);
    }
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = x[i] * sd;
    if constexpr (OUT == 2) (out ? static_cast<float*>(out) : x)[i] = v;
    else static_cast<uint16_t*>(out)[i] = (uint16_t)(pack2<OUT == 1>(v, 0.f) & 0xFFFFu);
  }
}

}  // namespace lce

cudaError_t launch_seed_scale(float* x, int64_t n, const float* seed, void* out, int out_dtype, int num_sms,
                              cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  int64_t blocks = (n / 4 + 255) / 256;
  if (blocks > 4 * (int64_t)num_sms) blocks = 4 * (int64_t)num_sms;
  if (blocks < 1) blocks = 1;
  if (out_dtype == 0) lce::seed_scale_kernel<0><<<(int)blocks, 256, 0, st>>>(x, n, seed, out);
  else if (out_dtype == 1) lce::seed_scale_kernel<1><<<(int)blocks, 256, 0, st>>>(x, n, seed, out);
  else lce::seed_scale_kernel<2><<<(int)blocks, 256, 0, st>>>(x, n, seed, out);
  return cudaGetLastError();
}

cudaError_t launch_lce_grad(const LceGradParams& p, int dtype, cudaStream_t st) {
  if (p.R == 0) return cudaSuccess;
  if (dtype == 1) lce::lce_grad_kernel<true><<<p.R, 256, 0, st>>>(p);
  else lce::lce_grad_kernel<false><<<p.R, 256, 0, st>>>(p);
  return cudaGetLastError();
}

}  // namespace sisa
