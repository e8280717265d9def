// norm.cu - fused RMSNorm at the blocks' boundaries (forward/backward) and the SwiGLU activation
// (forward/backward) of the model (reference: src/sisa/modeling.py:25-49, used at modeling.py:258-290).
//
// RMSNorm, as the reference computes it in fp32: rstd = rsqrt(mean(v^2) + eps), h = (v * rstd) * w,
// rounded to v's dtype (the reference's output), then stored in the dtype each consumer takes: under
// autocast the next linear's cast is that same single rounding, so storing h in the autocast dtype here
// replaces the cast kernel. Around it the kernels fold what the block does next to a norm in eager
// PyTorch: the residual add v = x + res before it (modeling.py:275-276), a second copy of h for a
// second consumer (the SwiGLU's gate and up projections each cast the norm output), and the attention's
// fp32 forget projection z = h W_f^T + b_f (modeling.py:167-168), whose only input is the norm output.
// Backward: with xh = v * rstd and G the sum of the gradients of h's copies and of dz W_f,
// dv = rstd * (G w - xh * mean(G w xh)) plus the gradient v receives from its other consumers; the
// weight gradients dw = sum_r G xh, dW_f = sum_r dz^T h, db_f = sum_r dz come from per-row-split
// partial sums reduced in a fixed order (deterministic).
//
// SwiGLU: a = silu(g) * u in fp32, rounded once; backward da -> dg = da * u * silu'(g),
// du = da * silu(g), silu(g) = g * sigmoid(g), silu'(g) = sigmoid(g) * (1 + g * (1 - sigmoid(g))).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <type_traits>

#include "norm.h"
#include "sm100.cuh"

namespace sisa {
namespace norm {

template <typename T> __device__ __forceinline__ float ld(const T* p, int64_t i);
template <> __device__ __forceinline__ float ld<float>(const float* p, int64_t i) { return __ldg(p + i); }
template <> __device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(__ldg(p + i));
}
template <> __device__ __forceinline__ float ld<__half>(const __half* p, int64_t i) { return __half2float(__ldg(p + i)); }

template <typename T> __device__ __forceinline__ void st(T* p, int64_t i, float v);
template <> __device__ __forceinline__ void st<float>(float* p, int64_t i, float v) { p[i] = v; }
template <> __device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, int64_t i, float v) {
  p[i] = __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ void st<__half>(__half* p, int64_t i, float v) { p[i] = __float2half_rn(v); }

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------- block-boundary RMSNorm
// Element access by runtime dtype code (0 bf16, 1 fp16, 2 fp32): the branch is uniform over the grid
// and these kernels are bound by HBM. V consecutive elements from element index i (V-aligned).
__device__ __forceinline__ float h2f(uint16_t b, int dt) {
  return dt == 0 ? __uint_as_float((uint32_t)b << 16) : __half2float(__ushort_as_half(b));
}
__device__ __forceinline__ uint16_t f2h(float v, int dt) {
  return dt == 0 ? __bfloat16_as_ushort(__float2bfloat16_rn(v)) : __half_as_ushort(__float2half_rn(v));
}
__device__ __forceinline__ float rnd_to(float v, int dt) { return dt == 2 ? v : h2f(f2h(v, dt), dt); }

template <int V>
__device__ __forceinline__ void ldv(const void* base, int dt, int64_t i, float* o) {
  if (dt == 2) {
    const float* p = static_cast<const float*>(base) + i;
    if constexpr (V == 4) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(p));
      o[0] = t.x; o[1] = t.y; o[2] = t.z; o[3] = t.w;
    } else if constexpr (V == 2) {
      const float2 t = __ldg(reinterpret_cast<const float2*>(p));
      o[0] = t.x; o[1] = t.y;
    } else {
      o[0] = __ldg(p);
    }
  } else {
    const uint16_t* p = static_cast<const uint16_t*>(base) + i;
    if constexpr (V == 4) {
      const uint2 t = __ldg(reinterpret_cast<const uint2*>(p));
      o[0] = h2f((uint16_t)(t.x & 0xffffu), dt); o[1] = h2f((uint16_t)(t.x >> 16), dt);
      o[2] = h2f((uint16_t)(t.y & 0xffffu), dt); o[3] = h2f((uint16_t)(t.y >> 16), dt);
    } else if constexpr (V == 2) {
      const uint32_t t = __ldg(reinterpret_cast<const unsigned int*>(p));
      o[0] = h2f((uint16_t)(t & 0xffffu), dt); o[1] = h2f((uint16_t)(t >> 16), dt);
    } else {
      o[0] = h2f(__ldg(reinterpret_cast<const unsigned short*>(p)), dt);
    }
  }
}

template <int V>
__device__ __forceinline__ void stv(void* base, int dt, int64_t i, const float* v) {
  if (dt == 2) {
    float* p = static_cast<float*>(base) + i;
    if constexpr (V == 4) *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    else if constexpr (V == 2) *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
    else p[0] = v[0];
  } else {
    uint16_t* p = static_cast<uint16_t*>(base) + i;
    if constexpr (V == 4) {
      *reinterpret_cast<uint2*>(p) = make_uint2((uint32_t)f2h(v[0], dt) | ((uint32_t)f2h(v[1], dt) << 16),
                                                (uint32_t)f2h(v[2], dt) | ((uint32_t)f2h(v[3], dt) << 16));
    } else if constexpr (V == 2) {
      *reinterpret_cast<uint32_t*>(p) = (uint32_t)f2h(v[0], dt) | ((uint32_t)f2h(v[1], dt) << 16);
    } else {
      p[0] = f2h(v[0], dt);
    }
  }
}

constexpr int kNormWarps = 8;   // rows in flight per CTA (one warp per row)
constexpr int kNormCache = 8;   // V-chunks per lane kept in registers between the two passes

// v = x (+ res) of row r at column c (V elements).
template <int V>
__device__ __forceinline__ void norm_input(const NormFwd& p, int64_t r, int c, float* v) {
  ldv<V>(p.x, p.xdt, r * p.xs + c, v);
  if (p.res) {
    float t[V];
    ldv<V>(p.res, p.resdt, r * p.ress + c, t);
#pragma unroll
    for (int k = 0; k < V; ++k) v[k] = rnd_to(v[k] + t[k], p.xdt);
  }
}

// One warp per row. kCache (the row fits in kNormCache chunks per lane): the row's loads are all issued
// before anything is stored (the compiler cannot move a load above a store through these untyped
// pointers), w is read from shared memory, and the row stays in registers for the second pass; else
// each pass reads the row again. NP: register slots of the projection (0: none).
template <int V, int NP, bool kCache>
__global__ void __launch_bounds__(256) norm_fwd_kernel(const __grid_constant__ NormFwd p) {
  extern __shared__ __align__(16) float smem[];   // [w (d) | pb (np, padded to 4) | pw (np x d)]
  const int d = (int)p.d, lane = threadIdx.x & 31;
  const int pad = (p.np + 3) & ~3;
  float* s_w = smem;
  float* s_pb = smem + (kCache ? d : 0);
  float* s_pw = s_pb + (NP > 0 ? pad : 0);
  if constexpr (kCache) {
    if ((d & 3) == 0 && (reinterpret_cast<uintptr_t>(p.w) & 15u) == 0) {
#pragma unroll 4
      for (int i = threadIdx.x; i < d / 4; i += blockDim.x)
        reinterpret_cast<float4*>(s_w)[i] = __ldg(reinterpret_cast<const float4*>(p.w) + i);
    } else {
      for (int i = threadIdx.x; i < d; i += blockDim.x) s_w[i] = __ldg(p.w + i);
    }
  }
  if constexpr (NP > 0) {
    // The projection (np x d fp32, 36 KB at d = 768) is staged by every CTA; with few rows per launch
    // (a decode step's 64) this copy is the kernel's critical path, so it moves as 16-byte loads issued
    // four at a time rather than as a chain of dependent scalar loads.
    const int n = p.np * d;
    if ((n & 3) == 0 && ((reinterpret_cast<uintptr_t>(p.pw) | reinterpret_cast<uintptr_t>(s_pw)) & 15u) == 0) {
      const float4* src = reinterpret_cast<const float4*>(p.pw);
      float4* dst = reinterpret_cast<float4*>(s_pw);
#pragma unroll 4
      for (int i = threadIdx.x; i < n / 4; i += blockDim.x) dst[i] = __ldg(src + i);
    } else {
      for (int i = threadIdx.x; i < n; i += blockDim.x) s_pw[i] = __ldg(p.pw + i);
    }
    for (int i = threadIdx.x; i < p.np; i += blockDim.x) s_pb[i] = __ldg(p.pb + i);
  }
  if constexpr (kCache || NP > 0) __syncthreads();
  for (int64_t r = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5); r < p.rows;
       r += (int64_t)gridDim.x * kNormWarps) {
    float z[NP > 0 ? NP : 1];
#pragma unroll
    for (int j = 0; j < (NP > 0 ? NP : 1); ++j) z[j] = 0.f;
    float rs;
    if constexpr (kCache) {
      constexpr int CH = kNormCache;
      float v[CH][V];
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        const int c = (lane + 32 * i) * V;
        if (c < d) ldv<V>(p.x, p.xdt, r * p.xs + c, v[i]);
        else
#pragma unroll
          for (int k = 0; k < V; ++k) v[i][k] = 0.f;
      }
      if (p.res) {
        float t[CH][V];
#pragma unroll
        for (int i = 0; i < CH; ++i) {
          const int c = (lane + 32 * i) * V;
          if (c < d) ldv<V>(p.res, p.resdt, r * p.ress + c, t[i]);
          else
#pragma unroll
            for (int k = 0; k < V; ++k) t[i][k] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < CH; ++i)
#pragma unroll
          for (int k = 0; k < V; ++k) v[i][k] = rnd_to(v[i][k] + t[i][k], p.xdt);
      }
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < CH; ++i)
#pragma unroll
        for (int k = 0; k < V; ++k) ss = fmaf(v[i][k], v[i][k], ss);
      ss = warp_sum(ss);
      rs = rsqrtf(ss / (float)d + p.eps);
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        const int c = (lane + 32 * i) * V;
        if (c >= d) continue;
        if (p.res && p.xsum) stv<V>(p.xsum, p.xdt, r * p.xsums + c, v[i]);
        float h[V];
#pragma unroll
        for (int k = 0; k < V; ++k) h[k] = rnd_to((v[i][k] * rs) * s_w[c + k], p.xdt);
        stv<V>(p.y[0], p.ydt[0], r * p.ys[0] + c, h);
        if (p.nout > 1) stv<V>(p.y[1], p.ydt[1], r * p.ys[1] + c, h);
        if constexpr (NP > 0) {
#pragma unroll
          for (int j = 0; j < NP; ++j)
            if (j < p.np) {
              if constexpr (V == 4) {
                const float4 wv = *reinterpret_cast<const float4*>(s_pw + j * d + c);
                z[j] = fmaf(h[0], wv.x, fmaf(h[1], wv.y, fmaf(h[2], wv.z, fmaf(h[3], wv.w, z[j]))));
              } else {
#pragma unroll
                for (int k = 0; k < V; ++k) z[j] = fmaf(h[k], s_pw[j * d + c + k], z[j]);
              }
            }
        }
      }
    } else {
      float ss = 0.f;
      for (int c = lane * V; c < d; c += 32 * V) {
        float v[V];
        norm_input<V>(p, r, c, v);
        if (p.res && p.xsum) stv<V>(p.xsum, p.xdt, r * p.xsums + c, v);
#pragma unroll
        for (int k = 0; k < V; ++k) ss = fmaf(v[k], v[k], ss);
      }
      ss = warp_sum(ss);
      rs = rsqrtf(ss / (float)d + p.eps);
      for (int c = lane * V; c < d; c += 32 * V) {
        float v[V], h[V];
        norm_input<V>(p, r, c, v);
#pragma unroll
        for (int k = 0; k < V; ++k) h[k] = rnd_to((v[k] * rs) * __ldg(p.w + c + k), p.xdt);
        stv<V>(p.y[0], p.ydt[0], r * p.ys[0] + c, h);
        if (p.nout > 1) stv<V>(p.y[1], p.ydt[1], r * p.ys[1] + c, h);
        if constexpr (NP > 0) {
#pragma unroll
          for (int j = 0; j < NP; ++j)
            if (j < p.np) {
#pragma unroll
              for (int k = 0; k < V; ++k) z[j] = fmaf(h[k], s_pw[j * d + c + k], z[j]);
            }
        }
      }
    }
    if constexpr (NP > 0) {
#pragma unroll
      for (int j = 0; j < NP; ++j)
        if (j < p.np) {
          const float t = warp_sum(z[j]);
          if (lane == 0) p.pz[r * p.np + j] = t + s_pb[j];
        }
    }
    if (lane == 0) p.rstd[r] = rs;
  }
}

// G (the gradient of h) and xh at row r, column c (the uncached path).
template <int V, int NP>
__device__ __forceinline__ void norm_grad_in(const NormBwd& p, int64_t r, int c, float rs, const float* dz,
                                             const float* s_pw, float* g, float* xh) {
  float v[V];
  ldv<V>(p.v, p.vdt, r * p.vs + c, v);
#pragma unroll
  for (int k = 0; k < V; ++k) { g[k] = 0.f; xh[k] = v[k] * rs; }
#pragma unroll
  for (int q = 0; q < 2; ++q)
    if (p.dy[q]) {
      float t[V];
      ldv<V>(p.dy[q], p.dydt[q], r * p.dys[q] + c, t);
#pragma unroll
      for (int k = 0; k < V; ++k) g[k] += t[k];
    }
  if constexpr (NP > 0) {
    const int d = (int)p.d;
#pragma unroll
    for (int k = 0; k < V; ++k) {
      float t = 0.f;
#pragma unroll
      for (int j = 0; j < NP; ++j)
        if (j < p.np) t = fmaf(dz[j], s_pw[j * d + c + k], t);
      g[k] += t;
    }
  }
}

// dv per row (one warp per row). kCache: as in the forward, all of the row's loads come before its
// stores and the row stays in registers.
template <int V, int NP, bool kCache>
__global__ void __launch_bounds__(256) norm_bwd_dx_kernel(const __grid_constant__ NormBwd p) {
  extern __shared__ __align__(16) float smem[];   // [w (d) | pw (np x d)]
  const int d = (int)p.d, lane = threadIdx.x & 31;
  float* s_w = smem;
  float* s_pw = smem + (kCache ? d : 0);
  if constexpr (kCache)
    for (int i = threadIdx.x; i < d; i += blockDim.x) s_w[i] = __ldg(p.w + i);
  if constexpr (NP > 0)
    for (int i = threadIdx.x; i < p.np * d; i += blockDim.x) s_pw[i] = __ldg(p.pw + i);
  if constexpr (kCache || NP > 0) __syncthreads();
  for (int64_t r = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5); r < p.rows;
       r += (int64_t)gridDim.x * kNormWarps) {
    const float rs = __ldg(p.rstd + r);
    float dz[NP > 0 ? NP : 1];
#pragma unroll
    for (int j = 0; j < (NP > 0 ? NP : 1); ++j) dz[j] = (NP > 0 && j < p.np) ? __ldg(p.dz + r * p.np + j) : 0.f;
    if constexpr (kCache) {
      constexpr int CH = kNormCache;
      float xh[CH][V], g[CH][V], e[CH][V];   // e: the gradient from v's other consumers
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        const int c = (lane + 32 * i) * V;
#pragma unroll
        for (int k = 0; k < V; ++k) { xh[i][k] = 0.f; g[i][k] = 0.f; e[i][k] = 0.f; }
        if (c < d) ldv<V>(p.v, p.vdt, r * p.vs + c, xh[i]);
      }
#pragma unroll
      for (int q = 0; q < 2; ++q)
        if (p.dy[q]) {
#pragma unroll
          for (int i = 0; i < CH; ++i) {
            const int c = (lane + 32 * i) * V;
            if (c < d) {
              float t[V];
              ldv<V>(p.dy[q], p.dydt[q], r * p.dys[q] + c, t);
#pragma unroll
              for (int k = 0; k < V; ++k) g[i][k] += t[k];
            }
          }
        }
      if (p.dvin) {
#pragma unroll
        for (int i = 0; i < CH; ++i) {
          const int c = (lane + 32 * i) * V;
          if (c < d) ldv<V>(p.dvin, p.dvindt, r * p.dvins + c, e[i]);
        }
      }
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        const int c = (lane + 32 * i) * V;
        if (c >= d) continue;
#pragma unroll
        for (int k = 0; k < V; ++k) {
          float gk = g[i][k];
          if constexpr (NP > 0) {
            float t = 0.f;
#pragma unroll
            for (int j = 0; j < NP; ++j)
              if (j < p.np) t = fmaf(dz[j], s_pw[j * d + c + k], t);
            gk += t;
          }
          gk *= s_w[c + k];
          xh[i][k] *= rs;
          g[i][k] = gk;
          dot = fmaf(gk, xh[i][k], dot);
        }
      }
      const float m = warp_sum(dot) / (float)d;
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        const int c = (lane + 32 * i) * V;
        if (c >= d) continue;
        float o[V];
#pragma unroll
        for (int k = 0; k < V; ++k) o[k] = rs * (g[i][k] - xh[i][k] * m) + e[i][k];
        stv<V>(p.dx, p.dxdt, r * p.dxs + c, o);
        if (p.dres) stv<V>(p.dres, p.dresdt, r * p.dress + c, o);
      }
    } else {
      float dot = 0.f;
      for (int c = lane * V; c < d; c += 32 * V) {
        float g[V], xh[V];
        norm_grad_in<V, NP>(p, r, c, rs, dz, s_pw, g, xh);
#pragma unroll
        for (int k = 0; k < V; ++k) dot = fmaf(g[k] * __ldg(p.w + c + k), xh[k], dot);
      }
      const float m = warp_sum(dot) / (float)d;
      for (int c = lane * V; c < d; c += 32 * V) {
        float g[V], xh[V], o[V];
        norm_grad_in<V, NP>(p, r, c, rs, dz, s_pw, g, xh);
#pragma unroll
        for (int k = 0; k < V; ++k) o[k] = rs * (g[k] * __ldg(p.w + c + k) - xh[k] * m);
        if (p.dvin) {
          float t[V];
          ldv<V>(p.dvin, p.dvindt, r * p.dvins + c, t);
#pragma unroll
          for (int k = 0; k < V; ++k) o[k] += t[k];
        }
        stv<V>(p.dx, p.dxdt, r * p.dxs + c, o);
        if (p.dres) stv<V>(p.dres, p.dresdt, r * p.dress + c, o);
      }
    }
  }
}

constexpr int kDwRows = 64;   // rows of a split staged in shared memory at a time

// Weight-gradient partial sums of one row split: thread = V adjacent columns, rows in order; rstd and dz
// of kDwRows rows at a time are staged in shared memory (dz rows are read by every thread). Partial
// row layout: [dw (d) | dW_f (np x d) | db_f (np)].
template <int V, int NP>
__global__ void __launch_bounds__(128) norm_bwd_dw_kernel(const __grid_constant__ NormBwd p, int64_t rows_per_split,
                                                           int64_t ncols) {
  __shared__ float s_rs[kDwRows];
  __shared__ float s_dz[NP > 0 ? kDwRows * NP : 1];
  const int d = (int)p.d;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_split;
  const int64_t r1 = r0 + rows_per_split < p.rows ? r0 + rows_per_split : p.rows;
  float* part = p.part + (int64_t)blockIdx.y * ncols;
  const int c = (blockIdx.x * 128 + threadIdx.x) * V;
  const bool on = c < d;
  float wc[V], pw[NP > 0 ? NP : 1][V], aw[V], af[NP > 0 ? NP : 1][V];
#pragma unroll
  for (int k = 0; k < V; ++k) { wc[k] = on ? __ldg(p.w + c + k) : 0.f; aw[k] = 0.f; }
#pragma unroll
  for (int j = 0; j < (NP > 0 ? NP : 1); ++j)
#pragma unroll
    for (int k = 0; k < V; ++k) {
      pw[j][k] = (NP > 0 && on && j < p.np) ? __ldg(p.pw + (int64_t)j * d + c + k) : 0.f;
      af[j][k] = 0.f;
    }
  float db = 0.f;   // thread j < np of column block 0: db_f[j] over the split
  for (int64_t rb = r0; rb < r1; rb += kDwRows) {
    const int nr = (int)(r1 - rb < kDwRows ? r1 - rb : kDwRows);
    __syncthreads();   // the previous chunk's readers are done
    for (int i = threadIdx.x; i < nr; i += blockDim.x) s_rs[i] = __ldg(p.rstd + rb + i);
    if constexpr (NP > 0)
      for (int i = threadIdx.x; i < nr * p.np; i += blockDim.x) s_dz[i] = __ldg(p.dz + rb * p.np + i);
    __syncthreads();
    if (NP > 0 && blockIdx.x == 0 && (int)threadIdx.x < p.np)
      for (int i = 0; i < nr; ++i) db += s_dz[i * p.np + threadIdx.x];
    if (!on) continue;
#pragma unroll 4
    for (int i = 0; i < nr; ++i) {
      const int64_t r = rb + i;
      const float rs = s_rs[i];
      float v[V], g[V];
      ldv<V>(p.v, p.vdt, r * p.vs + c, v);
#pragma unroll
      for (int k = 0; k < V; ++k) g[k] = 0.f;
#pragma unroll
      for (int q = 0; q < 2; ++q)
        if (p.dy[q]) {
          float t[V];
          ldv<V>(p.dy[q], p.dydt[q], r * p.dys[q] + c, t);
#pragma unroll
          for (int k = 0; k < V; ++k) g[k] += t[k];
        }
#pragma unroll
      for (int k = 0; k < V; ++k) {
        const float xh = v[k] * rs;
        if constexpr (NP > 0) {
          float t = 0.f;
#pragma unroll
          for (int j = 0; j < NP; ++j)
            if (j < p.np) t = fmaf(s_dz[i * p.np + j], pw[j][k], t);
          g[k] += t;
          const float h = rnd_to(xh * wc[k], p.vdt);
#pragma unroll
          for (int j = 0; j < NP; ++j)
            if (j < p.np) af[j][k] = fmaf(s_dz[i * p.np + j], h, af[j][k]);
        }
        aw[k] = fmaf(g[k], xh, aw[k]);
      }
    }
  }
  if (NP > 0 && blockIdx.x == 0 && (int)threadIdx.x < p.np) part[(int64_t)d * (1 + p.np) + threadIdx.x] = db;
  if (!on) return;
#pragma unroll
  for (int k = 0; k < V; ++k) part[c + k] = aw[k];
  if constexpr (NP > 0) {
#pragma unroll
    for (int j = 0; j < NP; ++j)
      if (j < p.np) {
#pragma unroll
        for (int k = 0; k < V; ++k) part[(int64_t)d * (1 + j) + c + k] = af[j][k];
      }
  }
}

// ------------------------------------------------- block-boundary RMSNorm, staged row batches
// The training shapes (fp32 residual stream; bf16 or fp32 outputs and gradients; d a multiple of 8 up
// to 1024; np in {0, 8, 12, 16}): a CTA of d/4 threads (rounded up to a warp) owns all columns, four
// per thread, and walks batches of rows. Each batch's rows arrive in shared memory by bulk copies
// (one per row and operand) issued kStages batches ahead, so the copy engine keeps the HBM traffic in
// flight while the threads compute; the thread's slices of w and of the projection (np x 4 values)
// stay in registers. Row sums are a butterfly over the warp plus one exchange between warps. The
// backward also accumulates the weight gradients of its columns over all of the CTA's rows in
// registers and writes one partial row per CTA. The warp-per-row kernels above serve other shapes.
constexpr int kStages = 2;
constexpr int kFwdRows = 8, kBwdRows = 4;
constexpr int kRowsMaxWarps = 8;       // d <= 1024
constexpr int kRowsGrid = 148 * 2;     // CTAs (fixed: the backward's partial rows depend on it)

// In-warp reduce-scatter of N = 2^k <= 32 values per lane: returns on lane l the warp sum of entry
// l >> (5 - k) (halving exchanges, then a plain butterfly on the last value).
template <int N>
__device__ __forceinline__ float warp_reduce_scatter(float (&v)[N], int lane) {
  static_assert(N >= 1 && N <= 32 && (N & (N - 1)) == 0, "power of two up to 32");
  int off = 16;
#pragma unroll
  for (int n = N; n > 1; n >>= 1, off >>= 1) {
    const bool up = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = up ? v[i] : v[i + n / 2];
      const float keep = up ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  float x = v[0];
#pragma unroll
  for (; off >= 1; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

template <int N> struct Log2 { static constexpr int value = 1 + Log2<N / 2>::value; };
template <> struct Log2<1> { static constexpr int value = 0; };

// The R per-row partial sums of every thread -> the CTA totals in s_tot[R], two barriers.
template <int R>
__device__ __forceinline__ void cta_row_sums(float (&v)[R], float* s_red, float* s_tot, int lane, int warp, int nw) {
  const float x = warp_reduce_scatter<R>(v, lane);
  constexpr int sh = 5 - Log2<R>::value;
  if ((lane & ((1 << sh) - 1)) == 0) s_red[warp * R + (lane >> sh)] = x;
  __syncthreads();
  if ((int)threadIdx.x < R) {
    float t = 0.f;
    for (int w = 0; w < nw; ++w) t += s_red[w * R + threadIdx.x];
    s_tot[threadIdx.x] = t;
  }
  __syncthreads();
}

__device__ __forceinline__ void lds4(const float* p, float* o) {
  const float4 t = *reinterpret_cast<const float4*>(p);
  o[0] = t.x; o[1] = t.y; o[2] = t.z; o[3] = t.w;
}
__device__ __forceinline__ void lds4(const __nv_bfloat16* p, float* o) {
  const uint2 t = *reinterpret_cast<const uint2*>(p);
  o[0] = bf16_lo(t.x); o[1] = bf16_hi(t.x); o[2] = bf16_lo(t.y); o[3] = bf16_hi(t.y);
}
__device__ __forceinline__ void stg4(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void stg4(__nv_bfloat16* p, const float* v) {
  *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]));
}

// Batches of a CTA: blockIdx.x, blockIdx.x + gridDim.x, ...
__device__ __forceinline__ int64_t cta_batches(int64_t nb) {
  return nb > (int64_t)blockIdx.x ? (nb - 1 - blockIdx.x) / gridDim.x + 1 : 0;
}

// TX: the residual stream's type (fp32 in training, the compute dtype in inference). With a 16-bit stream
// the sum x + res and the normalised row are rounded to it, as the eager model computes them (the
// warp-per-row kernel's rnd_to), before the norm and the projection read them.
template <int NP, typename TY, typename TX>
__global__ void __launch_bounds__(256) norm_fwd_tma_kernel(const __grid_constant__ NormFwd p) {
  constexpr bool kLowX = !std::is_same<TX, float>::value;
  constexpr int R = kFwdRows, NPP = NP > 0 ? NP : 1;
  constexpr int NZ = NP > 8 ? 16 : (NP > 0 ? 8 : 1);   // projection entries padded to 2^k
  extern __shared__ __align__(128) unsigned char sbuf[];
  __shared__ float s_red[kRowsMaxWarps * R], s_tot[R];
  __shared__ float s_z[NP > 0 ? kRowsMaxWarps * R * NZ : 1];
  __shared__ __align__(8) uint64_t s_bar[kStages];
  const int d = (int)p.d, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int c = 4 * threadIdx.x;
  const bool on = c < d, has_res = p.res != nullptr;
  const uint32_t xrow = (uint32_t)d * sizeof(TX), rrow = has_res ? (uint32_t)d * 2 : 0;
  const uint32_t stage_bytes = R * (xrow + rrow);
  const int64_t nb = (p.rows + R - 1) / R, my_n = cta_batches(nb);
  const TX* xg = static_cast<const TX*>(p.x);
  const __nv_bfloat16* rg = static_cast<const __nv_bfloat16*>(p.res);
  auto issue = [&](int64_t k) {
    const int s = (int)(k % kStages);
    const int64_t r0 = (blockIdx.x + k * gridDim.x) * R;
    const int nr = (int)(p.rows - r0 < R ? p.rows - r0 : R);
    const uint32_t bar = smem_u32(&s_bar[s]), base = smem_u32(sbuf) + s * stage_bytes;
    mbar_expect_tx(bar, nr * (xrow + rrow));
    for (int i = 0; i < nr; ++i) {
      bulk_load(base + i * xrow, xg + (r0 + i) * p.xs, xrow, bar);
      if (has_res) bulk_load(base + R * xrow + i * rrow, rg + (r0 + i) * p.ress, rrow, bar);
    }
  };
  if (threadIdx.x == 0) {
    for (int st = 0; st < kStages; ++st) mbar_init(smem_u32(&s_bar[st]), 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int64_t k = 0; k < kStages && k < my_n; ++k) issue(k);
  float w4[4], pw[NPP][4];
#pragma unroll
  for (int q = 0; q < 4; ++q) w4[q] = on ? __ldg(p.w + c + q) : 0.f;
#pragma unroll
  for (int j = 0; j < NPP; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) pw[j][q] = (NP > 0 && on) ? __ldg(p.pw + (int64_t)j * d + c + q) : 0.f;
  for (int64_t k = 0; k < my_n; ++k) {
    const int s = (int)(k % kStages);
    const int64_t r0 = (blockIdx.x + k * gridDim.x) * R;
    const int nr = (int)(p.rows - r0 < R ? p.rows - r0 : R);
    bool ok = true;
    if (threadIdx.x == 0) ok = mbar_wait(smem_u32(&s_bar[s]), (uint32_t)((k / kStages) & 1), p.status);
    if (__syncthreads_or(!ok)) break;   // every thread leaves together
    const TX* xs = reinterpret_cast<const TX*>(sbuf + s * stage_bytes);
    const __nv_bfloat16* rs_ = reinterpret_cast<const __nv_bfloat16*>(sbuf + s * stage_bytes + R * xrow);
    float v[R][4], ss[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
#pragma unroll
      for (int q = 0; q < 4; ++q) v[i][q] = 0.f;
      if (on && i < nr) {
        lds4(xs + i * d + c, v[i]);
        if (has_res) {
          float t[4];
          lds4(rs_ + i * d + c, t);
#pragma unroll
          for (int q = 0; q < 4; ++q) v[i][q] = kLowX ? round_lp<false>(v[i][q] + t[q]) : v[i][q] + t[q];
        }
      }
      ss[i] = fmaf(v[i][0], v[i][0], fmaf(v[i][1], v[i][1], fmaf(v[i][2], v[i][2], v[i][3] * v[i][3])));
    }
    cta_row_sums<R>(ss, s_red, s_tot, lane, warp, nw);
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int64_t r = r0 + i;
      const float rs = rsqrtf(s_tot[i] / (float)d + p.eps);
      const bool live = on && i < nr;
      float h[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) h[q] = kLowX ? round_lp<false>((v[i][q] * rs) * w4[q]) : (v[i][q] * rs) * w4[q];
      if (live) {
        if (has_res && p.xsum) stg4(static_cast<TX*>(p.xsum) + r * p.xsums + c, v[i]);
        stg4(static_cast<TY*>(p.y[0]) + r * p.ys[0] + c, h);
        if (p.nout > 1) stg4(static_cast<TY*>(p.y[1]) + r * p.ys[1] + c, h);
      }
      if constexpr (NP > 0) {
        float z[NZ];
#pragma unroll
        for (int j = 0; j < NZ; ++j) {
          const int jj = j < NP ? j : 0;
          z[j] = j < NP ? fmaf(h[0], pw[jj][0], fmaf(h[1], pw[jj][1], fmaf(h[2], pw[jj][2], h[3] * pw[jj][3]))) : 0.f;
        }
        const float zs = warp_reduce_scatter<NZ>(z, lane);
        constexpr int sh = 5 - Log2<NZ>::value;
        if ((lane & ((1 << sh) - 1)) == 0) s_z[(warp * R + i) * NZ + (lane >> sh)] = zs;
      }
      if (threadIdx.x == 0 && i < nr) p.rstd[r] = rs;
    }
    if constexpr (NP > 0) {
      __syncthreads();
      for (int e = threadIdx.x; e < R * NP; e += blockDim.x) {
        const int i = e / NP, j = e - i * NP;
        if (i < nr) {
          float t = 0.f;
          for (int w = 0; w < nw; ++w) t += s_z[(w * R + i) * NZ + j];
          p.pz[(r0 + i) * NP + j] = t + __ldg(p.pb + j);
        }
      }
    }
    __syncthreads();   // stage s and the shared scratch are free again
    if (threadIdx.x == 0 && k + kStages < my_n) issue(k + kStages);
  }
}

template <int NP, typename TD>
__global__ void __launch_bounds__(256) norm_bwd_tma_kernel(const __grid_constant__ NormBwd p, int64_t ncols) {
  constexpr int R = kBwdRows, NPP = NP > 0 ? NP : 1;
  extern __shared__ __align__(128) unsigned char sbuf[];
  __shared__ float s_red[kRowsMaxWarps * R], s_tot[R], s_rs[R];
  __shared__ __align__(16) float s_dz[R * NPP];
  __shared__ __align__(8) uint64_t s_bar[kStages];
  const int d = (int)p.d, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int c = 4 * threadIdx.x;
  const bool on = c < d;
  const bool h0 = p.dy[0] != nullptr, h1 = p.dy[1] != nullptr, he = p.dvin != nullptr;
  const uint32_t vrow = (uint32_t)d * 4, yrow = (uint32_t)d * sizeof(TD), erow = (uint32_t)d * 4;
  const uint32_t o_y0 = R * vrow, o_y1 = o_y0 + (h0 ? R * yrow : 0), o_e = o_y1 + (h1 ? R * yrow : 0);
  const uint32_t stage_bytes = o_e + (he ? R * erow : 0);
  const uint32_t row_bytes = vrow + (h0 ? yrow : 0) + (h1 ? yrow : 0) + (he ? erow : 0);
  const int64_t nb = (p.rows + R - 1) / R, my_n = cta_batches(nb);
  auto issue = [&](int64_t k) {
    const int s = (int)(k % kStages);
    const int64_t r0 = (blockIdx.x + k * gridDim.x) * R;
    const int nr = (int)(p.rows - r0 < R ? p.rows - r0 : R);
    const uint32_t bar = smem_u32(&s_bar[s]), base = smem_u32(sbuf) + s * stage_bytes;
    mbar_expect_tx(bar, nr * row_bytes);
    for (int i = 0; i < nr; ++i) {
      const int64_t r = r0 + i;
      bulk_load(base + i * vrow, static_cast<const float*>(p.v) + r * p.vs, vrow, bar);
      if (h0) bulk_load(base + o_y0 + i * yrow, static_cast<const TD*>(p.dy[0]) + r * p.dys[0], yrow, bar);
      if (h1) bulk_load(base + o_y1 + i * yrow, static_cast<const TD*>(p.dy[1]) + r * p.dys[1], yrow, bar);
      if (he) bulk_load(base + o_e + i * erow, static_cast<const float*>(p.dvin) + r * p.dvins, erow, bar);
    }
  };
  // rstd and dz of a batch: one value per thread t < R * NP + R, loaded a batch ahead into a register.
  auto prefetch = [&](int64_t k) -> float {
    const int64_t r0 = (blockIdx.x + k * gridDim.x) * R;
    const int t = threadIdx.x;
    if (t < R * NP) {
      const int64_t r = r0 + t / NPP;
      return r < p.rows ? __ldg(p.dz + r0 * NP + t) : 0.f;
    }
    if (t < R * NP + R) {
      const int64_t r = r0 + (t - R * NP);
      return r < p.rows ? __ldg(p.rstd + r) : 0.f;
    }
    return 0.f;
  };
  if (threadIdx.x == 0) {
    for (int st = 0; st < kStages; ++st) mbar_init(smem_u32(&s_bar[st]), 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int64_t k = 0; k < kStages && k < my_n; ++k) issue(k);
  float pre = my_n > 0 ? prefetch(0) : 0.f;
  float w4[4], pw[NPP][4], aw[4] = {0.f, 0.f, 0.f, 0.f}, af[NPP][4];
#pragma unroll
  for (int q = 0; q < 4; ++q) w4[q] = on ? __ldg(p.w + c + q) : 0.f;
#pragma unroll
  for (int j = 0; j < NPP; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      pw[j][q] = (NP > 0 && on) ? __ldg(p.pw + (int64_t)j * d + c + q) : 0.f;
      af[j][q] = 0.f;
    }
  float db = 0.f;   // thread j < NP: db_f[j] over this CTA's rows
  for (int64_t k = 0; k < my_n; ++k) {
    const int s = (int)(k % kStages);
    const int64_t r0 = (blockIdx.x + k * gridDim.x) * R;
    const int nr = (int)(p.rows - r0 < R ? p.rows - r0 : R);
    if ((int)threadIdx.x < R * NP) s_dz[threadIdx.x] = pre;
    else if ((int)threadIdx.x < R * NP + R) s_rs[threadIdx.x - R * NP] = pre;
    if (k + 1 < my_n) pre = prefetch(k + 1);
    bool ok = true;
    if (threadIdx.x == 0) ok = mbar_wait(smem_u32(&s_bar[s]), (uint32_t)((k / kStages) & 1), p.status);
    if (__syncthreads_or(!ok)) break;   // also publishes s_dz, s_rs
    if (NP > 0 && (int)threadIdx.x < NP)
      for (int i = 0; i < nr; ++i) db += s_dz[i * NP + threadIdx.x];
    const unsigned char* sb = sbuf + s * stage_bytes;
    const float* vs = reinterpret_cast<const float*>(sb);
    const TD* y0s = reinterpret_cast<const TD*>(sb + o_y0);
    const TD* y1s = reinterpret_cast<const TD*>(sb + o_y1);
    const float* es = reinterpret_cast<const float*>(sb + o_e);
    float gw[R][4], dot[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      dot[i] = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) gw[i][q] = 0.f;
      if (!on || i >= nr) continue;
      const float rs = s_rs[i];
      float v[4], g[4] = {0.f, 0.f, 0.f, 0.f};
      lds4(vs + i * d + c, v);
      if (h0) lds4(y0s + i * d + c, g);
      if (h1) {
        float t[4];
        lds4(y1s + i * d + c, t);
#pragma unroll
        for (int q = 0; q < 4; ++q) g[q] += t[q];
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float gq = g[q];
        const float xh = v[q] * rs;
        if constexpr (NP > 0) {
#pragma unroll
          for (int j = 0; j < NP; ++j) gq = fmaf(s_dz[i * NP + j], pw[j][q], gq);
          const float h = xh * w4[q];
#pragma unroll
          for (int j = 0; j < NP; ++j) af[j][q] = fmaf(s_dz[i * NP + j], h, af[j][q]);
        }
        aw[q] = fmaf(gq, xh, aw[q]);
        gw[i][q] = gq * w4[q];
        dot[i] = fmaf(gw[i][q], xh, dot[i]);
      }
    }
    cta_row_sums<R>(dot, s_red, s_tot, lane, warp, nw);
#pragma unroll
    for (int i = 0; i < R; ++i) {
      if (!on || i >= nr) continue;
      const int64_t r = r0 + i;
      const float rs = s_rs[i], m = s_tot[i] / (float)d;
      float v[4], e[4] = {0.f, 0.f, 0.f, 0.f}, o[4];
      lds4(vs + i * d + c, v);
      if (he) lds4(es + i * d + c, e);
#pragma unroll
      for (int q = 0; q < 4; ++q) o[q] = rs * (gw[i][q] - (v[q] * rs) * m) + e[q];
      stg4(static_cast<float*>(p.dx) + r * p.dxs + c, o);
      if (p.dres) stg4(static_cast<__nv_bfloat16*>(p.dres) + r * p.dress + c, o);
    }
    __syncthreads();   // stage s, s_dz, s_rs and the shared scratch are free again
    if (threadIdx.x == 0 && k + kStages < my_n) issue(k + kStages);
  }
  if (!p.part) return;
  float* part = p.part + (int64_t)blockIdx.x * ncols;
  if (NP > 0 && (int)threadIdx.x < NP) part[(int64_t)d * (1 + NP) + threadIdx.x] = db;
  if (!on) return;
#pragma unroll
  for (int q = 0; q < 4; ++q) part[c + q] = aw[q];
  if constexpr (NP > 0) {
#pragma unroll
    for (int j = 0; j < NP; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) part[(int64_t)d * (1 + j) + c + q] = af[j][q];
  }
}

// Column sums of the partials: a warp per column, lane j adds splits j, j + 32, ... in order, then a
// fixed xor tree over the lanes (deterministic). Column ranges go to dw, dW_f, db_f.
__global__ void __launch_bounds__(256) norm_reduce_kernel(const float* __restrict__ part, int nsplit, int64_t ncols,
                                                          int d, int np, float* __restrict__ dw, float* __restrict__ dpw,
                                                          float* __restrict__ dpb) {
  const int64_t col = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (col >= ncols) return;
  float acc = 0.f;
  int s = lane;
  for (; s + 7 * 32 < nsplit; s += 8 * 32) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = part[(int64_t)(s + 32 * k) * ncols + col];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc += v[k];
  }
  for (; s < nsplit; s += 32) acc += part[(int64_t)s * ncols + col];
  acc = warp_sum(acc);
  if (lane != 0) return;
  if (col < d) {
    if (dw) dw[col] = acc;
  } else if (col < (int64_t)d * (1 + np)) {
    if (dpw) dpw[col - d] = acc;
  } else if (dpb) {
    dpb[col - (int64_t)d * (1 + np)] = acc;
  }
}

__device__ __forceinline__ float sigmoidf_(float v) { return 1.f / (1.f + __expf(-v)); }

// SwiGLU on (rows, f) row-strided operands. Thread = 8 consecutive elements of a row (one 16-byte
// vector of a 16-bit type when kVec: f, the strides and the bases are 8-element aligned).
template <typename T, bool kVec>
__device__ __forceinline__ void ld8(const T* p, int n, float* o) {
  if constexpr (kVec && sizeof(T) == 2) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = to_f(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = i < n ? ld(p, i) : 0.f;
  }
}
template <typename T, bool kVec>
__device__ __forceinline__ void st8(T* p, int n, const float* o) {
  if constexpr (kVec && sizeof(T) == 2) {
    uint4 raw;
    T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) st(e, i, o[i]);
    *reinterpret_cast<uint4*>(p) = raw;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < n) st(p, i, o[i]);
  }
}

template <typename T, bool kVec>
__global__ void __launch_bounds__(256) swiglu_fwd_kernel(const T* __restrict__ g, int64_t gs, const T* __restrict__ u,
                                                         int64_t us, int rows, int f, T* __restrict__ a, int64_t as) {
  const int nch = (f + 7) >> 3;
  const int total = rows * nch;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int r = i / nch, c = (i - r * nch) * 8, n = f - c < 8 ? f - c : 8;
    float gv[8], uv[8], o[8];
    ld8<T, kVec>(g + (int64_t)r * gs + c, n, gv);
    ld8<T, kVec>(u + (int64_t)r * us + c, n, uv);
#pragma unroll
    for (int k = 0; k < 8; ++k) o[k] = gv[k] * sigmoidf_(gv[k]) * uv[k];
    st8<T, kVec>(a + (int64_t)r * as + c, n, o);
  }
}

template <typename T, bool kVec>
__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const T* __restrict__ da, int64_t das, const T* __restrict__ g,
                                                         int64_t gs, const T* __restrict__ u, int64_t us, int rows, int f,
                                                         T* __restrict__ dg, int64_t dgs, T* __restrict__ du, int64_t dus) {
  const int nch = (f + 7) >> 3;
  const int total = rows * nch;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int r = i / nch, c = (i - r * nch) * 8, n = f - c < 8 ? f - c : 8;
    float dv[8], gv[8], uv[8], og[8], ou[8];
    ld8<T, kVec>(da + (int64_t)r * das + c, n, dv);
    ld8<T, kVec>(g + (int64_t)r * gs + c, n, gv);
    ld8<T, kVec>(u + (int64_t)r * us + c, n, uv);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float sg = sigmoidf_(gv[k]);
      ou[k] = dv[k] * (gv[k] * sg);
      og[k] = dv[k] * uv[k] * (sg * (1.f + gv[k] * (1.f - sg)));
    }
    st8<T, kVec>(du + (int64_t)r * dus + c, n, ou);
    st8<T, kVec>(dg + (int64_t)r * dgs + c, n, og);
  }
}

}  // namespace norm

// ------------------------------------------------------------------------------------ launchers
namespace {
template <typename F32, typename BF, typename HF, typename Fn>
cudaError_t by_dtype(int dt, Fn&& fn) {
  if (dt == 0) return fn(BF{});
  if (dt == 1) return fn(HF{});
  return fn(F32{});
}
}  // namespace

namespace {
bool al(const void* ptr, int64_t stride, int dt, int v) {
  const int64_t eb = dt == 2 ? 4 : 2;
  return !ptr || ((reinterpret_cast<uintptr_t>(ptr) % (uintptr_t)(eb * v)) == 0 && stride % v == 0);
}

template <int V, int NP, bool kC>
cudaError_t fwd_v(const NormFwd& p, unsigned grid, size_t smem, cudaStream_t st) {
  auto k = norm::norm_fwd_kernel<V, NP, kC>;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  k<<<grid, 256, smem, st>>>(p);
  return cudaGetLastError();
}
template <int V, int NP, bool kC>
cudaError_t dx_v(const NormBwd& p, unsigned grid, size_t smem, cudaStream_t st) {
  auto k = norm::norm_bwd_dx_kernel<V, NP, kC>;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  k<<<grid, 256, smem, st>>>(p);
  return cudaGetLastError();
}

// Dispatch on the projection slots and the register-cached row.
template <int V>
cudaError_t fwd_np(const NormFwd& p, bool cache, unsigned grid, size_t smem, cudaStream_t st) {
  if (p.np == 0) return cache ? fwd_v<V, 0, true>(p, grid, smem, st) : fwd_v<V, 0, false>(p, grid, smem, st);
  if (p.np <= 16) return cache ? fwd_v<V, 16, true>(p, grid, smem, st) : fwd_v<V, 16, false>(p, grid, smem, st);
  return cache ? fwd_v<V, 32, true>(p, grid, smem, st) : fwd_v<V, 32, false>(p, grid, smem, st);
}
template <int V>
cudaError_t dx_np(const NormBwd& p, bool cache, unsigned grid, size_t smem, cudaStream_t st) {
  if (p.np == 0) return cache ? dx_v<V, 0, true>(p, grid, smem, st) : dx_v<V, 0, false>(p, grid, smem, st);
  if (p.np <= 16) return cache ? dx_v<V, 16, true>(p, grid, smem, st) : dx_v<V, 16, false>(p, grid, smem, st);
  return cache ? dx_v<V, 32, true>(p, grid, smem, st) : dx_v<V, 32, false>(p, grid, smem, st);
}

unsigned norm_grid(int64_t rows, int np) {
  const int64_t need = (rows + norm::kNormWarps - 1) / norm::kNormWarps;
  const int64_t cap = np ? 148 * 4 : 148 * 16;   // with a projection every CTA stages its weights once
  return (unsigned)(need < cap ? need : cap);
}
}  // namespace

// Splits of the weight-gradient partial sums: 16 rows each (64 with a projection, whose partial rows
// are np + 1 times longer), at most 4096 (1024).
int64_t norm_splits(int64_t rows, int64_t np) {
  const int64_t rps = np ? 64 : 16, cap = np ? 1024 : 4096;
  const int64_t s = (rows + rps - 1) / rps;
  return s < cap ? s : cap;
}
namespace {
int64_t tma_grid(int64_t rows, int R) {
  const int64_t nb = (rows + R - 1) / R;
  return nb < norm::kRowsGrid ? nb : norm::kRowsGrid;
}
bool tma_np_ok(int np) { return np == 0 || np == 8 || np == 12 || np == 16; }
// A bulk-copied or vector-stored row operand: 16-byte aligned base, row stride a multiple of 16 bytes.
bool rows16(const void* ptr, int64_t stride, int dt) {
  const int64_t eb = dt == 2 ? 4 : 2;
  return !ptr || ((reinterpret_cast<uintptr_t>(ptr) & 15u) == 0 && (stride * eb) % 16 == 0);
}
int tma_threads(int64_t d) { return (int)((d / 4 + 31) / 32 * 32); }

bool fwd_tma_ok(const NormFwd& p) {
  // the stream fp32 (training) or bf16 (inference); a bf16 residual
  if (p.d % 8 || p.d > 1024 || !tma_np_ok(p.np) || (p.xdt != 2 && p.xdt != 0) || (p.res && p.resdt != 0))
    return false;
  if (p.ydt[0] != 0 && p.ydt[0] != 2) return false;
  if (p.nout > 1 && p.ydt[1] != p.ydt[0]) return false;
  return rows16(p.x, p.xs, p.xdt) && rows16(p.res, p.ress, 0) && rows16(p.xsum, p.xsums, p.xdt) &&
         rows16(p.y[0], p.ys[0], p.ydt[0]) && (p.nout < 2 || rows16(p.y[1], p.ys[1], p.ydt[1])) &&
         rows16(p.w, 0, 2) && rows16(p.pw, 0, 2);
}
bool bwd_tma_ok(const NormBwd& p) {
  if (p.d % 8 || p.d > 1024 || !tma_np_ok(p.np) || p.vdt != 2 || p.dxdt != 2) return false;
  if (p.dvin && p.dvindt != 2) return false;
  if (p.dres && p.dresdt != 0) return false;
  const int t = p.dy[0] ? p.dydt[0] : (p.dy[1] ? p.dydt[1] : 0);
  if ((p.dy[0] && p.dydt[0] != t) || (p.dy[1] && p.dydt[1] != t) || (t != 0 && t != 2)) return false;
  if (tma_threads(p.d) < norm::kBwdRows * (p.np + 1)) return false;
  return rows16(p.v, p.vs, 2) && rows16(p.dy[0], p.dys[0], t) && rows16(p.dy[1], p.dys[1], t) &&
         rows16(p.dvin, p.dvins, 2) && rows16(p.dx, p.dxs, 2) && rows16(p.dres, p.dress, 0) && rows16(p.w, 0, 2) &&
         rows16(p.pw, 0, 2);
}

template <int NP, typename TY>
cudaError_t fwd_tma(const NormFwd& p, cudaStream_t st) {
  const size_t xb = p.xdt == 2 ? 4 : 2;
  const size_t smem = (size_t)norm::kStages * norm::kFwdRows * p.d * (xb + (p.res ? 2 : 0));
  auto k = p.xdt == 2 ? norm::norm_fwd_tma_kernel<NP, TY, float> : norm::norm_fwd_tma_kernel<NP, TY, __nv_bfloat16>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  k<<<(unsigned)tma_grid(p.rows, norm::kFwdRows), tma_threads(p.d), smem, st>>>(p);
  return cudaGetLastError();
}
template <typename TY>
cudaError_t fwd_tma_np(const NormFwd& p, cudaStream_t st) {
  switch (p.np) {
    case 0: return fwd_tma<0, TY>(p, st);
    case 8: return fwd_tma<8, TY>(p, st);
    case 12: return fwd_tma<12, TY>(p, st);
    default: return fwd_tma<16, TY>(p, st);
  }
}
template <int NP, typename TD>
cudaError_t bwd_tma(const NormBwd& p, int64_t ncols, cudaStream_t st) {
  const size_t ysz = sizeof(TD);
  const size_t row = p.d * (4 + (p.dy[0] ? ysz : 0) + (p.dy[1] ? ysz : 0) + (p.dvin ? 4 : 0));
  const size_t smem = (size_t)norm::kStages * norm::kBwdRows * row;
  auto k = norm::norm_bwd_tma_kernel<NP, TD>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  k<<<(unsigned)tma_grid(p.rows, norm::kBwdRows), tma_threads(p.d), smem, st>>>(p, ncols);
  return cudaGetLastError();
}
template <typename TD>
cudaError_t bwd_tma_np(const NormBwd& p, int64_t ncols, cudaStream_t st) {
  switch (p.np) {
    case 0: return bwd_tma<0, TD>(p, ncols, st);
    case 8: return bwd_tma<8, TD>(p, ncols, st);
    case 12: return bwd_tma<12, TD>(p, ncols, st);
    default: return bwd_tma<16, TD>(p, ncols, st);
  }
}
}  // namespace

int64_t norm_part_cols(int64_t d, int64_t np) { return d * (1 + np) + np; }

// Partial rows of the weight gradients: as many as the larger of the two paths needs.
int64_t norm_bwd_partials(int64_t rows, int64_t np) {
  const int64_t a = norm_splits(rows, np), b = tma_grid(rows, norm::kBwdRows);
  return a > b ? a : b;
}

cudaError_t launch_norm_fwd(const NormFwd& p, cudaStream_t st) {
  if (fwd_tma_ok(p)) return p.ydt[0] == 0 ? fwd_tma_np<__nv_bfloat16>(p, st) : fwd_tma_np<float>(p, st);
  const bool v4 = p.d % 4 == 0 && al(p.x, p.xs, p.xdt, 4) && al(p.res, p.ress, p.resdt, 4) &&
                  al(p.xsum, p.xsums, p.xdt, 4) && al(p.y[0], p.ys[0], p.ydt[0], 4) &&
                  (p.nout < 2 || al(p.y[1], p.ys[1], p.ydt[1], 4)) && al(p.w, 0, 2, 4);
  const int V = v4 ? 4 : 1;
  const bool cache = p.d <= (int64_t)32 * V * norm::kNormCache;
  const size_t smem = ((cache ? p.d : 0) + ((p.np + 3) & ~3) + (size_t)p.np * p.d) * 4;
  const unsigned grid = norm_grid(p.rows, p.np);
  return v4 ? fwd_np<4>(p, cache, grid, smem, st) : fwd_np<1>(p, cache, grid, smem, st);
}

cudaError_t launch_norm_bwd(const NormBwd& p, cudaStream_t st) {
  const bool want_w = p.dw || p.dpw || p.dpb;
  const int64_t ncols = norm_part_cols(p.d, p.np);
  if (bwd_tma_ok(p)) {
    NormBwd q = p;
    if (!want_w) q.part = nullptr;
    const int t = p.dy[0] ? p.dydt[0] : (p.dy[1] ? p.dydt[1] : 0);
    cudaError_t e = t == 0 ? bwd_tma_np<__nv_bfloat16>(q, ncols, st) : bwd_tma_np<float>(q, ncols, st);
    if (e != cudaSuccess || !want_w) return e;
    norm::norm_reduce_kernel<<<(unsigned)((ncols + 7) / 8), 256, 0, st>>>(
        p.part, (int)tma_grid(p.rows, norm::kBwdRows), ncols, (int)p.d, p.np, p.dw, p.dpw, p.dpb);
    return cudaGetLastError();
  }
  const bool v4 = p.d % 4 == 0 && al(p.v, p.vs, p.vdt, 4) && al(p.dy[0], p.dys[0], p.dydt[0], 4) &&
                  al(p.dy[1], p.dys[1], p.dydt[1], 4) && al(p.dvin, p.dvins, p.dvindt, 4) &&
                  al(p.dx, p.dxs, p.dxdt, 4) && al(p.dres, p.dress, p.dresdt, 4) && al(p.w, 0, 2, 4);
  const int V = v4 ? 4 : 1;
  const bool cache = p.d <= (int64_t)32 * V * norm::kNormCache;
  const size_t smem = ((cache ? p.d : 0) + (size_t)p.np * p.d) * 4;
  const unsigned grid = norm_grid(p.rows, p.np);
  cudaError_t e = v4 ? dx_np<4>(p, cache, grid, smem, st) : dx_np<1>(p, cache, grid, smem, st);
  if (e != cudaSuccess || !want_w) return e;
  const int64_t nsplit = norm_splits(p.rows, p.np);
  const int64_t rps = (p.rows + nsplit - 1) / nsplit;
  const bool v2 = p.d % 2 == 0 && al(p.v, p.vs, p.vdt, 2) && al(p.dy[0], p.dys[0], p.dydt[0], 2) &&
                  al(p.dy[1], p.dys[1], p.dydt[1], 2) && al(p.w, 0, 2, 2) && al(p.pw, p.d, 2, 2);
  const int cpt = v2 ? 2 : 1;
  const dim3 gdw((unsigned)((p.d + 128 * cpt - 1) / (128 * cpt)), (unsigned)nsplit);
  auto dw = [&](auto vw) {
    constexpr int VV = decltype(vw)::value;
    if (p.np == 0) norm::norm_bwd_dw_kernel<VV, 0><<<gdw, 128, 0, st>>>(p, rps, ncols);
    else if (p.np <= 16) norm::norm_bwd_dw_kernel<VV, 16><<<gdw, 128, 0, st>>>(p, rps, ncols);
    else norm::norm_bwd_dw_kernel<VV, 32><<<gdw, 128, 0, st>>>(p, rps, ncols);
  };
  if (v2) dw(std::integral_constant<int, 2>{}); else dw(std::integral_constant<int, 1>{});
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  norm::norm_reduce_kernel<<<(unsigned)((ncols + 7) / 8), 256, 0, st>>>(p.part, (int)nsplit, ncols, (int)p.d, p.np,
                                                                        p.dw, p.dpw, p.dpb);
  return cudaGetLastError();
}

namespace {
bool vec_ok(const void* ptr, int64_t stride) {
  return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0 && stride % 8 == 0;
}
}  // namespace

cudaError_t launch_swiglu_fwd(const SwiGluFwd& p, cudaStream_t st) {
  using namespace norm;
  const bool vec = p.dtype != 2 && p.f % 8 == 0 && vec_ok(p.g, p.gs) && vec_ok(p.u, p.us) && vec_ok(p.a, p.as);
  return by_dtype<float, __nv_bfloat16, __half>(p.dtype, [&](auto t) {
    using T = decltype(t);
    if (vec)
      swiglu_fwd_kernel<T, true><<<148 * 8, 256, 0, st>>>(static_cast<const T*>(p.g), p.gs, static_cast<const T*>(p.u),
                                                          p.us, (int)p.rows, (int)p.f, static_cast<T*>(p.a), p.as);
    else
      swiglu_fwd_kernel<T, false><<<148 * 8, 256, 0, st>>>(static_cast<const T*>(p.g), p.gs, static_cast<const T*>(p.u),
                                                           p.us, (int)p.rows, (int)p.f, static_cast<T*>(p.a), p.as);
    return cudaGetLastError();
  });
}

cudaError_t launch_swiglu_bwd(const SwiGluBwd& p, cudaStream_t st) {
  using namespace norm;
  const bool vec = p.dtype != 2 && p.f % 8 == 0 && vec_ok(p.da, p.das) && vec_ok(p.g, p.gs) && vec_ok(p.u, p.us) &&
                   vec_ok(p.dg, p.dgs) && vec_ok(p.du, p.dus);
  return by_dtype<float, __nv_bfloat16, __half>(p.dtype, [&](auto t) {
    using T = decltype(t);
    if (vec)
      swiglu_bwd_kernel<T, true><<<148 * 8, 256, 0, st>>>(static_cast<const T*>(p.da), p.das, static_cast<const T*>(p.g),
                                                          p.gs, static_cast<const T*>(p.u), p.us, (int)p.rows, (int)p.f,
                                                          static_cast<T*>(p.dg), p.dgs, static_cast<T*>(p.du), p.dus);
    else
      swiglu_bwd_kernel<T, false><<<148 * 8, 256, 0, st>>>(static_cast<const T*>(p.da), p.das, static_cast<const T*>(p.g),
                                                           p.gs, static_cast<const T*>(p.u), p.us, (int)p.rows, (int)p.f,
                                                           static_cast<T*>(p.dg), p.dgs, static_cast<T*>(p.du), p.dus);
    return cudaGetLastError();
  });
}

}  // namespace sisa
