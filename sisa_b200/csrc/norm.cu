// norm.cu - fused RMSNorm (forward/backward) and SwiGLU activation (forward/backward) for the
// model's blocks (reference: src/sisa/modeling.py:26-49).
//
// RMSNorm, as the reference computes it in fp32: rstd = rsqrt(mean(x^2) + eps), y = (x * rstd) * w,
// written directly in the dtype the next linear consumes (under autocast that is the autocast dtype,
// the single rounding the reference's cast would apply). Backward: with xh = x * rstd and g = dy * w,
// dx = rstd * (g - xh * mean(g * xh)); dw = sum over rows of dy * xh, from per-row-block partial sums
// reduced in a fixed order (deterministic).
//
// SwiGLU: a = silu(g) * u in fp32, rounded once; backward da -> dg = da * u * silu'(g),
// du = da * silu(g), silu(g) = g * sigmoid(g), silu'(g) = sigmoid(g) * (1 + g * (1 - sigmoid(g))).
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "norm.h"

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

// One warp per row; the row is read twice (the second time from L1/L2).
template <typename TX, typename TY>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const TX* __restrict__ x, int64_t xs, const float* __restrict__ w,
                                                          int64_t rows, int d, float eps, TY* __restrict__ y, int64_t ys,
                                                          float* __restrict__ rstd) {
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const TX* xr = x + r * xs;
  float ss = 0.f;
  for (int c = lane; c < d; c += 32) {
    const float v = ld(xr, c);
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / (float)d + eps);
  TY* yr = y + r * ys;
  for (int c = lane; c < d; c += 32) st(yr, c, (ld(xr, c) * rs) * __ldg(w + c));
  if (lane == 0) rstd[r] = rs;
}

// dx per row (one warp per row).
template <typename TX, typename TD, typename TO>
__global__ void __launch_bounds__(256) rmsnorm_bwd_dx_kernel(const TD* __restrict__ dy, int64_t dys, const TX* __restrict__ x,
                                                             int64_t xs, const float* __restrict__ w,
                                                             const float* __restrict__ rstd, int64_t rows, int d,
                                                             TO* __restrict__ dx, int64_t dxs) {
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const TX* xr = x + r * xs;
  const TD* dyr = dy + r * dys;
  const float rs = __ldg(rstd + r);
  float dot = 0.f;
  for (int c = lane; c < d; c += 32) dot = fmaf(ld(dyr, c) * __ldg(w + c), ld(xr, c) * rs, dot);
  const float m = warp_sum(dot) / (float)d;
  TO* dxr = dx + r * dxs;
  for (int c = lane; c < d; c += 32) {
    const float gv = ld(dyr, c) * __ldg(w + c), xh = ld(xr, c) * rs;
    st(dxr, c, rs * (gv - xh * m));
  }
}

// dw partial sums: block (column block, row split); thread = column, rows of the split in order.
template <typename TX, typename TD>
__global__ void __launch_bounds__(256) rmsnorm_bwd_dw_kernel(const TD* __restrict__ dy, int64_t dys, const TX* __restrict__ x,
                                                             int64_t xs, const float* __restrict__ rstd, int64_t rows,
                                                             int d, int64_t rows_per_split, float* __restrict__ part) {
  const int c = blockIdx.x * 256 + threadIdx.x;
  if (c >= d) return;
  const int64_t r0 = (int64_t)blockIdx.y * rows_per_split;
  const int64_t r1 = r0 + rows_per_split < rows ? r0 + rows_per_split : rows;
  float acc = 0.f;
  int64_t r = r0;
  for (; r + 8 <= r1; r += 8) {   // eight rows' loads in flight, added in row order
    float a[8], b[8], q[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) { a[k] = ld(dy + (r + k) * dys, c); b[k] = ld(x + (r + k) * xs, c); q[k] = __ldg(rstd + r + k); }
#pragma unroll
    for (int k = 0; k < 8; ++k) acc = fmaf(a[k], b[k] * q[k], acc);
  }
  for (; r < r1; ++r) acc = fmaf(ld(dy + r * dys, c), ld(x + r * xs, c) * __ldg(rstd + r), acc);
  part[(int64_t)blockIdx.y * d + c] = acc;
}

// dw[c] = sum of the partials: a warp per column, lane j adds splits j, j + 32, ... in order, then a
// fixed xor tree over the lanes (deterministic).
__global__ void __launch_bounds__(256) rmsnorm_dw_reduce_kernel(const float* __restrict__ part, int nsplit, int d,
                                                                float* __restrict__ dw) {
  const int c = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (c >= d) return;
  float acc = 0.f;
  int s = lane;
  for (; s + 7 * 32 < nsplit; s += 8 * 32) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = part[(int64_t)(s + 32 * k) * d + c];
#pragma unroll
    for (int k = 0; k < 8; ++k) acc += v[k];
  }
  for (; s < nsplit; s += 32) acc += part[(int64_t)s * d + c];
  acc = warp_sum(acc);
  if (lane == 0) dw[c] = acc;
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

cudaError_t launch_rmsnorm_fwd(const RmsNormFwd& p, cudaStream_t st) {
  using namespace norm;
  const unsigned grid = (unsigned)((p.rows + 7) / 8);
  return by_dtype<float, __nv_bfloat16, __half>(p.x_dtype, [&](auto tx) {
    using TX = decltype(tx);
    return by_dtype<float, __nv_bfloat16, __half>(p.y_dtype, [&](auto ty) {
      using TY = decltype(ty);
      rmsnorm_fwd_kernel<TX, TY><<<grid, 256, 0, st>>>(static_cast<const TX*>(p.x), p.xs, p.w, p.rows, (int)p.d, p.eps,
                                                       static_cast<TY*>(p.y), p.ys, p.rstd);
      return cudaGetLastError();
    });
  });
}

// dw partials: one per 16 rows (at most 4096), so that enough threads are in flight
int64_t rmsnorm_splits(int64_t rows) { const int64_t s = (rows + 15) / 16; return s < 4096 ? s : 4096; }

cudaError_t launch_rmsnorm_bwd(const RmsNormBwd& p, cudaStream_t st) {
  using namespace norm;
  const unsigned grid = (unsigned)((p.rows + 7) / 8);
  const int64_t nsplit = rmsnorm_splits(p.rows);
  const int64_t rps = (p.rows + nsplit - 1) / nsplit;
  const dim3 gdw((unsigned)((p.d + 255) / 256), (unsigned)nsplit);
  return by_dtype<float, __nv_bfloat16, __half>(p.x_dtype, [&](auto tx) {
    using TX = decltype(tx);
    return by_dtype<float, __nv_bfloat16, __half>(p.dy_dtype, [&](auto td) {
      using TD = decltype(td);
      return by_dtype<float, __nv_bfloat16, __half>(p.dx_dtype, [&](auto to) {
        using TO = decltype(to);
        rmsnorm_bwd_dx_kernel<TX, TD, TO><<<grid, 256, 0, st>>>(static_cast<const TD*>(p.dy), p.dys,
                                                                static_cast<const TX*>(p.x), p.xs, p.w, p.rstd, p.rows,
                                                                (int)p.d, static_cast<TO*>(p.dx), p.dxs);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess || !p.dw) return e;
        rmsnorm_bwd_dw_kernel<TX, TD><<<gdw, 256, 0, st>>>(static_cast<const TD*>(p.dy), p.dys, static_cast<const TX*>(p.x),
                                                           p.xs, p.rstd, p.rows, (int)p.d, rps, p.part);
        rmsnorm_dw_reduce_kernel<<<(unsigned)((p.d + 7) / 8), 256, 0, st>>>(p.part, (int)nsplit, (int)p.d, p.dw);
        return cudaGetLastError();
      });
    });
  });
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
