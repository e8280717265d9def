// optim.cu - AdamW with global-norm gradient clipping over flat fp32 buffers: the training step's
// `clip_grad_norm_` + `torch.optim.AdamW` (examples/train_minimal.py:253-301 of the reference) as two
// passes over the parameters' one contiguous layout instead of per-tensor launches.
//
// Pass 1 (adamw_sumsq_kernel): sum of squared gradients, fp64, a fixed grid and a fixed order
// (deterministic); block 0 also advances the step counter. Pass 2 (adamw_update_kernel): every block
// sums the pass-1 partials in the same order, forms the clip factor min(1, max_norm / (norm + 1e-6)),
// and updates its float4 chunks: decoupled weight decay p *= 1 - lr wd, then m, v and the bias-corrected
// step, with (lr, wd) of the parameter group the chunk belongs to (segments, binary search in shared
// memory; every segment is a multiple of 4 elements, so a float4 never straddles two). The tensor-list
// form below runs the same passes over separate parameter tensors.
#include <cuda_runtime.h>

#include <cstdint>

#include "optim.h"
#include "status.h"

namespace sisa {
namespace optim {

constexpr int kSumsqLoads = 4;     // 16-byte gradient loads in flight per thread in the norm passes

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Warp 0 of an update block: the clipping factor from the norm pass's partial sums, into *s_clip. Lane l
// adds partials l, l+32, ... in order and the warp folds the lane sums in a fixed butterfly, so every
// block and every run gets the same bits; the 32 lanes keep the partial loads in flight together instead
// of one thread reading them one after another while the whole grid waits.
__device__ __forceinline__ void clip_from_partials(const double* partials, int npart, float max_norm,
                                                   int32_t* status, float* s_clip) {
  double t = 0.0;
  for (int i = threadIdx.x; i < npart; i += 32) t += partials[i];
  t = warp_sum(t);
  if (threadIdx.x == 0) {
    const double norm = sqrt(t);
    float clip = 1.f;
    if (max_norm > 0.f) {
      const double c = (double)max_norm / (norm + 1e-6);
      clip = c < 1.0 ? (float)c : 1.f;
    }
    if (!isfinite(norm) && status) atomicOr(status, SISA_ST_NONFINITE);
    *s_clip = clip;
  }
}

__global__ void __launch_bounds__(256) adamw_sumsq_kernel(const float* __restrict__ g, int64_t n4, double* partials,
                                                          float* step) {
  __shared__ double red[8];
  double acc = 0.0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // kSumsqLoads loads in flight per thread (the fixed grid is small), added in the same chunk order
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + (kSumsqLoads - 1) * stride < n4; i += kSumsqLoads * stride) {
    float4 v[kSumsqLoads];
#pragma unroll
    for (int u = 0; u < kSumsqLoads; ++u) v[u] = reinterpret_cast<const float4*>(g)[i + u * stride];
#pragma unroll
    for (int u = 0; u < kSumsqLoads; ++u)
      acc += (double)v[u].x * v[u].x + (double)v[u].y * v[u].y + (double)v[u].z * v[u].z + (double)v[u].w * v[u].w;
  }
  for (; i < n4; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(g)[i];
    acc += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < 8; ++w) t += red[w];
    partials[blockIdx.x] = t;
    if (blockIdx.x == 0) *step += 1.f;
  }
}

__global__ void __launch_bounds__(256) adamw_update_kernel(AdamParams p) {
  extern __shared__ uint8_t smem[];
  AdamSeg* segs = reinterpret_cast<AdamSeg*>(smem);
  __shared__ float s_clip;
  for (int i = threadIdx.x; i < p.nseg; i += blockDim.x) segs[i] = p.segs[i];
  if (threadIdx.x < 32) clip_from_partials(p.partials, p.npart, p.max_norm, p.status, &s_clip);
  __syncthreads();
  const float clip = s_clip;
  const float t = *p.step;
  const float bc1 = 1.f - powf(p.beta1, t), bc2 = 1.f - powf(p.beta2, t);
  const float bc2_sqrt = sqrtf(bc2);
  const float b1 = p.beta1, b2 = p.beta2, omb1 = 1.f - p.beta1, omb2 = 1.f - p.beta2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < p.n4; i += stride) {
    // the segment holding element 4 i
    const int64_t e = 4 * i;
    int lo = 0, hi = p.nseg - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (segs[mid].start <= e) lo = mid; else hi = mid - 1;
    }
    const AdamSeg sg = segs[lo];
    if (e >= sg.end) continue;                      // padding between segments: untouched
    const float lr = sg.lr, decay = 1.f - sg.lr * sg.weight_decay;
    const float step_size = lr / bc1;
    float4 pv = reinterpret_cast<float4*>(p.param)[i];
    const float4 gv = reinterpret_cast<const float4*>(p.grad)[i];
    float4 mv = reinterpret_cast<float4*>(p.m)[i];
    float4 vv = reinterpret_cast<float4*>(p.v)[i];
    float* pp = &pv.x;
    const float* gp = &gv.x;
    float* mp = &mv.x;
    float* vp = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gr = gp[k] * clip;
      pp[k] *= decay;
      mp[k] = b1 * mp[k] + omb1 * gr;
      vp[k] = b2 * vp[k] + omb2 * gr * gr;
      const float denom = sqrtf(vp[k]) / bc2_sqrt + p.eps;
      pp[k] -= step_size * mp[k] / denom;
    }
    reinterpret_cast<float4*>(p.param)[i] = pv;
    reinterpret_cast<float4*>(p.m)[i] = mv;
    reinterpret_cast<float4*>(p.v)[i] = vv;
  }
}

// ----------------------------------------------------------------------------- tensor-list form
// The same two passes over parameters that stay separate tensors (gradients as autograd hands them
// over). The m / v index space is split into 4-element chunks; tensor k owns the chunks from off_k / 4
// on, and chunks past its n elements (its padding, or a tensor without a gradient left out of the
// table) belong to no one. A thread walks its grid-stride chunks in increasing order with a cursor
// into the table.
__device__ __forceinline__ int find_tensor(const AdamListParams& p, int64_t e) {
  int lo = 0, hi = p.nt - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.t[mid].off <= e) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(256) adamw_list_sumsq_kernel(const __grid_constant__ AdamListParams p) {
  __shared__ double red[8];
  double acc = 0.0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int k = i < p.n4 ? find_tensor(p, 4 * i) : 0;
  while (i < p.n4) {
    while (k + 1 < p.nt && p.t[k + 1].off <= 4 * i) ++k;
    // tensor k's entry in registers for all of this thread's chunks inside it
    const int64_t off = p.t[k].off, n = p.t[k].n;
    if (4 * i < off || 4 * i >= off + n) { i += stride; continue; }   // a chunk nobody owns
    const float* grad = p.t[k].grad;
    // 16-byte loads where the tensor allows them (a gradient inside a DDP bucket may start anywhere)
    const bool vec = (reinterpret_cast<uintptr_t>(grad) & 15u) == 0;
    const int64_t end = (off + n + 3) / 4, full = vec ? (off + (n & ~(int64_t)3)) / 4 : off / 4;
    for (; i + (kSumsqLoads - 1) * stride < full; i += kSumsqLoads * stride) {   // loads in flight, chunk order
      float4 v[kSumsqLoads];
#pragma unroll
      for (int u = 0; u < kSumsqLoads; ++u)
        v[u] = *reinterpret_cast<const float4*>(grad + (4 * (i + u * stride) - off));
#pragma unroll
      for (int u = 0; u < kSumsqLoads; ++u)
        acc += (double)v[u].x * v[u].x + (double)v[u].y * v[u].y + (double)v[u].z * v[u].z + (double)v[u].w * v[u].w;
    }
    for (; i < full; i += stride) {
      const float4 v = *reinterpret_cast<const float4*>(grad + (4 * i - off));
      acc += (double)v.x * v.x + (double)v.y * v.y + (double)v.z * v.z + (double)v.w * v.w;
    }
    for (; i < end; i += stride) {           // the tensor's last, partial chunk (every chunk if unaligned)
      const int64_t loc = 4 * i - off, stop = loc + 4 < n ? loc + 4 : n;
      for (int64_t j = loc; j < stop; ++j) acc += (double)grad[j] * grad[j];
    }
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < 8; ++w) t += red[w];
    p.partials[blockIdx.x] = t;
    if (blockIdx.x == 0) *p.step += 1.f;
  }
}

__global__ void __launch_bounds__(256) adamw_list_update_kernel(const __grid_constant__ AdamListParams p) {
  __shared__ float s_clip;
  if (threadIdx.x < 32) clip_from_partials(p.partials, p.npart, p.max_norm, p.status, &s_clip);
  __syncthreads();
  const float clip = s_clip;
  const float t = *p.step;
  const float bc1 = 1.f - powf(p.beta1, t), bc2 = 1.f - powf(p.beta2, t);
  const float bc2_sqrt = sqrtf(bc2);
  const float b1 = p.beta1, b2 = p.beta2, omb1 = 1.f - p.beta1, omb2 = 1.f - p.beta2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int k = i < p.n4 ? find_tensor(p, 4 * i) : 0;
  // one chunk of 4 elements (cnt of them real); the arithmetic of the flat kernel
  auto update = [&](float* pv, const float* gv, int64_t ci, float decay, float step_size) {
    float4 mv = reinterpret_cast<float4*>(p.m)[ci];
    float4 vv = reinterpret_cast<float4*>(p.v)[ci];
    float* mp = &mv.x;
    float* vp = &vv.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gr = gv[j] * clip;
      pv[j] *= decay;
      mp[j] = b1 * mp[j] + omb1 * gr;
      vp[j] = b2 * vp[j] + omb2 * gr * gr;
      const float denom = sqrtf(vp[j]) / bc2_sqrt + p.eps;
      pv[j] -= step_size * mp[j] / denom;
    }
    reinterpret_cast<float4*>(p.m)[ci] = mv;
    reinterpret_cast<float4*>(p.v)[ci] = vv;
  };
  while (i < p.n4) {
    while (k + 1 < p.nt && p.t[k + 1].off <= 4 * i) ++k;
    // tensor k's entry in registers for all of this thread's chunks inside it
    const int64_t off = p.t[k].off, n = p.t[k].n;
    if (4 * i < off || 4 * i >= off + n) { i += stride; continue; }   // a chunk nobody owns
    float* param = p.t[k].param;
    const float* grad = p.t[k].grad;
    const float decay = 1.f - p.t[k].lr * p.t[k].weight_decay, step_size = p.t[k].lr / bc1;
    const bool vec = ((reinterpret_cast<uintptr_t>(param) | reinterpret_cast<uintptr_t>(grad)) & 15u) == 0;
    const int64_t end = (off + n + 3) / 4, full = vec ? (off + (n & ~(int64_t)3)) / 4 : off / 4;
    for (; i < full; i += stride) {
      const int64_t loc = 4 * i - off;
      const float4 a = *reinterpret_cast<const float4*>(param + loc);
      const float4 b = *reinterpret_cast<const float4*>(grad + loc);
      float pv[4] = {a.x, a.y, a.z, a.w};
      const float gv[4] = {b.x, b.y, b.z, b.w};
      update(pv, gv, i, decay, step_size);
      *reinterpret_cast<float4*>(param + loc) = make_float4(pv[0], pv[1], pv[2], pv[3]);
    }
    for (; i < end; i += stride) {           // the tensor's last, partial chunk (every chunk if unaligned)
      const int64_t loc = 4 * i - off;
      const int cnt = n - loc < 4 ? (int)(n - loc) : 4;
      float pv[4], gv[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        pv[j] = j < cnt ? param[loc + j] : 0.f;
        gv[j] = j < cnt ? grad[loc + j] : 0.f;
      }
      update(pv, gv, i, decay, step_size);
      for (int j = 0; j < cnt; ++j) param[loc + j] = pv[j];
    }
  }
}

}  // namespace optim

cudaError_t launch_adamw_list(const AdamListParams& p, cudaStream_t st) {
  if (p.n4 == 0 || p.nt == 0) return cudaSuccess;
  optim::adamw_list_sumsq_kernel<<<p.npart, 256, 0, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  optim::adamw_list_update_kernel<<<p.nblocks, 256, 0, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_adamw(const AdamParams& p, cudaStream_t st) {
  if (p.n4 == 0) return cudaSuccess;
  optim::adamw_sumsq_kernel<<<p.npart, 256, 0, st>>>(p.grad, p.n4, p.partials, p.step);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const size_t smem = (size_t)p.nseg * sizeof(AdamSeg);
  if (smem > 48 * 1024) {
    e = cudaFuncSetAttribute(optim::adamw_update_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  optim::adamw_update_kernel<<<p.nblocks, 256, smem, st>>>(p);
  return cudaGetLastError();
}

}  // namespace sisa
