// optim.cu - AdamW with global-norm gradient clipping over flat fp32 buffers: the training step's
// `clip_grad_norm_` + `torch.optim.AdamW` (examples/train_minimal.py:253-301 of the reference) as two
// passes over the parameters' one contiguous layout instead of per-tensor launches.
//
// Pass 1 (adamw_sumsq_kernel): sum of squared gradients, fp64, a fixed grid and a fixed order
// (deterministic); block 0 also advances the step counter. Pass 2 (adamw_update_kernel): every block
// sums the pass-1 partials in the same order, forms the clip factor min(1, max_norm / (norm + 1e-6)),
// and updates its float4 chunks: decoupled weight decay p *= 1 - lr wd, then m, v and the bias-corrected
// step, with (lr, wd) of the parameter group the chunk belongs to (segments, binary search in shared
// memory; every segment is a multiple of 4 elements, so a float4 never straddles two).
#include <cuda_runtime.h>

#include <cstdint>

#include "optim.h"
#include "status.h"

namespace sisa {
namespace optim {

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(256) adamw_sumsq_kernel(const float* __restrict__ g, int64_t n4, double* partials,
                                                          float* step) {
  __shared__ double red[8];
  double acc = 0.0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
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
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < p.npart; ++i) t += p.partials[i];
    const double norm = sqrt(t);
    float clip = 1.f;
    if (p.max_norm > 0.f) {
      const double c = (double)p.max_norm / (norm + 1e-6);
      clip = c < 1.0 ? (float)c : 1.f;
    }
    if (!isfinite(norm) && p.status) atomicOr(p.status, SISA_ST_NONFINITE);
    s_clip = clip;
  }
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

}  // namespace optim

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
