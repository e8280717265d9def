// gate_math.cuh - the scalar gate functions of the preparation and decode kernels, as torch computes
// them (softplus with threshold 20, log-sigmoid, and their derivatives).
#pragma once
#include <cmath>

namespace sisa {

__device__ __forceinline__ float neg_softplus(float a) {       // torch softplus, threshold 20
  return -(a > 20.f ? a : log1pf(expf(a)));
}
__device__ __forceinline__ float softplus_grad(float a) {      // torch softplus_backward
  if (a > 20.f) return 1.f;
  const float e = expf(a);
  return e / (e + 1.f);
}
__device__ __forceinline__ float logsigmoid(float z) {         // torch log_sigmoid_forward; NaN propagates
  const float m = (z != z) ? z : fminf(z, 0.f);
  return m - log1pf(expf(-fabsf(z)));
}
__device__ __forceinline__ float logsigmoid_grad(float z) {    // torch log_sigmoid_backward
  const float e = expf(-fabsf(z));
  const float r = e / (1.f + e);
  return z < 0.f ? 1.f - r : r;
}

}  // namespace sisa
