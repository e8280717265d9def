// Host-side launch parameters of the flat AdamW kernels (optim.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace sisa {

// One parameter (or run of parameters of one group) in the flat layout: elements [start, end), both
// multiples of 4, with its group's learning rate and weight decay. Same layout as sisa_adam_seg.
struct AdamSeg {
  int64_t start, end;
  float lr, weight_decay;
};

struct AdamParams {
  float* param;            // fp32, n4 * 4 elements each
  const float* grad;
  float* m;
  float* v;
  int64_t n4;
  const AdamSeg* segs;     // device, sorted by start
  int nseg;
  float* step;             // device step counter (advanced by the first pass)
  double* partials;        // npart doubles
  int npart, nblocks;
  float beta1, beta2, eps, max_norm;
  int32_t* status;
};

cudaError_t launch_adamw(const AdamParams& p, cudaStream_t st);

// One parameter tensor of the tensor-list form; the same layout as sisa_adam_tensor.
struct AdamTensor {
  float* param;            // n fp32 values (16-byte loads where 16-byte aligned)
  const float* grad;       // n fp32 values
  int64_t off, n;          // its first element in m / v (a multiple of 4) and its size
  float lr, weight_decay;
};

// The table travels by value in the kernels' parameters (no device copy, captured with a graph).
constexpr int kMaxAdamTensors = 384;
struct AdamListParams {
  AdamTensor t[kMaxAdamTensors];   // sorted by off
  int nt;
  float* m;
  float* v;
  int64_t n4;              // 4-element chunks of m / v covered by the table
  float* step;
  double* partials;
  int npart, nblocks;
  float beta1, beta2, eps, max_norm;
  int32_t* status;
};

cudaError_t launch_adamw_list(const AdamListParams& p, cudaStream_t st);

}  // namespace sisa
