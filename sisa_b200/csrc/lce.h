// Host-side launch parameters of the linear + cross-entropy kernels (lce.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace sisa {

struct LceParams {
  CUtensorMap tm_x;        // (D, R) rows of the chunk, box (64, 128), 128B swizzle
  CUtensorMap tm_w;        // (D, Vp) padded weight rows, box (64, 256), 128B swizzle
  char* logits;            // (R, ld) low precision, row-major
  int64_t ld;
  float2* part;            // (R, n_nblk) {max, sum 2^(x log2e - max)} in log2 units
  float* tgt;              // (R) target logit
  const int64_t* labels;   // (R)
  int R, D, V, Vp, n_mblk, n_nblk;
  int32_t* status;
};

struct LceGradParams {
  char* logits;
  int64_t ld;
  const float2* part;
  const float* tgt;
  const int64_t* labels;
  const float* inv_n;      // device scalar 1 / (number of non-ignored rows of the whole call)
  float gscale;
  float* loss_rows;
  int64_t ignore_index;
  int R, V, Vp, n_nblk, compute_grad;
  int32_t* status;
};

cudaError_t launch_lce_logits(const LceParams& p, int dtype, int num_sms, cudaStream_t st);
cudaError_t launch_lce_grad(const LceGradParams& p, int dtype, cudaStream_t st);

}  // namespace sisa
