// Host-side launch parameters of the linear + cross-entropy kernels of lce.cu (the logits GEMM is in gemm.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace sisa {

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

cudaError_t launch_lce_grad(const LceGradParams& p, int dtype, cudaStream_t st);
// out_dtype: 0 bf16, 1 fp16, 2 fp32 (out null: in place).
cudaError_t launch_seed_scale(float* x, int64_t n, const float* seed, void* out, int out_dtype, int num_sms,
                              cudaStream_t st);

}  // namespace sisa
