// Host-side launch parameters of the embedding weight-gradient kernel (embed.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace sisa {

struct EmbedBwd {
  const int64_t* ids;      // n token ids; ids outside [0, V) add nothing
  const float* grad;       // n rows of D fp32 values, row stride grad_ld
  float* dw;               // V x D fp32, contiguous: written entirely
  int64_t n, V, D, grad_ld;
  int64_t rows_per_block;  // set by the launcher
};
cudaError_t launch_embed_bwd(const EmbedBwd& p, int num_sms, cudaStream_t st);

}  // namespace sisa
