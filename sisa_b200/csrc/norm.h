// Host-side launch descriptors of the fused RMSNorm and SwiGLU kernels (norm.cu).
// dtype codes: 0 bf16, 1 fp16, 2 fp32.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace sisa {

struct RmsNormFwd {
  const void* x; int64_t xs; int x_dtype;
  const float* w;
  int64_t rows, d;
  float eps;
  void* y; int64_t ys; int y_dtype;
  float* rstd;
};

struct RmsNormBwd {
  const void* dy; int64_t dys; int dy_dtype;
  const void* x; int64_t xs; int x_dtype;
  const float* w;
  const float* rstd;
  int64_t rows, d;
  void* dx; int64_t dxs; int dx_dtype;
  float* dw;      // (d,) or null (no weight gradient)
  float* part;    // workspace: rmsnorm_splits(rows) x d floats
};

struct SwiGluFwd {
  const void* g; int64_t gs;
  const void* u; int64_t us;
  int64_t rows, f;
  void* a; int64_t as;
  int dtype;
};

struct SwiGluBwd {
  const void* da; int64_t das;
  const void* g; int64_t gs;
  const void* u; int64_t us;
  int64_t rows, f;
  void* dg; int64_t dgs;
  void* du; int64_t dus;
  int dtype;
};

int64_t rmsnorm_splits(int64_t rows);
cudaError_t launch_rmsnorm_fwd(const RmsNormFwd& p, cudaStream_t st);
cudaError_t launch_rmsnorm_bwd(const RmsNormBwd& p, cudaStream_t st);
cudaError_t launch_swiglu_fwd(const SwiGluFwd& p, cudaStream_t st);
cudaError_t launch_swiglu_bwd(const SwiGluBwd& p, cudaStream_t st);

}  // namespace sisa
