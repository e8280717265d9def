// Host-side launch descriptors of the fused RMSNorm and SwiGLU kernels (norm.cu).
// dtype codes: 0 bf16, 1 fp16, 2 fp32.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace sisa {

// One RMSNorm at a block boundary: v = x (+ res, rounded to x's type; written to xsum), rstd =
// rsqrt(mean(v^2) + eps), h = (v rstd) w rounded to x's type (the reference's output), stored once per
// output in that output's type, and optionally z = h proj_w^T + proj_b in fp32 (np <= 32 columns).
struct NormFwd {
  const void* x; int64_t xs; int xdt;
  const void* res; int64_t ress; int resdt;   // null: no residual add
  void* xsum; int64_t xsums;                  // with res: x + res (may be null)
  const float* w;
  int64_t rows, d;
  float eps;
  int nout;                                   // 1 or 2
  void* y[2]; int64_t ys[2]; int ydt[2];
  float* rstd;
  const float* pw; const float* pb; int np; float* pz;   // np 0: no projection
  int32_t* status;                            // bounded-wait timeouts (may be null)
};

// Its backward. The gradient of h is G = sum of dy[k] (null entries skipped) + dz proj_w; then
// dv = rstd (G w - xh mean(G w xh)) + dvin with xh = v rstd, stored as dx (and dres in res's type);
// dw = sum_r G xh, dpw = sum_r dz^T h, dpb = sum_r dz, from per-split partials in a fixed order.
struct NormBwd {
  const void* v; int64_t vs; int vdt;         // the normalised rows (x, or xsum with a residual add)
  const float* w;
  const float* rstd;
  int64_t rows, d;
  const void* dy[2]; int64_t dys[2]; int dydt[2];
  const void* dvin; int64_t dvins; int dvindt;   // gradient reaching v from its other consumers (may be null)
  const float* pw; int np; const float* dz;      // dz (rows, np) fp32, null when np == 0
  void* dx; int64_t dxs; int dxdt;
  void* dres; int64_t dress; int dresdt;         // may be null
  float* dw; float* dpw; float* dpb;             // may be null (then part may be null too)
  float* part;                                   // workspace: norm_bwd_partials(rows, np) x norm_part_cols(d, np) floats
  int32_t* status;                               // bounded-wait timeouts (may be null)
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

int64_t norm_splits(int64_t rows, int64_t np);
int64_t norm_part_cols(int64_t d, int64_t np);
int64_t norm_bwd_partials(int64_t rows, int64_t np);
cudaError_t launch_norm_fwd(const NormFwd& p, cudaStream_t st);
cudaError_t launch_norm_bwd(const NormBwd& p, cudaStream_t st);
cudaError_t launch_swiglu_fwd(const SwiGluFwd& p, cudaStream_t st);
cudaError_t launch_swiglu_bwd(const SwiGluBwd& p, cudaStream_t st);

}  // namespace sisa
