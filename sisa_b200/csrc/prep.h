// Host-side launch descriptors of the preparation kernels (prep.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace sisa {

struct PrepFwdLaunch {
  const void* proj;
  int64_t proj_sb, proj_sl;
  int dtype;
  const float* z;
  int64_t z_sb, z_sl;
  int64_t B, L, H;
  int64_t col_b, col_c, col_th, col_a;
  void* c_rot;
  void* b_rot;
  float* pos;      // (B*H, 4, Lp) planes
  int64_t Lp;
  float* tot;
  int32_t* status;
};

struct PackLaunch {
  const float* g;
  int64_t g_sb, g_sh, g_sl;
  const float* f;
  int64_t f_sb, f_sh, f_sl;
  int64_t B, H, L, Lp;
  float* pos;
  int32_t* status;
};

struct PrepBwdLaunch {
  const void* proj;
  int64_t proj_sb, proj_sl;
  int dtype;
  const float* z;
  int64_t z_sb, z_sl;
  int64_t B, L, H;
  int64_t col_b, col_c, col_th, col_a, ntot, npad;
  const float* tot;
  const float* dc;
  const float* db;
  const float* dg;
  const float* dF;
  void* dproj;
  int64_t dproj_sb, dproj_sl;
  float* dz;
  double* bt;
  int32_t* status;
};

cudaError_t launch_prep_fwd(const PrepFwdLaunch& p, cudaStream_t st);
cudaError_t launch_pack_positions(const PackLaunch& p, cudaStream_t st);
cudaError_t launch_prep_bwd(const PrepBwdLaunch& p, cudaStream_t st);

}  // namespace sisa
