// Host-side launch parameters of the incremental-decode kernels (decode.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace sisa {

struct DecodeParams {
  const char* q;  int64_t q_sb, q_sh;     // (B, H, 1, 64) low precision
  const char* c;  int64_t c_sb, c_sh;     // (B, H, 1, 32)
  const float* g_q;                        // (B, H) contiguous
  const float* f_q;                        // (B, H) contiguous or null
  const char* k;  int64_t k_sb, k_sh, k_sl;
  const char* v;  int64_t v_sb, v_sh, v_sl;
  const char* bm; int64_t b_sb, b_sh, b_sl;
  const float* g;                          // (B*H, gf_stride) fp32, first N valid
  const float* f;                          // same layout or null
  int64_t gf_stride;
  const float* lam;
  char* y; int64_t y_sb, y_sh;             // (B, H, 1, 64) low precision
  float* ws;                               // (splits, B*H, 66) fp32
  int B, H, N, splits;
  int32_t* status;
};

int decode_splits(int64_t B, int64_t H, int64_t N);
cudaError_t launch_decode(const DecodeParams& p, int dtype, cudaStream_t st);

}  // namespace sisa
