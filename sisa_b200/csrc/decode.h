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
  int B, H, N, splits;                     // with d_pos: N is the largest key count the caches hold
  int32_t* status;
  const int32_t* d_pos;                    // null, or the new position on the device: N = *d_pos + 1 keys
};

// One decode step's layer input from the fused projection row (decode_prep_kernel).
struct DecodePrepParams {
  const uint16_t* proj; int64_t proj_sb;        // (B, NPAD) low precision, row stride in elements
  const float* z; int64_t z_sb;                 // (B, H) forget logits or null
  int col_k, col_v, col_b, col_c, col_th, col_a;
  uint16_t* k; int64_t k_sb, k_sh, k_sl;        // caches, element strides; the new row goes to pos
  uint16_t* v; int64_t v_sb, v_sh, v_sl;
  uint16_t* bm; int64_t b_sb, b_sh, b_sl;
  float* g; float* f; int64_t gf_stride;        // (B*H, gf_stride); f null without forget logits
  float* phi;                                   // (B, H, 16) contiguous, advanced in place
  uint16_t* c_out;                              // (B, H, 32) contiguous
  float* g_out; float* f_out;                   // (B, H)
  int B, H;
  int64_t pos;
  const int32_t* d_pos;                         // null, or the position on the device (replaces pos)
  int64_t max_pos;                              // with d_pos: positions must lie in [1, max_pos)
  int32_t* status;                              // with d_pos: SISA_ST_BAD_POS for a position out of range
};

int decode_splits(int64_t B, int64_t H, int64_t N);
cudaError_t launch_decode(const DecodeParams& p, int dtype, cudaStream_t st);
cudaError_t launch_decode_prep(const DecodePrepParams& p, int dtype, cudaStream_t st);

}  // namespace sisa
