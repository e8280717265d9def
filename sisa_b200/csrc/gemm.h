// Host-side launch parameters of the CTA-pair tcgen05 GEMM (gemm.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace sisa {

struct GemmParams {
  // A: M x K, B: N x K (C = A B^T). Each is K-major (element (r, k) at r * ld + k) or MN-major
  // (element (r, k) at k * ld + r). The tensor maps load one CTA's half tile per stage: 128 rows x 64 K.
  CUtensorMap tm_a, tm_b;
  CUtensorMap tm_c;     // C: M x N row-major; box 32 rows x 128 bytes, 128-byte swizzle
  int64_t ldc;
  int M, N, K;
  int num_m, num_n;     // 256-row pair tiles along M, tiles along N (set by launch_gemm for its tile width)
  int accumulate;       // fp32 output only: C += A B^T (TMA reduce-add)
  int32_t* status;
  // linear-CE logits epilogue only: per (row, 64-column segment) online {max, sum 2^(x log2 e - max)}
  // over the columns below V (part[row * n_part + col / 64]), and the label's logit (tgt[row])
  const int64_t* labels;
  float2* part;
  float* tgt;
  int V, n_part;
};

enum GemmOut : int { GEMM_OUT_F32 = 0, GEMM_OUT_BF16 = 1, GEMM_OUT_F16 = 2 };
enum GemmEpilogue : int { EPI_STORE = 0, EPI_LCE = 1 };

// in_dtype: 0 bf16, 1 fp16 operands; a_mn / b_mn: operand majorness; out: GemmOut; wide: 256 x 512
// pair tiles (else 256 x 256).
cudaError_t launch_gemm(const GemmParams& p, int in_dtype, int a_mn, int b_mn, int out, int wide, int num_sms,
                        cudaStream_t st);
// The linear-CE logits: C (bf16/fp16 as in_dtype) = A B^T with both operands K-major, narrow tiles, and
// the EPI_LCE epilogue.
cudaError_t launch_lce_logits_gemm(const GemmParams& p, int in_dtype, int num_sms, cudaStream_t st);

}  // namespace sisa
