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
  CUtensorMap tm_c2;    // SwiGLU epilogue: a (M x N / 2); box 32 rows x 64 bytes, 64-byte swizzle
  int64_t ldc;
  int M, N, K;
  int num_m, num_n;     // 256-row pair tiles along M, tiles along N (set by launch_gemm for its tile width)
  int accumulate;       // fp32 output only: C += A B^T (TMA reduce-add)
  int32_t* status;
  const void* bias;     // optional, per column of C, added in fp32 before the output rounding
  int bias_dtype;       // 0 bf16, 1 fp16, 2 fp32
  // the bias covers columns [bias_c0, bias_c1) (bias[c - bias_c0]; zero elsewhere); bias_vec: 16-byte
  // loads allowed (aligned pointer, bias_c0 a multiple of 8); bias_round: round each bias value to the
  // 16-bit output type before the add
  int bias_c0, bias_c1, bias_vec, bias_round;
  // split-K (fp32 output, narrow tiles): K is cut into k_split slices of kb_split 64-wide blocks; each
  // slice writes its partial to the workspace and the last of a tile's slices (counted in sema, zero at
  // launch) sums them in slice order and stores C
  int k_split, kb_split;
  uint32_t* sema;       // the workspace (counters, then partials); null: no split
  int64_t ws_bytes;
  float* partials;
  // linear-CE logits epilogue only: per (row, 256-column tile) online {max, sum 2^(x log2 e - max)}
  // over the columns below V (part[row * n_part + col / 256]), and the label's logit (tgt[row])
  const int64_t* labels;
  float2* part;
  float* tgt;
  int V, n_part;
  int skip_c;           // SwiGLU epilogue: store only the activation (inference), not C
};

enum GemmOut : int { GEMM_OUT_F32 = 0, GEMM_OUT_BF16 = 1, GEMM_OUT_F16 = 2 };
enum GemmEpilogue : int { EPI_STORE = 0, EPI_LCE = 1, EPI_SWIGLU = 2 };

// in_dtype: 0 bf16, 1 fp16 operands; a_mn / b_mn: operand majorness; out: GemmOut.
// tile: -1 chooses between the tile shapes and a split of K from the problem's size (a split needs an
// fp32 output and a workspace p.sema of gemm_workspace_bytes(M, N, K, out) bytes); 0 narrow, 1 wide
// (no split).
cudaError_t launch_gemm(const GemmParams& p, int in_dtype, int a_mn, int b_mn, int out, int tile, int num_sms,
                        cudaStream_t st);
int64_t gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int out, int num_sms);
// The linear-CE logits: C (bf16/fp16 as in_dtype) = A B^T with both operands K-major, narrow tiles, and
// the EPI_LCE epilogue.
cudaError_t launch_lce_logits_gemm(const GemmParams& p, int in_dtype, int num_sms, cudaStream_t st);
// The SwiGLU gate and up projections: C (gate and up outputs, interleaved in blocks of 8 columns) = A B^T
// and a = silu(gate) up to tm_c2, both operands K-major, narrow tiles, the EPI_SWIGLU epilogue.
cudaError_t launch_gemm_swiglu(const GemmParams& p, int in_dtype, int num_sms, cudaStream_t st);

}  // namespace sisa
