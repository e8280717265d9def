// Host-side launch parameters of the batched weight-copy kernel (copy.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace sisa {

// One row-block copy; the same layout as sisa_row_copy.
struct RowCopy {
  const float* src;            // null: zero-fill the destination rows
  void* dst;
  int64_t rows, cols, src_ld, dst_ld;
  int64_t block_rows, dst_block_stride;
};

// jobs: njobs entries in device memory; max_vectors: the largest rows * cols / 8 among them.
cudaError_t launch_copy_rows(const RowCopy* jobs, int njobs, int64_t max_vectors, int dtype, cudaStream_t st);

// Per-head rows of 16-bit elements between two (batch, head, position) layouts (element strides).
struct HeadsCopy {
  const void* src;
  int64_t ssb, ssh, ssl;
  void* dst;
  int64_t dsb, dsh, dsl;
  int64_t B, H, L, width;
};
cudaError_t launch_copy_heads(const HeadsCopy& p, int num_sms, cudaStream_t st);

// Rows of fp32 values taken out of a buffer that interleaves two matrices in blocks of `block` rows
// (block of matrix 0, block of matrix 1, ...): dst_h row r = src row (r / block) 2 block + h block + r % block.
struct SplitRows {
  const float* src;
  float* dst0;
  float* dst1;
  int64_t rows, cols, src_ld, dst_ld, block;     // rows of each destination
};
cudaError_t launch_split_rows(const SplitRows& p, int num_sms, cudaStream_t st);

}  // namespace sisa
