// copy.cu - many fp32 -> bf16/fp16 row-block copies in one launch: the compute-dtype copies of a model's
// weights (the concatenated projection weight, the interleaved gate/up weight, the plain linears), which
// change after every optimizer step and were otherwise refreshed by one small cast kernel per weight.
//
// copy_heads_kernel moves per-head rows of 16-bit elements between two (batch, head, position)
// layouts: the prompt's keys, values and rotated B~ into a decode cache's buffers. split_rows_kernel
// takes two fp32 matrices out of a buffer that interleaves them in blocks of rows: the weight gradients
// of the gate and up projections out of the one gradient GEMM over their interleaved weight.
//
// Job j (one row of the grid's y dimension) copies source rows r = 0 .. rows-1 of `cols` fp32 values to
// destination row (r / block_rows) * dst_block_stride + r % block_rows, rounding to nearest even; a job
// without a source zero-fills its destination rows. Each thread moves 8 values at a time (two 16-byte
// loads, one 16-byte store), grid-striding over its job.
#include <cuda_runtime.h>

#include <cstdint>

#include "attn_common.cuh"
#include "copy.h"

namespace sisa {
namespace copy {

template <bool kHalf>
__global__ void __launch_bounds__(256) copy_rows_kernel(const RowCopy* __restrict__ jobs) {
  const RowCopy jb = jobs[blockIdx.y];
  const int64_t vpr = jb.cols / 8;                         // 8-value vectors per row
  const int64_t n = jb.rows * vpr;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int64_t r = i / vpr, v = i - r * vpr;
    const int64_t dr = (r / jb.block_rows) * jb.dst_block_stride + r % jb.block_rows;
    uint4 o = make_uint4(0u, 0u, 0u, 0u);
    if (jb.src) {
      const float4* s = reinterpret_cast<const float4*>(jb.src + r * jb.src_ld + 8 * v);
      const float4 a = s[0], b = s[1];
      o = make_uint4(pack2<kHalf>(a.x, a.y), pack2<kHalf>(a.z, a.w), pack2<kHalf>(b.x, b.y), pack2<kHalf>(b.z, b.w));
    }
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(jb.dst) + dr * jb.dst_ld + 8 * v) = o;
  }
}

// dst[b, h, t, 0:width] = src[b, h, t, 0:width] for 16-bit elements, both sides with their own
// (batch, head, position) strides and `width` contiguous elements (a multiple of 8): thread (x, y) of a
// block takes 16-byte vector x of position row y, the vectors of all heads of a position side by side.
__global__ void __launch_bounds__(256) copy_heads_kernel(HeadsCopy p) {
  const int nv = (int)(p.width / 8), per_row = (int)p.H * nv;
  const int j = threadIdx.x;
  if (j >= per_row) return;
  const int h = j / nv, v = j - h * nv;
  const int64_t rows = p.B * p.L;
  for (int64_t r = (int64_t)blockIdx.x * blockDim.y + threadIdx.y; r < rows; r += (int64_t)gridDim.x * blockDim.y) {
    const int64_t b = r / p.L, t = r - b * p.L;
    const uint4 x = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.src) + b * p.ssb + h * p.ssh +
                                                    t * p.ssl + 8 * v);
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.dst) + b * p.dsb + h * p.dsh + t * p.dsl + 8 * v) = x;
  }
}

// dst_h[r, :] = src[(r / block) 2 block + h block + r % block, :]: thread i moves 16-byte vector i of
// the 2 * rows * cols / 4 destination vectors (the two destinations one after the other).
__global__ void __launch_bounds__(256) split_rows_kernel(SplitRows p) {
  const int64_t vpr = p.cols / 4;
  const int64_t n = 2 * p.rows * vpr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t hr = i / vpr, v = i - hr * vpr;
    const int h = hr >= p.rows ? 1 : 0;
    const int64_t r = hr - h * p.rows;
    const int64_t sr = (r / p.block) * 2 * p.block + h * p.block + r % p.block;
    const float4 x = *reinterpret_cast<const float4*>(p.src + sr * p.src_ld + 4 * v);
    *reinterpret_cast<float4*>((h ? p.dst1 : p.dst0) + r * p.dst_ld + 4 * v) = x;
  }
}

}  // namespace copy

cudaError_t launch_split_rows(const SplitRows& p, int num_sms, cudaStream_t st) {
  const int64_t n = 2 * p.rows * (p.cols / 4);
  if (n == 0) return cudaSuccess;
  int64_t grid = (n + 255) / 256;
  if (grid > 8 * (int64_t)num_sms) grid = 8 * (int64_t)num_sms;
  copy::split_rows_kernel<<<(unsigned)grid, 256, 0, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_copy_heads(const HeadsCopy& p, int num_sms, cudaStream_t st) {
  const int64_t rows = p.B * p.L;
  if (rows == 0 || p.H == 0) return cudaSuccess;
  const int per_row = (int)(p.H * (p.width / 8));
  const int tx = (per_row + 31) / 32 * 32, ty = 256 / tx > 0 ? 256 / tx : 1;
  int64_t grid = (rows + ty - 1) / ty;
  if (grid > 8 * (int64_t)num_sms) grid = 8 * (int64_t)num_sms;
  copy::copy_heads_kernel<<<(unsigned)grid, dim3(tx, ty), 0, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_copy_rows(const RowCopy* jobs, int njobs, int64_t max_vectors, int dtype, cudaStream_t st) {
  if (njobs == 0) return cudaSuccess;
  int64_t gx = (max_vectors + 2047) / 2048;                // about 8 vectors per thread for the largest job
  if (gx < 1) gx = 1;
  if (gx > 64) gx = 64;
  const dim3 grid((unsigned)gx, (unsigned)njobs);
  if (dtype == 1) copy::copy_rows_kernel<true><<<grid, 256, 0, st>>>(jobs);
  else copy::copy_rows_kernel<false><<<grid, 256, 0, st>>>(jobs);
  return cudaGetLastError();
}

}  // namespace sisa
