// embed.cu - the token embedding's weight gradient, deterministic and without a sort.
//
// dW[v, :] = sum over positions i with ids[i] = v of grad[i, :], for the (V, D) fp32 embedding of
// src/sisa/modeling.py (nn.Embedding, whose weight the LM head shares). torch computes it by sorting the
// ids, finding segments and summing them in several launches. Here block c owns vocabulary rows
// [c R, (c + 1) R): it zeroes them, scans all ids in position order, collects the positions that fall in
// its rows (an ordered compaction in shared memory), and adds those gradient rows into its rows in
// increasing position order. Each (row, column) is summed by one thread in position order, so the result
// is the same bits on every run, with no atomics; the scan of the ids costs each block N ids from L2,
// which bounds the entry point to moderate N (a training batch: 16 K tokens).
#include <cuda_runtime.h>

#include <cstdint>

#include "embed.h"

namespace sisa {
namespace embed {

constexpr int kThreads = 256;
constexpr int kList = 2048;          // positions collected before they are added (then the scan goes on)

// dw[row[k], :] += grad[pos[k], :] for k = 0 .. count-1 in order, this thread's 16-byte columns: the
// gradient rows of four entries are loaded together, the read-modify-writes of dw stay in list order.
__device__ __forceinline__ void add_rows(const EmbedBwd& p, const int* pos, const int* row, int count, int tid,
                                         int nv4) {
  for (int k0 = 0; k0 < count; k0 += 4) {
    const int kn = count - k0 < 4 ? count - k0 : 4;
    for (int c = tid; c < nv4; c += kThreads) {
      float4 a[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (j < kn) a[j] = reinterpret_cast<const float4*>(p.grad + (int64_t)pos[k0 + j] * p.grad_ld)[c];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (j < kn) {
          float4* w = reinterpret_cast<float4*>(p.dw + (int64_t)row[k0 + j] * p.D) + c;
          float4 b = *w;
          b.x += a[j].x; b.y += a[j].y; b.z += a[j].z; b.w += a[j].w;
          *w = b;
        }
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads) embed_bwd_kernel(EmbedBwd p) {
  __shared__ int s_pos[kList];
  __shared__ int s_row[kList];
  __shared__ int s_warp[kThreads / 32];
  __shared__ int s_count;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t v0 = (int64_t)blockIdx.x * p.rows_per_block;
  const int64_t v1 = v0 + p.rows_per_block < p.V ? v0 + p.rows_per_block : p.V;
  if (v0 >= v1) return;
  const int nv4 = (int)(p.D / 4);
  // zero this block's rows; thread t keeps the same 16-byte columns for the zeroing and the sums below
  for (int64_t v = v0; v < v1; ++v)
    for (int c = tid; c < nv4; c += kThreads)
      reinterpret_cast<float4*>(p.dw + v * p.D)[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (tid == 0) s_count = 0;
  __syncthreads();
  for (int64_t base = 0; base < p.n; base += kThreads) {
    // ordered compaction of this chunk's matching positions
    const int64_t i = base + tid;
    const int64_t id = i < p.n ? p.ids[i] : -1;
    const bool hit = id >= v0 && id < v1;
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    if (lane == 0) s_warp[warp] = __popc(m);
    __syncthreads();
    int before = 0, total = 0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) {
      before += w < warp ? s_warp[w] : 0;
      total += s_warp[w];
    }
    const int count = s_count;
    if (count + total > kList) {
      // the list is full: add what it holds first (every thread walks the same list in order)
      add_rows(p, s_pos, s_row, count, tid, nv4);
      __syncthreads();
      if (hit) {
        const int slot = before + __popc(m & ((1u << lane) - 1u));
        s_pos[slot] = (int)i;
        s_row[slot] = (int)id;
      }
      __syncthreads();
      if (tid == 0) s_count = total;
    } else {
      if (hit) {
        const int slot = count + before + __popc(m & ((1u << lane) - 1u));
        s_pos[slot] = (int)i;
        s_row[slot] = (int)id;
      }
      __syncthreads();
      if (tid == 0) s_count = count + total;
    }
    __syncthreads();
  }
  add_rows(p, s_pos, s_row, s_count, tid, nv4);
}

}  // namespace embed

cudaError_t launch_embed_bwd(const EmbedBwd& p0, int num_sms, cudaStream_t st) {
  EmbedBwd p = p0;
  if (p.V == 0) return cudaSuccess;
  int64_t blocks = 4 * (int64_t)num_sms;
  if (blocks > p.V) blocks = p.V;
  p.rows_per_block = (p.V + blocks - 1) / blocks;
  blocks = (p.V + p.rows_per_block - 1) / p.rows_per_block;
  embed::embed_bwd_kernel<<<(unsigned)blocks, embed::kThreads, 0, st>>>(p);
  return cudaGetLastError();
}

}  // namespace sisa
