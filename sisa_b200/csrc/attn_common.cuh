// attn_common.cuh - shared definitions of the tcgen05 SISA attention kernels.
//
// Score (reference: src/sisa/kernels/attention.py:1-107, src/sisa/functional.py:69-103):
//   s_ij = q_i.k_j / sqrt(64) + lam_h exp(g_i - g_j) (c_i.b_j) + (F_i - F_j),   j <= i
// kept in log2 units inside the kernels: x_ij = s_ij * log2(e).
//
// Decay factorisation (attention.py:11-22): for a key block that ends before the query block starts,
//   exp(g_i - g_j) = rowf_i * mid * colf_j   with every factor <= 1,
// applied in fp32 after the c.b GEMM (the GEMM runs on the unscaled bf16 operands). The factors
// relative to 64-row blocks come precomputed in the position records {g, F, rowf64, colf64}; the
// kernel's own 128-row tile anchors its side of the factorisation itself. Tiles that intersect
// the diagonal use the pairwise exp2(min((g_i - g_j) log2e, 0)).
#pragma once
#include <cuda.h>
#include <cstdint>

#include "sm100.cuh"

namespace sisa {

constexpr int kD = 64;        // head dimension
constexpr int kDS = 32;       // state dimension
constexpr float kLOG2E = 1.4426950408889634f;
constexpr float kScale = 0.125f;          // 1/sqrt(64)

// Shared-memory descriptors of the operand tiles used by the attention kernels.
//  - K-major tile of 64-element (128-byte) rows, 128-byte swizzle: SBO = 1024 (8 rows).
//  - K-major tile of 32-element (64-byte) rows, 64-byte swizzle: SBO = 512.
//  - MN-major tile whose rows (the K index) are 128 bytes = 64 MN elements, 128-byte swizzle:
//    8-row groups at SBO = 1024; one UMMA K-step (16 rows) is 2048 bytes.
//  - MN-major tile with 64-byte rows (32 MN elements), 64-byte swizzle: SBO = 512; K-step 1024.
__device__ __forceinline__ uint64_t desc_k128(uint32_t saddr) { return make_sdesc(saddr, 16, 1024, SW_128B); }
__device__ __forceinline__ uint64_t desc_k64(uint32_t saddr) { return make_sdesc(saddr, 16, 512, SW_64B); }
__device__ __forceinline__ uint64_t desc_mn128(uint32_t saddr) { return make_sdesc(saddr, 8192, 1024, SW_128B); }
__device__ __forceinline__ uint64_t desc_mn64(uint32_t saddr) { return make_sdesc(saddr, 4096, 512, SW_64B); }

// tcgen05 TMEM address of (warp's lane quarter, column).
__device__ __forceinline__ uint32_t tmem_addr(uint32_t base, int warp_quarter, int col) {
  return base + ((uint32_t)(warp_quarter * 32) << 16) + (uint32_t)col;
}

// Work order of the attention kernels: heads are taken in groups of 16, and within a group every
// head's heaviest tile goes out before any lighter one. Light tiles then finish the kernel (a short
// last wave), while at any time only about one group's K/V/B~ tiles (16 heads, ~22 MB at L = 4096) are
// live in L2. Maps the linear work index to (bh, rank); rank 0 is the heaviest tile.
__device__ __forceinline__ void tile_order_lin(int lin, int ntile, int BH, int& bh, int& rank) {
  constexpr int GH = 16;
  const int full = BH / GH, per = GH * ntile;
  const int g = lin / per;
  if (g < full) {
    const int k = lin - g * per;
    rank = k / GH;
    bh = g * GH + k % GH;
  } else {
    const int rem = BH - full * GH, k = lin - full * per;
    rank = k / rem;
    bh = full * GH + k % rem;
  }
}

// The same order for a grid of (ntile, B*H) blocks, dispatched in linear order.
__device__ __forceinline__ void tile_order(int ntile, int BH, int& bh, int& rank) {
  tile_order_lin((int)blockIdx.x + (int)gridDim.x * (int)blockIdx.y, ntile, BH, bh, rank);
}

// Warp-uniform bounded wait used by the compute warps.
template <bool kSleep = false>
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, int32_t* status) {
  const bool ok = mbar_wait<kSleep>(bar, parity, status);
  return __all_sync(0xffffffffu, ok);
}

// The same, testing the phase once without blocking before it waits: for warps whose phases have
// usually completed by the time they ask, and which have few other warps to hide a wait's latency.
template <bool kSleep = false>
__device__ __forceinline__ bool warp_wait_tested(uint32_t bar, uint32_t parity, int32_t* status) {
  bool ok = mbar_test(bar, parity);
  if (!ok) ok = mbar_wait<kSleep>(bar, parity, status);
  return __all_sync(0xffffffffu, ok);
}

}  // namespace sisa
