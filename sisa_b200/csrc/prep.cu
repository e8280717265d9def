// prep.cu - fused SISA layer preparation (forward and backward) and the position records of the
// unfused entry point.
//
// Forward (reference: src/sisa/kernels/fused_prep.py:247-352):
//   g_t   = sum_{s<=t} -softplus(alpha_s)      (softplus threshold 20, torch formula)
//   F_t   = sum_{s<=t} logsigmoid(z_s)         (min(z,0) - log1p(exp(-|z|)))
//   Phi_t = sum_{s<=t} theta_s                  (16 pairs per head)
//   c~_t, b~_t = R(Phi_t) c_t, R(Phi_t) b_t     (interleaved pairs (0,1),(2,3)..., fp32, one rounding)
// Scans are two-level: a warp scan inside 64-row blocks plus a sequential fp32 sum of the totals of
// the preceding blocks. The block totals come from the same scan code as the in-block values, so
// the last g of a block equals the next block's prefix exactly and g stays monotone across blocks.
//
// Backward (reference: src/sisa/kernels/fused_prep.py:385-494): reverse cumulative sums in fp64
// (block totals + in-block warp scans), rounded to fp32 once; inverse rotation of dc~/db~; d theta
// from both rotations; zero padding columns. Two passes: the first recomputes Phi, writes dC and dB
// (final), the per-token d Phi (fp32 workspace) and the fp64 block totals; the second reads only dg,
// dF, alpha, z and d Phi, so the rotation inputs are read once.
//
// Layout: one CTA = one batch row b and one 64-token block; warp w handles heads w, w+8, ...;
// lane l handles tokens 2l and 2l+1 of the block. The backward's rotation pass stages its rows in
// shared memory instead (prep_brot_kernel).
#include <cuda_runtime.h>
#include <cstdint>

#include "sm100.cuh"
#include "prep.h"
#include "gate_math.cuh"

namespace sisa {

constexpr int kBlk = 64;          // rows per scan block (also the rowf/colf grouping)
constexpr int kS2 = 16;           // rotation pairs per head (d_state / 2)
constexpr int kTot = 2 + kS2;     // totals per (b, h, block): log alpha, log f, theta[16]
constexpr float kLog2e = 1.4426950408889634f;

// Read-only global loads go through the non-coherent path (ld.global.nc): the inputs are never written
// by these kernels, and the compiler may then hoist the loads above the outputs' stores instead of
// serialising every load round trip behind them.
template <bool kHalf>
__device__ __forceinline__ float ld_lp(const void* p, int64_t i) {
  const unsigned short bits = __ldg(reinterpret_cast<const unsigned short*>(p) + i);
  if constexpr (kHalf) return __half2float(__ushort_as_half(bits));
  else return __bfloat162float(__ushort_as_bfloat16(bits));
}

// Inclusive scan of a 64-element sequence held two per lane (x0 = element 2l, x1 = element 2l+1).
// s0/s1 are the inclusive prefixes of both elements; the block total is lane 31's s1.
template <typename T>
__device__ __forceinline__ void scan64(T x0, T x1, T& s0, T& s1) {
  const int lane = threadIdx.x & 31;
  T incl = x0 + x1;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const T y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl = incl + y;
  }
  T excl = __shfl_up_sync(0xffffffffu, incl, 1);
  if (lane == 0) excl = T(0);
  s0 = excl + x0;
  s1 = incl;
}

// Reverse (suffix) inclusive scan of the same 64-element arrangement: r0 = sum_{s>=2l}, r1 = sum_{s>=2l+1};
// the block total is lane 0's r0.
template <typename T>
__device__ __forceinline__ void rscan64(T x0, T x1, T& r0, T& r1) {
  const int lane = threadIdx.x & 31;
  T incl = x0 + x1;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const T y = __shfl_down_sync(0xffffffffu, incl, d);
    if (lane + d < 32) incl = incl + y;
  }
  T excl = __shfl_down_sync(0xffffffffu, incl, 1);
  if (lane == 31) excl = T(0);
  r1 = excl + x1;
  r0 = incl;
}

struct PrepArgs {
  const void* proj;
  int64_t proj_sb, proj_sl;
  const float* z;
  int64_t z_sb, z_sl;
  int B, L, H, nch;
  int col_b, col_c, col_th, col_a;
  void* c_rot;
  void* b_rot;
  float* pos;      // (B*H, 4, Lp) planes {g, F, rowf, colf}
  int Lp;
  float* tot;      // (B*H, nch, kTot)
  int32_t* status;
};

// Element values of one head for the two tokens of this lane: log alpha, log f, theta[16].
template <bool kHalf>
__device__ __forceinline__ void load_elems(const PrepArgs& a, int b, int h, int t0, float la[2], float lf[2],
                                           float th[2][kS2]) {
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int t = t0 + r;
    const bool ok = t < a.L;
    const int64_t row = (int64_t)b * a.proj_sb + (int64_t)(ok ? t : 0) * a.proj_sl;
    la[r] = ok ? neg_softplus(ld_lp<kHalf>(a.proj, row + a.col_a + h)) : 0.f;
    lf[r] = (ok && a.z) ? logsigmoid(__ldg(a.z + (int64_t)b * a.z_sb + (int64_t)t * a.z_sl + h)) : 0.f;
    const uint4* tp = reinterpret_cast<const uint4*>(
        reinterpret_cast<const char*>(a.proj) + (row + a.col_th + h * kS2) * 2);
    uint4 v0 = make_uint4(0, 0, 0, 0), v1 = make_uint4(0, 0, 0, 0);
    if (ok) { v0 = __ldg(tp); v1 = __ldg(tp + 1); }
    const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      th[r][2 * i] = unpack_lo<kHalf>(w[i]);
      th[r][2 * i + 1] = unpack_hi<kHalf>(w[i]);
    }
  }
}

// One warp per head (up to 32 heads per block; more take further rounds), so that every head's loads
// are in flight at once instead of eight warps walking the heads one after another.
template <bool kHalf>
__global__ void __launch_bounds__(1024) prep_sums_kernel(PrepArgs a) {
  const int c = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int t0 = c * kBlk + 2 * lane;
  for (int h = warp; h < a.H; h += nwarps) {
    float la[2], lf[2], th[2][kS2];
    load_elems<kHalf>(a, b, h, t0, la, lf, th);
    float s0, s1, tv[kTot];
    scan64(la[0], la[1], s0, s1);
    tv[0] = __shfl_sync(0xffffffffu, s1, 31);
    scan64(lf[0], lf[1], s0, s1);
    tv[1] = __shfl_sync(0xffffffffu, s1, 31);
#pragma unroll
    for (int p = 0; p < kS2; ++p) {
      scan64(th[0][p], th[1][p], s0, s1);
      tv[2 + p] = __shfl_sync(0xffffffffu, s1, 31);
    }
    float* dst = a.tot + ((int64_t)(b * a.H + h) * a.nch + c) * kTot;
    bool bad = false;
#pragma unroll
    for (int k = 0; k < kTot; ++k) bad |= !isfinite(tv[k]);
    if (lane < kTot) {
      float mine = tv[0];
#pragma unroll
      for (int k = 1; k < kTot; ++k) if (lane == k) mine = tv[k];
      dst[lane] = mine;
    }
    if (bad && lane == 0 && a.status) atomicOr(a.status, SISA_ST_NONFINITE);
  }
}

// Store the records of positions t0, t0 + 1 (t0 even) into the four planes {g, F, rowf, colf} of one
// (batch, head): one 8-byte store per plane when both positions exist (Lp is a multiple of 4).
__device__ __forceinline__ void store_planes(float* pl, int Lp, int t0, int L, const float g[2], const float f[2],
                                             const float rf[2], const float cf[2]) {
  if (t0 + 1 < L) {
    *reinterpret_cast<float2*>(pl + t0) = make_float2(g[0], g[1]);
    *reinterpret_cast<float2*>(pl + Lp + t0) = make_float2(f[0], f[1]);
    *reinterpret_cast<float2*>(pl + 2 * Lp + t0) = make_float2(rf[0], rf[1]);
    *reinterpret_cast<float2*>(pl + 3 * Lp + t0) = make_float2(cf[0], cf[1]);
  } else if (t0 < L) {
    pl[t0] = g[0]; pl[Lp + t0] = f[0]; pl[2 * Lp + t0] = rf[0]; pl[3 * Lp + t0] = cf[0];
  }
}

// In-place exclusive scans of the per-block totals along the block axis, one warp per (row, component)
// chain; lane j of a round of 32 blocks takes the running sum before block j is added, so the additions
// stay in block order. Forward (fp32, increasing blocks): pre[c] = ((t_0 + t_1) + ...) + t_{c-1}, the
// order of prefix_total, which keeps g non-increasing across blocks. Backward (fp64, decreasing blocks):
// suf[c] = sum of the totals of the blocks after c.
template <typename T, bool kReverse>
__global__ void __launch_bounds__(256) block_scan_kernel(T* tot, int64_t nchains, int nch) {
  const int64_t w = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (w >= nchains) return;
  const int lane = threadIdx.x & 31;
  T* base = tot + (w / kTot) * (int64_t)nch * kTot + w % kTot;
  T acc = T(0);
  for (int c0 = 0; c0 < nch; c0 += 32) {
    const bool ok = c0 + lane < nch;
    const int64_t c = kReverse ? nch - 1 - (c0 + lane) : c0 + lane;
    const T v = ok ? base[c * kTot] : T(0);
    T mine = acc;
    const int n = min(32, nch - c0);
    for (int j = 0; j < n; ++j) {
      if (lane == j) mine = acc;
      acc += __shfl_sync(0xffffffffu, v, j);
    }
    if (ok) base[c * kTot] = mine;
  }
}

// Shared-memory layout of the rotation passes (prep_fwd_kernel, prep_brot_kernel): one CTA per
// (batch, 64-token block, kHG heads); the rows' C, B and theta columns of those heads (and, backward,
// their dc~ and db~ rows) are staged with coalesced 16-byte copies (16 threads per 256-byte row
// segment) instead of one scattered row segment per lane.
constexpr int kHG = 4;
constexpr uint32_t kRotRow = kHG * 64;   // bytes of one token's C (or B) columns of kHG heads
constexpr uint32_t kThRow = kHG * 32;    // theta bytes of one token
constexpr uint32_t kSmC = 0, kSmB = kSmC + kBlk * kRotRow, kSmTh = kSmB + kBlk * kRotRow;
constexpr uint32_t kSmFrot = kSmTh + kBlk * kThRow;     // 40960 bytes
constexpr uint32_t kSmDc = kSmFrot, kSmDb = kSmDc + kHG * kBlk * 128;
constexpr uint32_t kSmBrot = kSmDb + kHG * kBlk * 128;  // 106496 bytes
// 16-byte chunk ch of token row t sits at chunk (ch & ~7) | ((ch ^ (t >> 1)) & 7): the 32 lanes of a
// warp, owning tokens 2l and 2l+1, read one logical chunk from eight different bank groups.
__device__ __forceinline__ uint32_t swz_chunk(int t, int ch) {
  return ((uint32_t)ch & ~7u) | (((uint32_t)ch ^ ((uint32_t)t >> 1)) & 7u);
}

// Coalesced copies of the C, B (which = 0, 1 at byte offsets kSmC, kSmB) and theta columns of heads
// [h0, h0 + kHG) for tokens [tb, tb + 64); rows past L and heads past H become zeros.
__device__ __forceinline__ void stage_rot_rows(const void* projv, int64_t proj_sb, int64_t proj_sl, int b, int tb,
                                               int h0, int L, int H, int col_c, int col_b, int col_th, uint32_t sb) {
  const char* proj = static_cast<const char*>(projv);
  for (int k = threadIdx.x; k < kBlk * 16; k += blockDim.x) {
    const int t = k >> 4, ch = k & 15;
    const bool ok = tb + t < L && h0 + (ch >> 2) < H;
    const int64_t row = (int64_t)b * proj_sb + (int64_t)(ok ? tb + t : 0) * proj_sl;
    const uint32_t so = (uint32_t)t * kRotRow + swz_chunk(t, ch) * 16;
    cp_async16(sb + kSmC + so, proj + (row + col_c + h0 * 32) * 2 + (ok ? ch * 16 : 0), ok ? 16 : 0);
    cp_async16(sb + kSmB + so, proj + (row + col_b + h0 * 32) * 2 + (ok ? ch * 16 : 0), ok ? 16 : 0);
  }
  for (int k = threadIdx.x; k < kBlk * 8; k += blockDim.x) {
    const int t = k >> 3, ch = k & 7;
    const bool ok = tb + t < L && h0 + (ch >> 1) < H;
    const int64_t row = (int64_t)b * proj_sb + (int64_t)(ok ? tb + t : 0) * proj_sl;
    cp_async16(sb + kSmTh + (uint32_t)t * kThRow + swz_chunk(t, ch) * 16,
               proj + (row + col_th + h0 * kS2) * 2 + (ok ? ch * 16 : 0), ok ? 16 : 0);
  }
}

// Phi of pairs [kP pg, kP pg + kP) of head hl for tokens tl, tl + 1 (tl = 2 lane): the staged theta,
// the in-block warp scan and the block's prefix (the forward's exact arithmetic).
template <bool kHalf, int kP>
__device__ __forceinline__ void stage_phi(uint32_t sb, const float* pre_row, int hl, int pg, float phi[2][kP]) {
  static_assert(kP == 8 || kP == 4, "eight or four pairs per warp");
  const int lane = threadIdx.x & 31, tl = 2 * lane;
  float th[2][kP];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const uint32_t ca = sb + kSmTh + (uint32_t)(tl + r) * kThRow + swz_chunk(tl + r, 2 * hl + kP * pg / 8) * 16;
    uint32_t w[kP / 2];
    if constexpr (kP == 8) {
      const uint4 v = ld_shared_v4(ca);
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else {
      asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(w[0]), "=r"(w[1]) : "r"(ca + 8 * (pg & 1)) : "memory");
    }
#pragma unroll
    for (int i = 0; i < kP / 2; ++i) { th[r][2 * i] = unpack_lo<kHalf>(w[i]); th[r][2 * i + 1] = unpack_hi<kHalf>(w[i]); }
  }
  const float mypre = lane < kP ? __ldg(pre_row + 2 + kP * pg + lane) : 0.f;
#pragma unroll
  for (int p = 0; p < kP; ++p) {
    float s0, s1;
    scan64(th[0][p], th[1][p], s0, s1);
    const float pre = __shfl_sync(0xffffffffu, mypre, p);
    phi[0][p] = pre + s0;
    phi[1][p] = pre + s1;
  }
}

// Forward, one CTA per (batch, 64-token block, kHG heads); warp (head hl, pair half ph). While the
// copies are in flight, the ph = 0 warp of a head scans g and writes the g, rowf and colf planes, the
// ph = 1 warp scans F; then each warp rotates its eight pairs of C and B in shared memory, and the
// rotated rows leave as coalesced runs (64 tokens x 64 bytes per head are contiguous in c~, b~).
template <bool kHalf>
__global__ void __launch_bounds__(256) prep_fwd_kernel(PrepArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  constexpr int kP = kS2 / 2;
  const int h0 = blockIdx.x * kHG, c = blockIdx.y, b = blockIdx.z;   // head groups of one row block adjacent
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sb = smem_u32(sm);
  const int tb = c * kBlk, tl = 2 * lane;
  stage_rot_rows(a.proj, a.proj_sb, a.proj_sl, b, tb, h0, a.L, a.H, a.col_c, a.col_b, a.col_th, sb);
  const int hl = warp >> 1, ph = warp & 1, h = h0 + hl;
  const int64_t bh = (int64_t)b * a.H + h;
  const float* pre_row = a.tot + (bh * a.nch + c) * kTot;   // exclusive prefixes of this block
  if (h < a.H) {
    float x[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int t = tb + tl + r;
      const bool ok = t < a.L;
      if (ph == 0) {
        const int64_t row = (int64_t)b * a.proj_sb + (int64_t)(ok ? t : 0) * a.proj_sl;
        x[r] = ok ? neg_softplus(ld_lp<kHalf>(a.proj, row + a.col_a + h)) : 0.f;
      } else {
        x[r] = (ok && a.z) ? logsigmoid(__ldg(a.z + (int64_t)b * a.z_sb + (int64_t)t * a.z_sl + h)) : 0.f;
      }
    }
    float s0, s1;
    scan64(x[0], x[1], s0, s1);
    const float pre = __ldg(pre_row + ph);
    const float v[2] = {pre + s0, pre + s1};
    float* pl = a.pos + bh * 4 * a.Lp;
    const int t0 = tb + tl;
    auto store_plane = [&](float* q, float e0, float e1) {
      if (t0 + 1 < a.L) *reinterpret_cast<float2*>(q + t0) = make_float2(e0, e1);
      else if (t0 < a.L) q[t0] = e0;
    };
    if (ph == 0) {
      const float gs = __shfl_sync(0xffffffffu, v[0], 0);
      const float ge = __shfl_sync(0xffffffffu, v[1], 31);   // masked rows add 0: equals the last valid g
      float rf[2], cf[2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        rf[r] = exp2f(fmin_nan((v[r] - gs) * kLog2e, 0.f));
        cf[r] = exp2f(fmin_nan((ge - v[r]) * kLog2e, 0.f));
      }
      store_plane(pl, v[0], v[1]);
      store_plane(pl + 2 * a.Lp, rf[0], rf[1]);
      store_plane(pl + 3 * a.Lp, cf[0], cf[1]);
    } else {
      store_plane(pl + a.Lp, v[0], v[1]);
    }
  }
  cp_async_wait_all();
  __syncthreads();
  if (h < a.H) {
    float phi[2][kP];
    stage_phi<kHalf, kP>(sb, pre_row, hl, ph, phi);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int t = tl + r;
      if (tb + t >= a.L) continue;
      float cs[kP], sn[kP];
#pragma unroll
      for (int p = 0; p < kP; ++p) sincosf(phi[r][p], &sn[p], &cs[p]);
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint32_t zrow = sb + (which == 0 ? kSmC : kSmB) + (uint32_t)t * kRotRow;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint32_t za = zrow + swz_chunk(t, 4 * hl + 2 * ph + q) * 16;
          const uint4 v = ld_shared_v4(za);
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int p = q * 4 + i;
            const float ze = unpack_lo<kHalf>(w[i]), zo = unpack_hi<kHalf>(w[i]);
            o[i] = pack2<kHalf>(ze * cs[p] - zo * sn[p], ze * sn[p] + zo * cs[p]);
          }
          st_shared_v4(za, o[0], o[1], o[2], o[3]);
        }
      }
    }
  }
  __syncthreads();
  for (int k = threadIdx.x; k < kHG * kBlk * 4; k += blockDim.x) {
    const int hk = k >> 8, t = (k >> 2) & (kBlk - 1), q = k & 3;
    if (tb + t >= a.L || h0 + hk >= a.H) continue;
    const uint32_t so = (uint32_t)t * kRotRow + swz_chunk(t, 4 * hk + q) * 16;
    const int64_t e = (((int64_t)b * a.H + h0 + hk) * a.L + tb + t) * 64 + q * 16;   // bytes
    *reinterpret_cast<uint4*>(static_cast<char*>(a.c_rot) + e) = ld_shared_v4(sb + kSmC + so);
    *reinterpret_cast<uint4*>(static_cast<char*>(a.b_rot) + e) = ld_shared_v4(sb + kSmB + so);
  }
}

// ------------------------------------------------------------------------------------ positions
struct PackArgs {
  const float* g;
  int64_t g_sb, g_sh, g_sl;
  const float* f;
  int64_t f_sb, f_sh, f_sl;
  int H, L, Lp;
  float* pos;      // (B*H, 4, Lp) planes
  int32_t* status;
};

// One warp per (b*H + h, 64-row block).
__global__ void __launch_bounds__(256) pack_positions_kernel(PackArgs a, int nch, int64_t nwork) {
  const int64_t wid = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (wid >= nwork) return;
  const int lane = threadIdx.x & 31;
  const int64_t bh = wid / nch;
  const int c = (int)(wid % nch);
  const int b = (int)(bh / a.H), h = (int)(bh % a.H);
  const float* gp = a.g + (int64_t)b * a.g_sb + (int64_t)h * a.g_sh;
  const float* fp = a.f ? a.f + (int64_t)b * a.f_sb + (int64_t)h * a.f_sh : nullptr;
  const int base = c * kBlk;
  const int last = min(base + kBlk - 1, a.L - 1);
  const float gs = __ldg(gp + (int64_t)base * a.g_sl);
  const float ge = __ldg(gp + (int64_t)last * a.g_sl);
  bool bad = false;
  float gg[2] = {0.f, 0.f}, ff[2] = {0.f, 0.f}, rf[2] = {0.f, 0.f}, cf[2] = {0.f, 0.f};
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int t = base + 2 * lane + r;
    if (t >= a.L) continue;
    const float g = __ldg(gp + (int64_t)t * a.g_sl);
    gg[r] = g;
    ff[r] = fp ? __ldg(fp + (int64_t)t * a.f_sl) : 0.f;
    // NaN-propagating clamps, as the reference: a NaN g gives NaN factors.
    rf[r] = exp2f(fmin_nan((g - gs) * kLog2e, 0.f));
    cf[r] = exp2f(fmin_nan((ge - g) * kLog2e, 0.f));
    if (t > 0) {
      const float inc = g - __ldg(gp + (int64_t)(t - 1) * a.g_sl);
      bad |= !(inc <= 1e-3f);
    }
  }
  store_planes(a.pos + bh * 4 * a.Lp, a.Lp, base + 2 * lane, a.L, gg, ff, rf, cf);
  if (__any_sync(0xffffffffu, bad) && lane == 0 && a.status) atomicOr(a.status, SISA_ST_NONMONOTONE);
}

// ------------------------------------------------------------------------------------ backward
struct PrepBwdArgs {
  const void* proj;
  int64_t proj_sb, proj_sl;
  const float* z;
  int64_t z_sb, z_sl;
  int B, L, H, nch;
  int col_b, col_c, col_th, col_a, ntot, npad;
  const float* tot;        // forward block prefixes (fp32, exclusive)
  const float* dc;         // (B,H,L,32) fp32
  const float* db;
  const float* dg;         // (B,H,L)
  const float* dF;         // (B,H,L) or null
  void* dproj;
  int64_t dproj_sb, dproj_sl;
  float* dz;               // (B,L,H)
  double* bt;              // (B*H, nch, kTot) fp64 block totals, then their exclusive suffixes
  float* dphi;             // (B*H, L, kS2) fp32: per-token d Phi of both rotations
  int32_t* status;
};

// First backward pass, one CTA per (batch, 64-token block, kHG heads), laid out like the forward's
// rotation pass plus the heads' dc~ and db~ rows; warp (head, pair half) computes, per lane, tokens 2l
// and 2l+1 with the forward's Phi: dC and dB (final, written back into the staged rows and stored
// coalesced), the per-token d Phi and the fp64 block totals of dg, dF and d Phi.
constexpr int kBrotP = 4;                                    // pairs per warp
constexpr int kBrotThreads = kHG * (kS2 / kBrotP) * 32;      // 512
template <bool kHalf>
__global__ void __launch_bounds__(kBrotThreads, 2) prep_brot_kernel(PrepBwdArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  constexpr int kP = kBrotP, kWph = kS2 / kP;
  const int h0 = blockIdx.x * kHG, c = blockIdx.y, b = blockIdx.z;   // head groups of one row block adjacent
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t sb = smem_u32(sm);
  const int tb = c * kBlk;
  // ---- coalesced copies; rows past L and heads past H become zeros
  stage_rot_rows(a.proj, a.proj_sb, a.proj_sl, b, tb, h0, a.L, a.H, a.col_c, a.col_b, a.col_th, sb);
  for (int k = tid; k < kHG * kBlk * 8; k += blockDim.x) {
    const int hl = k >> 9, t = (k >> 3) & (kBlk - 1), ch = k & 7;
    const bool ok = tb + t < a.L && h0 + hl < a.H;
    const int64_t e = (((int64_t)b * a.H + (ok ? h0 + hl : 0)) * a.L + (ok ? tb + t : 0)) * 32 + ch * 4;
    const uint32_t so = (uint32_t)hl * (kBlk * 128) + (uint32_t)t * 128 + swz_chunk(t, ch) * 16;
    cp_async16(sb + kSmDc + so, a.dc + e, ok ? 16 : 0);
    cp_async16(sb + kSmDb + so, a.db + e, ok ? 16 : 0);
  }
  cp_async_wait_all();
  __syncthreads();

  const int hl = warp / kWph, pg = warp % kWph;   // head in the group; pairs kP pg .. kP pg + kP - 1
  const int h = h0 + hl;
  if (h < a.H) {
    const int64_t bh = (int64_t)b * a.H + h;
    const int tl = 2 * lane;
    double* dst = a.bt + (bh * a.nch + c) * kTot;
    if (pg == 0) {
      // block totals of dg and dF
      double x0, x1, r0, r1, tg, tf;
      x0 = tb + tl < a.L ? (double)__ldg(a.dg + bh * a.L + tb + tl) : 0.0;
      x1 = tb + tl + 1 < a.L ? (double)__ldg(a.dg + bh * a.L + tb + tl + 1) : 0.0;
      rscan64(x0, x1, r0, r1);
      tg = __shfl_sync(0xffffffffu, r0, 0);
      x0 = (a.dF && tb + tl < a.L) ? (double)__ldg(a.dF + bh * a.L + tb + tl) : 0.0;
      x1 = (a.dF && tb + tl + 1 < a.L) ? (double)__ldg(a.dF + bh * a.L + tb + tl + 1) : 0.0;
      rscan64(x0, x1, r0, r1);
      tf = __shfl_sync(0xffffffffu, r0, 0);
      if (lane == 0) { dst[0] = tg; dst[1] = tf; }
    }
    // Phi of this warp's pairs, exactly as the forward computed it
    float phi[2][kP];
    stage_phi<kHalf, kP>(sb, a.tot + (bh * a.nch + c) * kTot, hl, pg, phi);
    // d Phi from both rotations; dC = R(Phi)^T dc~, dB = R(Phi)^T db~ written over the staged C, B
    float dphi[2][kP];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int t = tl + r;
#pragma unroll
      for (int p = 0; p < kP; ++p) dphi[r][p] = 0.f;
      if (tb + t >= a.L) continue;
      float cs[kP], sn[kP];
#pragma unroll
      for (int p = 0; p < kP; ++p) sincosf(phi[r][p], &sn[p], &cs[p]);
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        const uint32_t zrow = sb + (which == 0 ? kSmC : kSmB) + (uint32_t)t * kRotRow;
        const uint32_t grow = sb + (which == 0 ? kSmDc : kSmDb) + (uint32_t)hl * (kBlk * 128) + (uint32_t)t * 128;
#pragma unroll
        for (int q = 0; q < kP / 4; ++q) {   // four pairs: one 16-byte chunk of C (B), two of dc~ (db~)
          const uint32_t za = zrow + swz_chunk(t, 4 * hl + (kP / 4) * pg + q) * 16;
          const uint4 v = ld_shared_v4(za);
          const uint4 g0 = ld_shared_v4(grow + swz_chunk(t, (kP / 2) * pg + 2 * q) * 16);
          const uint4 g1 = ld_shared_v4(grow + swz_chunk(t, (kP / 2) * pg + 2 * q + 1) * 16);
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
          const float gd[8] = {__uint_as_float(g0.x), __uint_as_float(g0.y), __uint_as_float(g0.z), __uint_as_float(g0.w),
                               __uint_as_float(g1.x), __uint_as_float(g1.y), __uint_as_float(g1.z), __uint_as_float(g1.w)};
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int p = q * 4 + i;
            const float ze = unpack_lo<kHalf>(w[i]), zo = unpack_hi<kHalf>(w[i]);
            const float oe = ze * cs[p] - zo * sn[p];
            const float oo = ze * sn[p] + zo * cs[p];
            const float de = gd[2 * i], dd = gd[2 * i + 1];
            dphi[r][p] += dd * oe - de * oo;
            o[i] = pack2<kHalf>(de * cs[p] + dd * sn[p], dd * cs[p] - de * sn[p]);
          }
          st_shared_v4(za, o[0], o[1], o[2], o[3]);
        }
      }
      float4* dp = reinterpret_cast<float4*>(a.dphi + (bh * a.L + tb + t) * kS2 + kP * pg);
#pragma unroll
      for (int q = 0; q < kP / 4; ++q)
        dp[q] = make_float4(dphi[r][4 * q], dphi[r][4 * q + 1], dphi[r][4 * q + 2], dphi[r][4 * q + 3]);
    }
    double tv[kP];
#pragma unroll
    for (int p = 0; p < kP; ++p) {
      double r0, r1;
      rscan64((double)dphi[0][p], (double)dphi[1][p], r0, r1);
      tv[p] = __shfl_sync(0xffffffffu, r0, 0);
    }
    if (lane < kP) {
      double mine = tv[0];
#pragma unroll
      for (int k = 1; k < kP; ++k) if (lane == k) mine = tv[k];
      dst[2 + kP * pg + lane] = mine;
    }
  }
  __syncthreads();
  // ---- coalesced stores of dC and dB
  char* dproj = static_cast<char*>(a.dproj);
  for (int k = tid; k < kBlk * 16; k += blockDim.x) {
    const int t = k >> 4, ch = k & 15;
    if (tb + t >= a.L || h0 + (ch >> 2) >= a.H) continue;
    const int64_t drow = (int64_t)b * a.dproj_sb + (int64_t)(tb + t) * a.dproj_sl;
    const uint32_t so = (uint32_t)t * kRotRow + swz_chunk(t, ch) * 16;
    *reinterpret_cast<uint4*>(dproj + (drow + a.col_c + h0 * 32) * 2 + ch * 16) = ld_shared_v4(sb + kSmC + so);
    *reinterpret_cast<uint4*>(dproj + (drow + a.col_b + h0 * 32) * 2 + ch * 16) = ld_shared_v4(sb + kSmB + so);
  }
}

template <bool kHalf>
__device__ __forceinline__ void st_lp(void* p, int64_t i, float v) {
  if constexpr (kHalf) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// Second backward pass, one CTA per (batch, 64-token block, kHG heads), laid out like the rotation
// passes. The heads' per-token d Phi rows (64 bytes, contiguous per head) are staged with coalesced
// copies, two tokens per 128-byte line, chunk-swizzled by line. Warp (head hl, pair half ph) forms d
// theta of its eight pairs (fp64 suffix sums, rounded once) into a staged theta tile that leaves as
// coalesced row segments; while the copies fly, the ph = 0 warp of a head writes d alpha, the ph = 1
// warp dz.
constexpr uint32_t kSmDphi = 0;                                   // [kHG][32 lines][128 B] fp32
constexpr uint32_t kSmDth = kSmDphi + kHG * kBlk * 64;            // [64 tokens][kThRow] low precision
constexpr uint32_t kSmBwd2 = kSmDth + kBlk * kThRow;              // 24576 bytes

template <bool kHalf>
__global__ void __launch_bounds__(256) prep_bwd_kernel(PrepBwdArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  constexpr int kP = kS2 / 2;
  const int h0 = blockIdx.x * kHG, c = blockIdx.y, b = blockIdx.z;   // head groups of one row block adjacent
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sb = smem_u32(sm);
  const int tb = c * kBlk, tl = 2 * lane;
  for (int k = threadIdx.x; k < kHG * kBlk * 4; k += blockDim.x) {
    const int hk = k >> 8, t = (k >> 2) & (kBlk - 1), q = k & 3;
    const bool ok = tb + t < a.L && h0 + hk < a.H;
    const int64_t e = (((int64_t)b * a.H + (ok ? h0 + hk : 0)) * a.L + (ok ? tb + t : 0)) * kS2 + q * 4;
    cp_async16(sb + kSmDphi + (uint32_t)hk * (kBlk * 64) + (uint32_t)(t >> 1) * 128 + swz_chunk(t, (t & 1) * 4 + q) * 16,
               a.dphi + e, ok ? 16 : 0);
  }
  const int hl = warp >> 1, ph = warp & 1, h = h0 + hl;
  const int64_t bh = (int64_t)b * a.H + h;
  const double* suf_row = a.bt + (bh * a.nch + c) * kTot;   // sums of the totals of the blocks after c
  if (h < a.H && (ph == 0 || a.z)) {
    // ph 0: d alpha = -(sum_{s>=t} dg_s) softplus'(alpha); ph 1: dz = (sum_{s>=t} dF_s) logsigmoid'(z)
    const float* src = ph == 0 ? a.dg : a.dF;
    double r0, r1;
    const double x0 = (src && tb + tl < a.L) ? (double)__ldg(src + bh * a.L + tb + tl) : 0.0;
    const double x1 = (src && tb + tl + 1 < a.L) ? (double)__ldg(src + bh * a.L + tb + tl + 1) : 0.0;
    rscan64(x0, x1, r0, r1);
    const double suf = __ldg(suf_row + ph);
    const double rr[2] = {r0, r1};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int t = tb + tl + r;
      if (t >= a.L) continue;
      const float sum = (float)(suf + rr[r]);
      if (ph == 0) {
        const int64_t row = (int64_t)b * a.proj_sb + (int64_t)t * a.proj_sl;
        const float al = ld_lp<kHalf>(a.proj, row + a.col_a + h);
        st_lp<kHalf>(a.dproj, (int64_t)b * a.dproj_sb + (int64_t)t * a.dproj_sl + a.col_a + h, -sum * softplus_grad(al));
      } else {
        const float zv = __ldg(a.z + (int64_t)b * a.z_sb + (int64_t)t * a.z_sl + h);
        a.dz[((int64_t)b * a.L + t) * a.H + h] = sum * logsigmoid_grad(zv);
      }
    }
  }
  cp_async_wait_all();
  __syncthreads();
  if (h < a.H) {
    // d theta = sum_{s>=t} dPhi_s (dC and dB were written by the first pass)
    float dphi[2][kP];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int t = tl + r;
      const uint32_t line = sb + kSmDphi + (uint32_t)hl * (kBlk * 64) + (uint32_t)(t >> 1) * 128;
      const uint4 v0 = ld_shared_v4(line + swz_chunk(t, (t & 1) * 4 + 2 * ph) * 16);
      const uint4 v1 = ld_shared_v4(line + swz_chunk(t, (t & 1) * 4 + 2 * ph + 1) * 16);
      const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
      for (int p = 0; p < kP; ++p) dphi[r][p] = __uint_as_float(w[p]);
    }
    const double mysuf = lane < kP ? __ldg(suf_row + 2 + kP * ph + lane) : 0.0;
    float dth[2][kP];
#pragma unroll
    for (int p = 0; p < kP; ++p) {
      double r0, r1;
      rscan64((double)dphi[0][p], (double)dphi[1][p], r0, r1);
      const double suf = __shfl_sync(0xffffffffu, mysuf, p);
      dth[0][p] = (float)(suf + r0);
      dth[1][p] = (float)(suf + r1);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int t = tl + r;
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = pack2<kHalf>(dth[r][2 * i], dth[r][2 * i + 1]);
      st_shared_v4(sb + kSmDth + (uint32_t)t * kThRow + swz_chunk(t, 2 * hl + ph) * 16, o[0], o[1], o[2], o[3]);
    }
  }
  __syncthreads();
  char* dproj = static_cast<char*>(a.dproj);
  for (int k = threadIdx.x; k < kBlk * 8; k += blockDim.x) {
    const int t = k >> 3, ch = k & 7;
    if (tb + t >= a.L || h0 + (ch >> 1) >= a.H) continue;
    const int64_t drow = (int64_t)b * a.dproj_sb + (int64_t)(tb + t) * a.dproj_sl;
    *reinterpret_cast<uint4*>(dproj + (drow + a.col_th + h0 * kS2) * 2 + ch * 16) =
        ld_shared_v4(sb + kSmDth + (uint32_t)t * kThRow + swz_chunk(t, ch) * 16);
  }
  // zero the padding columns [ntot, npad) of this block's rows (first head group only)
  const int npadc = a.npad - a.ntot;
  if (npadc > 0 && blockIdx.x == 0) {
    for (int i = threadIdx.x; i < kBlk * npadc; i += blockDim.x) {
      const int t = tb + i / npadc;
      if (t < a.L) st_lp<kHalf>(a.dproj, (int64_t)b * a.dproj_sb + (int64_t)t * a.dproj_sl + a.ntot + i % npadc, 0.f);
    }
  }
}

// ------------------------------------------------------------------------------------ launchers
cudaError_t launch_prep_fwd(const PrepFwdLaunch& p, cudaStream_t st) {
  PrepArgs a;
  a.proj = p.proj; a.proj_sb = p.proj_sb; a.proj_sl = p.proj_sl;
  a.z = p.z; a.z_sb = p.z_sb; a.z_sl = p.z_sl;
  a.B = (int)p.B; a.L = (int)p.L; a.H = (int)p.H; a.nch = (int)((p.L + kBlk - 1) / kBlk);
  a.col_b = (int)p.col_b; a.col_c = (int)p.col_c; a.col_th = (int)p.col_th; a.col_a = (int)p.col_a;
  a.c_rot = p.c_rot; a.b_rot = p.b_rot; a.pos = p.pos; a.Lp = (int)p.Lp;
  a.tot = p.tot; a.status = p.status;
  dim3 grid(a.nch, a.B);
  dim3 grid_rot((a.H + kHG - 1) / kHG, a.nch, a.B);
  const int sums_threads = 32 * (a.H < 32 ? a.H : 32);
  if (p.dtype == 1) {
    prep_sums_kernel<true><<<grid, sums_threads, 0, st>>>(a);
  } else {
    prep_sums_kernel<false><<<grid, sums_threads, 0, st>>>(a);
  }
  const int64_t nchains = (int64_t)a.B * a.H * kTot;
  block_scan_kernel<float, false><<<(unsigned)((nchains + 7) / 8), 256, 0, st>>>(a.tot, nchains, a.nch);
  if (p.dtype == 1) prep_fwd_kernel<true><<<grid_rot, 256, kSmFrot, st>>>(a);
  else prep_fwd_kernel<false><<<grid_rot, 256, kSmFrot, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_pack_positions(const PackLaunch& p, cudaStream_t st) {
  PackArgs a;
  a.g = p.g; a.g_sb = p.g_sb; a.g_sh = p.g_sh; a.g_sl = p.g_sl;
  a.f = p.f; a.f_sb = p.f_sb; a.f_sh = p.f_sh; a.f_sl = p.f_sl;
  a.H = (int)p.H; a.L = (int)p.L; a.Lp = (int)p.Lp; a.pos = p.pos; a.status = p.status;
  const int nch = (int)((p.L + kBlk - 1) / kBlk);
  const int64_t nwork = p.B * p.H * nch;
  pack_positions_kernel<<<(unsigned)((nwork + 7) / 8), 256, 0, st>>>(a, nch, nwork);
  return cudaGetLastError();
}

cudaError_t launch_prep_bwd(const PrepBwdLaunch& p, cudaStream_t st) {
  PrepBwdArgs a;
  a.proj = p.proj; a.proj_sb = p.proj_sb; a.proj_sl = p.proj_sl;
  a.z = p.z; a.z_sb = p.z_sb; a.z_sl = p.z_sl;
  a.B = (int)p.B; a.L = (int)p.L; a.H = (int)p.H; a.nch = (int)((p.L + kBlk - 1) / kBlk);
  a.col_b = (int)p.col_b; a.col_c = (int)p.col_c; a.col_th = (int)p.col_th; a.col_a = (int)p.col_a;
  a.ntot = (int)p.ntot; a.npad = (int)p.npad;
  a.tot = p.tot; a.dc = p.dc; a.db = p.db; a.dg = p.dg; a.dF = p.dF;
  a.dproj = p.dproj; a.dproj_sb = p.dproj_sb; a.dproj_sl = p.dproj_sl; a.dz = p.dz; a.bt = p.bt;
  a.dphi = reinterpret_cast<float*>(p.bt + (int64_t)a.B * a.H * a.nch * kTot);
  a.status = p.status;
  dim3 grid_rot((a.H + kHG - 1) / kHG, a.nch, a.B);
  if (p.dtype == 1) {
    cudaFuncSetAttribute(prep_brot_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmBrot);
    prep_brot_kernel<true><<<grid_rot, kBrotThreads, kSmBrot, st>>>(a);
  } else {
    cudaFuncSetAttribute(prep_brot_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmBrot);
    prep_brot_kernel<false><<<grid_rot, kBrotThreads, kSmBrot, st>>>(a);
  }
  const int64_t nchains = (int64_t)a.B * a.H * kTot;
  block_scan_kernel<double, true><<<(unsigned)((nchains + 7) / 8), 256, 0, st>>>(a.bt, nchains, a.nch);
  if (p.dtype == 1) prep_bwd_kernel<true><<<grid_rot, 256, kSmBwd2, st>>>(a);
  else prep_bwd_kernel<false><<<grid_rot, 256, kSmBwd2, st>>>(a);
  return cudaGetLastError();
}

}  // namespace sisa
