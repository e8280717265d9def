// decode.cu - incremental-decode attention: one new query row per (batch, head) against the cache.
//
// Reference semantics: src/sisa/modeling.py:224-238 (decode step) via src/sisa/functional.py:69-103,
// computed in fp32 over the low-precision cache: for every cached key j (all j <= the new position)
//   s_j = q.k_j / 8 + lam_h exp(min(g_q - g_j, 0)) (c.b~_j) + (F_q - F_j),   y = sum_j softmax(s)_j v_j.
//
// HBM-bound: per cached key and head it reads k (128 B), v (128 B), b~ (64 B), g and F (8 B).
// Split-K over the key axis: grid (splits, B*H) of 256-thread CTAs. Every warp runs its own online
// softmax over groups of four keys: eight lanes per key, each lane holding one 16-byte slice (8 head
// dims) of the key's k, v and b~ rows, so one warp step reads four whole k and v rows (512 bytes each,
// coalesced) and the v loads of a step travel with its k loads. A 3-step shuffle finishes each dot
// product, the running maximum is rescaled lazily (only when a key exceeds it by more than 2^8), and
// each lane accumulates p v over its 8 head dims. There is no block-wide barrier in the key loop; the
// eight warps' (m, l, acc) are merged once at the end, and a second kernel merges the splits.
#include <cuda_runtime.h>
#include <cstdint>
#include <mutex>

#include "sm100.cuh"
#include "gate_math.cuh"
#include "decode.h"
#include "capi_util.h"

namespace sisa {
namespace dec {

constexpr int NT = 256;          // threads per CTA
constexpr int NW = NT / 32;
constexpr float kLog2e = 1.4426950408889634f;

template <bool kHalf>
__device__ __forceinline__ void load_row(const char* p, int n16, float* out) {
  // n16 chunks of 16 bytes (8 low-precision values each)
#pragma unroll
  for (int i = 0; i < n16; ++i) {
    const uint4 v = reinterpret_cast<const uint4*>(p)[i];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      out[i * 8 + 2 * e] = unpack_lo<kHalf>(w[e]);
      out[i * 8 + 2 * e + 1] = unpack_hi<kHalf>(w[e]);
    }
  }
}

// One group of four keys as the warp's lanes load it (eight lanes per key, 16 bytes of k, v and b~ each).
struct KeyGroup {
  uint4 k, v, b;
  float g, f;
};

template <bool kHalf>
__global__ void __launch_bounds__(NT, 4) decode_split_kernel(DecodeParams p) {
  const int split = blockIdx.x, bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // key count: the host's N, or the device position + 1 (a position outside [0, N) attends to nothing)
  int N = p.N;
  if (p.d_pos) {
    const int pos = *p.d_pos;
    N = (pos >= 1 && pos < p.N) ? pos + 1 : 0;
    if (N == 0 && split == 0 && tid == 0 && p.status) atomicOr(p.status, SISA_ST_BAD_POS);
  }
  const int per = (N + p.splits - 1) / p.splits;
  const int j_begin = split * per;
  const int j_end = min(N, j_begin + per);

  __shared__ float s_m[NW], s_l[NW];
  __shared__ float s_acc[NW][64];

  // lanes are grouped eight per key: sub = which of the step's four keys, part = 16-byte slice, i.e. head
  // dims [8 part, 8 part + 8) of q, k and v and, for part < 4, state dims [8 part, 8 part + 8) of c and b~
  const int sub = lane >> 3, part = lane & 7;
  float q8[8], c8[8];
  {
    const uint4 v = reinterpret_cast<const uint4*>(p.q + 2 * ((int64_t)b * p.q_sb + (int64_t)h * p.q_sh))[part];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) { q8[2 * e] = unpack_lo<kHalf>(w[e]); q8[2 * e + 1] = unpack_hi<kHalf>(w[e]); }
  }
  {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (part < 4) v = reinterpret_cast<const uint4*>(p.c + 2 * ((int64_t)b * p.c_sb + (int64_t)h * p.c_sh))[part];
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) { c8[2 * e] = unpack_lo<kHalf>(w[e]); c8[2 * e + 1] = unpack_hi<kHalf>(w[e]); }
  }
  const float gq = p.g_q[bh];
  const float fq = p.f_q ? p.f_q[bh] : 0.f;
  const float lam = p.lam[h];
  const float c1 = 0.125f * kLog2e;
  const float lam2 = lam * kLog2e;
  const char* kbase = p.k + 2 * ((int64_t)b * p.k_sb + (int64_t)h * p.k_sh);
  const char* vbase = p.v + 2 * ((int64_t)b * p.v_sb + (int64_t)h * p.v_sh);
  const char* bbase = p.bm + 2 * ((int64_t)b * p.b_sb + (int64_t)h * p.b_sh);
  const float* gbase = p.g + (int64_t)bh * p.gf_stride;
  const float* fbase = p.f ? p.f + (int64_t)bh * p.gf_stride : nullptr;
  // this lane's slices of key j (j clamped into the split so that every load stays in bounds)
  auto load_group = [&](int j0, KeyGroup& d) {
    const int j = j0 + sub;
    const int jj = j < j_end ? j : j_begin;
    d.k = __ldg(reinterpret_cast<const uint4*>(kbase + 2 * (int64_t)jj * p.k_sl) + part);
    d.v = __ldg(reinterpret_cast<const uint4*>(vbase + 2 * (int64_t)jj * p.v_sl) + part);
    d.b = make_uint4(0, 0, 0, 0);
    if (part < 4) d.b = __ldg(reinterpret_cast<const uint4*>(bbase + 2 * (int64_t)jj * p.b_sl) + part);
    d.g = __ldg(gbase + jj);
    d.f = fbase ? __ldg(fbase + jj) : 0.f;
  };

  float m_ref = -INFINITY;        // this warp's reference maximum (log2 units)
  float acc[8];                   // this lane's 8 head dims of the warp's sum of p v (its key sub-group)
#pragma unroll
  for (int d = 0; d < 8; ++d) acc[d] = 0.f;
  float lsum = 0.f;               // sum of p over this lane's sub-group keys
  // Warp w takes the groups of four keys w, w + 8, w + 16, ... of the split. The next group's loads are
  // issued before the current group is processed, so two groups are in flight per warp whatever the
  // compiler does around the data-dependent rescale branch.
  int j0 = j_begin + 4 * warp;
  KeyGroup cur{};
  if (j0 < j_end) load_group(j0, cur);
#pragma unroll 1
  for (; j0 < j_end; j0 += 4 * NW) {
    KeyGroup nxt = cur;
    if (j0 + 4 * NW < j_end) load_group(j0 + 4 * NW, nxt);
    const bool ok = j0 + sub < j_end;
    const uint32_t kw[4] = {cur.k.x, cur.k.y, cur.k.z, cur.k.w}, bw[4] = {cur.b.x, cur.b.y, cur.b.z, cur.b.w};
    float qk = 0.f, cb = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      qk = fmaf(q8[2 * e], unpack_lo<kHalf>(kw[e]), qk);
      qk = fmaf(q8[2 * e + 1], unpack_hi<kHalf>(kw[e]), qk);
      cb = fmaf(c8[2 * e], unpack_lo<kHalf>(bw[e]), cb);
      cb = fmaf(c8[2 * e + 1], unpack_hi<kHalf>(bw[e]), cb);
    }
    const float dec = exp2f(fmin_nan((gq - cur.g) * kLog2e, 0.f));
    float x = fmaf(qk, c1, lam2 * (dec * cb));
    x += __shfl_xor_sync(0xffffffffu, x, 1);
    x += __shfl_xor_sync(0xffffffffu, x, 2);
    x += __shfl_xor_sync(0xffffffffu, x, 4);
    x = ok ? fmaf(fq - cur.f, kLog2e, x) : -INFINITY;
    // step maximum over the four keys; rescale only when it exceeds the reference by more than 2^8
    float mx = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 8));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    if (mx > m_ref + 8.f) {
      const float corr = (m_ref == -INFINITY) ? 0.f : exp2f(m_ref - mx);
#pragma unroll
      for (int d = 0; d < 8; ++d) acc[d] *= corr;
      lsum *= corr;
      m_ref = mx;
    }
    const float pj = ok ? exp2f(x - m_ref) : 0.f;
    const uint32_t vw[4] = {cur.v.x, cur.v.y, cur.v.z, cur.v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      acc[2 * e] = fmaf(pj, unpack_lo<kHalf>(vw[e]), acc[2 * e]);
      acc[2 * e + 1] = fmaf(pj, unpack_hi<kHalf>(vw[e]), acc[2 * e + 1]);
    }
    lsum += pj;
    cur = nxt;
  }
  // ---- the warp's sums over its four key sub-groups (all lanes of a sub-group hold the same lsum)
#pragma unroll
  for (int d = 0; d < 8; ++d) {
    acc[d] += __shfl_xor_sync(0xffffffffu, acc[d], 8);
    acc[d] += __shfl_xor_sync(0xffffffffu, acc[d], 16);
  }
  lsum += __shfl_xor_sync(0xffffffffu, lsum, 8);
  lsum += __shfl_xor_sync(0xffffffffu, lsum, 16);
  if (sub == 0) {
#pragma unroll
    for (int d = 0; d < 8; ++d) s_acc[warp][8 * part + d] = acc[d];
  }
  if (lane == 0) { s_m[warp] = m_ref; s_l[warp] = lsum; }
  __syncthreads();
  // ---- merge the warps (rescaled to their common maximum) and write this split's (m, l, acc[64])
  float m = s_m[0];
#pragma unroll
  for (int w = 1; w < NW; ++w) m = fmaxf(m, s_m[w]);
  float* out = p.ws + ((int64_t)split * p.B * p.H + bh) * 66;
  if (tid < 64) {
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float sc = (s_m[w] == -INFINITY) ? 0.f : exp2f(s_m[w] - m);
      a = fmaf(s_acc[w][tid], sc, a);
    }
    out[2 + tid] = a;
  }
  if (tid == 0) {
    float l = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float sc = (s_m[w] == -INFINITY) ? 0.f : exp2f(s_m[w] - m);
      l = fmaf(s_l[w], sc, l);
    }
    out[0] = m;
    out[1] = l;
  }
}

// One warp per (batch, head): merge the splits, normalise, write y in the low-precision dtype. The
// splits' (m, l) records are read by the lanes in parallel (lane s takes splits s, s + 32, ...) and
// reduced across the warp; then each lane owns two head dims and walks the splits with independent
// 8-byte loads, the split weights arriving by shuffle from the lane that computed them.
template <bool kHalf>
__global__ void __launch_bounds__(256) decode_combine_kernel(DecodeParams p) {
  const int bh = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (bh >= p.B * p.H) return;
  const int lane = threadIdx.x & 31;
  const int b = bh / p.H, h = bh % p.H;
  const int64_t stride = (int64_t)p.B * p.H * 66;
  const float* rec = p.ws + (int64_t)bh * 66;
  float m = -INFINITY;
  for (int s = lane; s < p.splits; s += 32) m = fmaxf(m, rec[s * stride]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float l = 0.f;
  for (int s = lane; s < p.splits; s += 32) {
    const float ms = rec[s * stride];
    l = fmaf(rec[s * stride + 1], (ms == -INFINITY) ? 0.f : exp2f(ms - m), l);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
  float a0 = 0.f, a1 = 0.f;
  for (int s0 = 0; s0 < p.splits; s0 += 32) {
    float wl = 0.f;
    if (s0 + lane < p.splits) {
      const float ms = rec[(s0 + lane) * stride];
      wl = (ms == -INFINITY) ? 0.f : exp2f(ms - m);
    }
    const int cnt = min(32, p.splits - s0);
#pragma unroll 4
    for (int i = 0; i < cnt; ++i) {
      const float w = __shfl_sync(0xffffffffu, wl, i);
      const float2 v = *reinterpret_cast<const float2*>(rec + (s0 + i) * stride + 2 + 2 * lane);
      a0 = fmaf(v.x, w, a0);
      a1 = fmaf(v.y, w, a1);
    }
  }
  const float ls = (l == 0.f) ? 1.f : l;
  uint32_t* y = reinterpret_cast<uint32_t*>(p.y + 2 * ((int64_t)b * p.y_sb + (int64_t)h * p.y_sh));
  y[lane] = pack2<kHalf>(a0 / ls, a1 / ls);
  if (lane == 0 && p.status && !isfinite(m + __log2f(ls))) atomicOr(p.status, SISA_ST_NONFINITE);
}

}  // namespace dec

// Splits of the key axis: about eight waves of the split kernel at four 256-thread CTAs per SM (so the
// last, partial wave is a small share), at least 256 keys per split, at most 64 splits.
int decode_splits(int64_t B, int64_t H, int64_t N) {
  const int64_t target = 148 * 4 * 8;
  const int64_t bh = B * H;
  int64_t s = (target + bh - 1) / bh;
  const int64_t maxs = (N + dec::NT - 1) / dec::NT;
  if (s > maxs) s = maxs;
  if (s < 1) s = 1;
  if (s > 64) s = 64;
  return (int)s;
}

// One decode step's layer input (the single-token case of modeling.py:171-199 / fused_prep.py:247-352),
// one warp per (batch, head): g_t = g_{t-1} - softplus(alpha_t), F_t = F_{t-1} + logsigmoid(z_t),
// Phi_t = Phi_{t-1} + theta_t (16 pairs), c~ = R(Phi_t) c and b~ = R(Phi_t) b in fp32 with torch's
// separate products (no contraction), rounded once; k, v, b~, g, F go into the caches at pos, c~, g_t,
// F_t to the query-side outputs, and Phi advances in place.
template <bool kHalf>
__global__ void __launch_bounds__(256) decode_prep_kernel(DecodePrepParams p) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (w >= p.B * p.H) return;
  int64_t pos = p.pos;
  if (p.d_pos) {                  // position read on the device: out of range writes nothing
    pos = *p.d_pos;
    if (pos < 1 || pos >= p.max_pos) {
      if (w == 0 && lane == 0 && p.status) atomicOr(p.status, SISA_ST_BAD_POS);
      return;
    }
  }
  const int b = w / p.H, h = w - b * p.H;
  const uint16_t* row = p.proj + (int64_t)b * p.proj_sb;
  auto to_f = [](uint16_t x) {
    if constexpr (kHalf) return __half2float(__ushort_as_half(x));
    else return __uint_as_float((uint32_t)x << 16);
  };
  auto to_lp = [](float x) -> uint16_t {
    if constexpr (kHalf) return __half_as_ushort(__float2half_rn(x));
    else return __bfloat16_as_ushort(__float2bfloat16_rn(x));
  };
  // k and v rows: 64 elements, two per lane
  {
    const uint32_t kk = reinterpret_cast<const uint32_t*>(row + p.col_k + h * 64)[lane];
    const uint32_t vv = reinterpret_cast<const uint32_t*>(row + p.col_v + h * 64)[lane];
    reinterpret_cast<uint32_t*>(p.k + (int64_t)b * p.k_sb + (int64_t)h * p.k_sh + pos * p.k_sl)[lane] = kk;
    reinterpret_cast<uint32_t*>(p.v + (int64_t)b * p.v_sb + (int64_t)h * p.v_sh + pos * p.v_sl)[lane] = vv;
  }
  const int64_t bh = (int64_t)b * p.H + h;
  if (lane < 16) {
    float* ph = p.phi + bh * 16 + lane;
    const float phin = to_f(row[p.col_th + h * 16 + lane]) + *ph;
    *ph = phin;
    const float cs = cosf(phin), sn = sinf(phin);
    const int e = 2 * lane;
    const float ce = to_f(row[p.col_c + h * 32 + e]), co = to_f(row[p.col_c + h * 32 + e + 1]);
    const float be = to_f(row[p.col_b + h * 32 + e]), bo = to_f(row[p.col_b + h * 32 + e + 1]);
    const uint32_t cr = (uint32_t)to_lp(__fsub_rn(__fmul_rn(ce, cs), __fmul_rn(co, sn))) |
                        ((uint32_t)to_lp(__fadd_rn(__fmul_rn(ce, sn), __fmul_rn(co, cs))) << 16);
    const uint32_t br = (uint32_t)to_lp(__fsub_rn(__fmul_rn(be, cs), __fmul_rn(bo, sn))) |
                        ((uint32_t)to_lp(__fadd_rn(__fmul_rn(be, sn), __fmul_rn(bo, cs))) << 16);
    reinterpret_cast<uint32_t*>(p.c_out + bh * 32)[lane] = cr;
    reinterpret_cast<uint32_t*>(p.bm + (int64_t)b * p.b_sb + (int64_t)h * p.b_sh + pos * p.b_sl)[lane] = br;
  } else if (lane == 16) {
    const float gq = neg_softplus(to_f(row[p.col_a + h])) + p.g[bh * p.gf_stride + pos - 1];
    p.g[bh * p.gf_stride + pos] = gq;
    p.g_out[bh] = gq;
  } else if (lane == 17 && p.f) {
    const float fq = logsigmoid(p.z[(int64_t)b * p.z_sb + h]) + p.f[bh * p.gf_stride + pos - 1];
    p.f[bh * p.gf_stride + pos] = fq;
    p.f_out[bh] = fq;
  }
}

cudaError_t launch_decode_prep(const DecodePrepParams& p, int dtype, cudaStream_t st) {
  const unsigned grid = (unsigned)((p.B * p.H + 7) / 8);
  if (dtype == 1) decode_prep_kernel<true><<<grid, 256, 0, st>>>(p);
  else decode_prep_kernel<false><<<grid, 256, 0, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_decode(const DecodeParams& p, int dtype, cudaStream_t st) {
  dim3 grid(p.splits, p.B * p.H);
  const unsigned nb = (unsigned)((p.B * p.H + 7) / 8);
  if (dtype == 1) {
    dec::decode_split_kernel<true><<<grid, dec::NT, 0, st>>>(p);
    dec::decode_combine_kernel<true><<<nb, 256, 0, st>>>(p);
  } else {
    dec::decode_split_kernel<false><<<grid, dec::NT, 0, st>>>(p);
    dec::decode_combine_kernel<false><<<nb, 256, 0, st>>>(p);
  }
  return cudaGetLastError();
}

}  // namespace sisa

// =============================================================================================
// Allocation-free decode entry point.
//
// Some callers of this library cannot allocate device memory when they decode: a host program that
// binds only this C ABI (from another language, through an FFI) and has no device allocator of its
// own, and a serving loop that runs under a fixed, pre-reserved memory budget, where an allocation
// at decode time could fail or fragment the pool. sisa_decode_attn needs a caller-provided workspace
// for its split-K partials; this variant keeps those partials in a fixed array that the library
// owns instead, so the caller passes only inputs and outputs.
//
// The array below lives in every GPU that loads this library, from module load until process exit.
// Its device address is resolved once per device, on the first call made on that device, with that
// device current; that first call should therefore come before any stream capture. A
// cudaDeviceReset of a device unloads the module, so the address recorded for that device is stale
// afterwards: do not call this entry point on a device that has been reset in the same process.
// All calls on a device share the one array and it keeps the last call's contents: every call
// rewrites each partial record it reads before reading it, so nothing needs clearing, but two calls
// that overlap on the GPU (different streams, no ordering between them) race on the array and
// corrupt each other's results.
// =============================================================================================
namespace sisa {
namespace dec {
constexpr int64_t kStaticRecords = 16384;        // (split, batch, head) partial records of 66 floats: 4.3 MB
static __device__ __align__(256) float g_static_partials[kStaticRecords * 66];
}  // namespace dec
}  // namespace sisa

extern "C" int sisa_decode_attn_noalloc(const sisa_view4* q, const sisa_view4* c, const float* g_q, const float* f_q,
                                        const sisa_view4* k_cache, const sisa_view4* v_cache,
                                        const sisa_view4* b_cache, const float* g_cache, const float* f_cache,
                                        int64_t gf_stride, const float* lam, int64_t B, int64_t H, int64_t N,
                                        int dtype, const sisa_view4* y, int32_t* status, void* stream) {
  using sisa::capi_fail;
  static std::mutex mu;
  static void* scratch_by_device[256] = {};
  int rc;
  // the same argument checks as sisa_decode_attn
  if ((rc = sisa::capi_check_dims(B, H, N)) || (rc = sisa::capi_check_dtype(dtype))) return rc;
  if ((rc = sisa::capi_check_view(q, 2, "q")) || (rc = sisa::capi_check_view(c, 2, "c")) ||
      (rc = sisa::capi_check_view(k_cache, 2, "k_cache")) || (rc = sisa::capi_check_view(v_cache, 2, "v_cache")) ||
      (rc = sisa::capi_check_view(b_cache, 2, "b_cache")) || (rc = sisa::capi_check_view(y, 2, "y")))
    return rc;
  if (B * H > sisa::dec::kStaticRecords)
    return capi_fail(SISA_ERR_VALUE,
                     "sisa_decode_attn_noalloc: B*H exceeds the 16384 (batch, head) rows of the library's fixed "
                     "scratch; use sisa_decode_attn with a caller workspace");
  if (!g_q || !g_cache || !lam) return capi_fail(SISA_ERR_VALUE, "sisa_decode_attn_noalloc: null pointer");
  if ((f_q == nullptr) != (f_cache == nullptr))
    return capi_fail(SISA_ERR_VALUE, "sisa_decode_attn_noalloc: f_q and f_cache must both be given or both be null");
  if (gf_stride < N) return capi_fail(SISA_ERR_VALUE, "sisa_decode_attn_noalloc: g/F cache row stride < N");
  // The scratch address is resolved on the device that owns the data, with that device current; the
  // caller's current device is restored when this call returns.
  sisa::DeviceScope scope;
  if ((rc = scope.bind(q->data))) return rc;
  const int dev = scope.device();
  if (dev < 0 || dev >= 256) return capi_fail(SISA_ERR_VALUE, "sisa_decode_attn_noalloc: bad device");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(mu);
    scratch = scratch_by_device[dev];
    if (!scratch) {
      const cudaError_t e = cudaGetSymbolAddress(&scratch, sisa::dec::g_static_partials);
      if (e != cudaSuccess || !scratch)
        return capi_fail(SISA_ERR_CUDA, "sisa_decode_attn_noalloc: cudaGetSymbolAddress of the fixed scratch failed");
      scratch_by_device[dev] = scratch;
    }
  }
  sisa::DecodeParams p{};
  p.q = static_cast<const char*>(q->data); p.q_sb = q->stride_b; p.q_sh = q->stride_h;
  p.c = static_cast<const char*>(c->data); p.c_sb = c->stride_b; p.c_sh = c->stride_h;
  p.g_q = g_q; p.f_q = f_q;
  p.k = static_cast<const char*>(k_cache->data); p.k_sb = k_cache->stride_b; p.k_sh = k_cache->stride_h;
  p.k_sl = k_cache->stride_l;
  p.v = static_cast<const char*>(v_cache->data); p.v_sb = v_cache->stride_b; p.v_sh = v_cache->stride_h;
  p.v_sl = v_cache->stride_l;
  p.bm = static_cast<const char*>(b_cache->data); p.b_sb = b_cache->stride_b; p.b_sh = b_cache->stride_h;
  p.b_sl = b_cache->stride_l;
  p.g = g_cache; p.f = f_cache; p.gf_stride = gf_stride; p.lam = lam;
  p.y = static_cast<char*>(y->data); p.y_sb = y->stride_b; p.y_sh = y->stride_h;
  p.ws = static_cast<float*>(scratch);
  p.B = (int)B; p.H = (int)H; p.N = (int)N;
  int64_t splits = sisa::decode_splits(B, H, N);
  const int64_t cap = sisa::dec::kStaticRecords / (B * H);     // >= 1 by the check above
  p.splits = (int)(splits < cap ? splits : cap);
  p.status = status;
  const cudaError_t e = sisa::launch_decode(p, dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : capi_fail(SISA_ERR_CUDA, "sisa_decode_attn_noalloc launch failed");
}
