// capi.cu - the extern "C" boundary of libsisa_b200.so: argument validation, TMA tensor-map
// encoding and kernel launches. No device allocation, no host synchronisation, no exceptions.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "sisa_b200.h"
#include "attn.h"
#include "prep.h"
#include "decode.h"
#include "lce.h"
#include "gemm.h"
#include "optim.h"
#include "copy.h"
#include "embed.h"
#include "norm.h"
#include "capi_util.h"

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(SISA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// (X, L, H, B) view of a (B, H, L, X) tensor with element strides; box (X, rows, 1, 1).
int map_view4(CUtensorMap* m, const sisa_view4* v, int64_t B, int64_t H, int64_t L, int64_t X, int elem_bytes,
              CUtensorMapDataType dt, int rows, CUtensorMapSwizzle sw, const char* name) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(SISA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[4] = {(cuuint64_t)X, (cuuint64_t)L, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(v->stride_l * elem_bytes), (cuuint64_t)(v->stride_h * elem_bytes),
                           (cuuint64_t)(v->stride_b * elem_bytes)};
  // size-1 axes may carry any stride; give them a legal one
  if (H == 1) strides[1] = strides[0] * (cuuint64_t)L;
  if (B == 1) strides[2] = (H == 1 ? strides[1] : strides[1] * (cuuint64_t)H);
  cuuint32_t box[4] = {(cuuint32_t)X, (cuuint32_t)rows, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = enc(m, dt, 4, v->data, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SISA_ERR_ALIGN, "%s: cuTensorMapEncodeTiled failed (%d)", name, (int)r);
  return SISA_OK;
}

// (4, L, B*H) fp32 records, box (4, 64, 1).
// Planar per-position records (B*H, 4, Lp) fp32: dims (L, 4, B*H), box (64, 4, 1), so one copy
// brings the four planes of a 64-row block as [4][64] floats.
int map_records(CUtensorMap* m, const void* ptr, int64_t BH, int64_t L, int64_t Lp, const char* name) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(SISA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {(cuuint64_t)L, 4, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)(Lp * 4), (cuuint64_t)(Lp * 16)};
  cuuint32_t box[3] = {64, 4, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(ptr), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SISA_ERR_ALIGN, "%s: cuTensorMapEncodeTiled failed (%d)", name, (int)r);
  return SISA_OK;
}

// Dense (B*H, L, X) rows as a (X, L, B*H) map, box (box_x, rows, 1).
int map_rows3(CUtensorMap* m, const void* ptr, int64_t BH, int64_t L, int64_t X, int elem_bytes,
              CUtensorMapDataType dt, int box_x, int rows, CUtensorMapSwizzle sw, const char* name) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(SISA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {(cuuint64_t)X, (cuuint64_t)L, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)(X * elem_bytes), (cuuint64_t)(X * elem_bytes * L)};
  cuuint32_t box[3] = {(cuuint32_t)box_x, (cuuint32_t)rows, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, dt, 3, const_cast<void*>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SISA_ERR_ALIGN, "%s: cuTensorMapEncodeTiled failed (%d)", name, (int)r);
  return SISA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

using CtxGetFn = CUresult (*)(CUcontext*);
using CtxSetFn = CUresult (*)(CUcontext);

// cuCtxGetCurrent / cuCtxSetCurrent through the runtime's driver entry-point query (no link against
// libcuda), resolved once; null if the driver does not offer them.
struct CtxFns {
  CtxGetFn get = nullptr;
  CtxSetFn set = nullptr;
};
const CtxFns& ctx_fns() {
  static CtxFns f;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      f.get = reinterpret_cast<CtxGetFn>(p);
    if (cudaGetDriverEntryPoint("cuCtxSetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      f.set = reinterpret_cast<CtxSetFn>(p);
  });
  return f;
}

int check_view(const sisa_view4* v, int elem_bytes, const char* name) {
  if (!v || !v->data) return fail(SISA_ERR_VALUE, "%s: null view", name);
  if (!aligned16(v->data)) return fail(SISA_ERR_ALIGN, "%s: data pointer is not 16-byte aligned", name);
  const int64_t unit = 16 / elem_bytes;
  if (v->stride_l % unit || v->stride_h % unit || v->stride_b % unit)
    return fail(SISA_ERR_ALIGN, "%s: strides (%lld, %lld, %lld) must be multiples of %lld elements", name,
                (long long)v->stride_b, (long long)v->stride_h, (long long)v->stride_l, (long long)unit);
  if (v->stride_l <= 0 || v->stride_h < 0 || v->stride_b < 0)
    return fail(SISA_ERR_VALUE, "%s: negative or zero strides are not supported", name);
  return SISA_OK;
}

int check_dims(int64_t B, int64_t H, int64_t L) {
  if (B < 1 || H < 1 || L < 1) return fail(SISA_ERR_VALUE, "B, H and L must be >= 1 (got %lld, %lld, %lld)",
                                           (long long)B, (long long)H, (long long)L);
  // The attention grids are (L/128, B*H) and the preparation grids (H/4, L/64, B): their second and
  // third grid dimensions are limited to 65535 blocks.
  if (L > 65535ll * 64 || B > 65535 || H > 65535 || B * H > 65535)
    return fail(SISA_ERR_VALUE, "problem too large (B*H=%lld, L=%lld)", (long long)(B * H), (long long)L);
  return SISA_OK;
}

int check_dtype(int dtype) {
  if (dtype != SISA_BF16 && dtype != SISA_F16) return fail(SISA_ERR_TYPE, "dtype must be SISA_BF16 or SISA_F16");
  return SISA_OK;
}

void layout(int64_t H, int64_t* o) {
  o[0] = 0;                    // Q
  o[1] = H * 64;               // K
  o[2] = 2 * H * 64;           // V
  o[3] = 3 * H * 64;           // B
  o[4] = o[3] + H * 32;        // C
  o[5] = o[4] + H * 32;        // TH
  o[6] = o[5] + H * 16;        // A
  o[7] = o[6] + H;             // NTOT = 273 H
  o[8] = (o[7] + 15) / 16 * 16;  // NPAD
}

int64_t nch64(int64_t L) { return (L + 63) / 64; }

}  // namespace

namespace sisa {
// Records an error for sisa_last_error() from entry points defined outside this file.
int capi_fail(int code, const char* msg) { return fail(code, "%s", msg); }
int capi_check_dims(int64_t B, int64_t H, int64_t L) { return check_dims(B, H, L); }
int capi_check_view(const sisa_view4* v, int elem_bytes, const char* name) { return check_view(v, elem_bytes, name); }
int capi_check_dtype(int dtype) { return check_dtype(dtype); }

int DeviceScope::bind(const void* ptr) {
  cudaPointerAttributes a;
  cudaError_t e = cudaPointerGetAttributes(&a, ptr);
  if (e != cudaSuccess) return cuda_fail(e, "cudaPointerGetAttributes");
  if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged)
    return fail(SISA_ERR_VALUE, "tensor data is not device memory");
  const CtxFns& f = ctx_fns();
  CUcontext cur = nullptr;
  if (f.get && f.set && f.get(&cur) == CUDA_SUCCESS) {
    prev_ = cur;
    bound_ = true;
  }
  e = cudaSetDevice(a.device);   // makes the device's primary context current on this thread
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  device_ = a.device;
  return SISA_OK;
}

DeviceScope::~DeviceScope() {
  if (!bound_) return;
  const CtxFns& f = ctx_fns();
  CUcontext now = nullptr;
  if (f.get(&now) == CUDA_SUCCESS && now != static_cast<CUcontext>(prev_)) f.set(static_cast<CUcontext>(prev_));
}
}  // namespace sisa

extern "C" {

const char* sisa_version(void) { return "sisa_b200 0.1.0 (sm_100a)"; }
const char* sisa_last_error(void) { return g_err.c_str(); }

int sisa_device_check(int device) {
  cudaDeviceProp prop;
  cudaError_t e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  if (prop.major != 10 || prop.minor != 0)
    return fail(SISA_ERR_UNSUPPORTED, "%s is sm_%d%d; this library is built for sm_100a only", prop.name,
                prop.major, prop.minor);
  return SISA_OK;
}

int sisa_fused_layout(int64_t n_head, int64_t* out9) {
  if (n_head < 1) return fail(SISA_ERR_VALUE, "n_head must be >= 1");
  if (!out9) return fail(SISA_ERR_VALUE, "out9 is null");
  layout(n_head, out9);
  return SISA_OK;
}

int64_t sisa_prep_fwd_workspace(int64_t B, int64_t H, int64_t L) { return B * H * nch64(L) * 18 * 4; }
// fp64 block totals (B*H, nch, 18), then the per-token d Phi (B*H, L, 16) fp32
int64_t sisa_prep_bwd_workspace(int64_t B, int64_t H, int64_t L) { return B * H * (nch64(L) * 18 * 8 + L * 16 * 4); }
int64_t sisa_pos_len(int64_t L) { return (L + 3) & ~int64_t(3); }
// rstat planes (B*H, 4, Lp) fp32, then rg, rf, rl (B*H, L) fp32 each
int64_t sisa_attn_bwd_workspace(int64_t B, int64_t H, int64_t L) { return B * H * (sisa_pos_len(L) * 16 + L * 12); }

int sisa_prep_fwd(const void* proj, int64_t B, int64_t L, int64_t H, int64_t proj_sb, int64_t proj_sl, int dtype,
                  const float* z, int64_t z_sb, int64_t z_sl, void* c_rot, void* b_rot, float* pos, void* workspace,
                  int32_t* status, void* stream) {
  int rc;
  if ((rc = check_dims(B, H, L)) || (rc = check_dtype(dtype))) return rc;
  if (!proj || !c_rot || !b_rot || !pos || !workspace) return fail(SISA_ERR_VALUE, "sisa_prep_fwd: null pointer");
  int64_t off[9];
  layout(H, off);
  if (proj_sl < off[8]) return fail(SISA_ERR_VALUE, "proj row stride %lld < NPAD %lld", (long long)proj_sl,
                                    (long long)off[8]);
  if (!aligned16(proj) || proj_sl % 8 || proj_sb % 8)
    return fail(SISA_ERR_ALIGN, "proj must be 16-byte aligned with strides that are multiples of 8 elements");
  if (!aligned16(c_rot) || !aligned16(b_rot) || !aligned16(pos))
    return fail(SISA_ERR_ALIGN, "c_rot, b_rot and pos must be 16-byte aligned");
  sisa::PrepFwdLaunch p{};
  p.proj = proj; p.proj_sb = proj_sb; p.proj_sl = proj_sl; p.dtype = dtype;
  p.z = z; p.z_sb = z_sb; p.z_sl = z_sl;
  p.B = B; p.L = L; p.H = H;
  p.col_b = off[3]; p.col_c = off[4]; p.col_th = off[5]; p.col_a = off[6];
  p.c_rot = c_rot; p.b_rot = b_rot; p.pos = pos; p.Lp = sisa_pos_len(L);
  p.tot = static_cast<float*>(workspace); p.status = status;
  cudaError_t e = sisa::launch_prep_fwd(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_prep_fwd launch");
}

int sisa_pack_positions(const float* g, int64_t g_sb, int64_t g_sh, int64_t g_sl, const float* fgate, int64_t f_sb,
                        int64_t f_sh, int64_t f_sl, int64_t B, int64_t H, int64_t L, float* pos, int32_t* status,
                        void* stream) {
  int rc;
  if ((rc = check_dims(B, H, L))) return rc;
  if (!g || !pos) return fail(SISA_ERR_VALUE, "sisa_pack_positions: null pointer");
  if (!aligned16(pos)) return fail(SISA_ERR_ALIGN, "pos must be 16-byte aligned");
  sisa::PackLaunch p{};
  p.g = g; p.g_sb = g_sb; p.g_sh = g_sh; p.g_sl = g_sl;
  p.f = fgate; p.f_sb = f_sb; p.f_sh = f_sh; p.f_sl = f_sl;
  p.B = B; p.H = H; p.L = L; p.Lp = sisa_pos_len(L); p.pos = pos; p.status = status;
  cudaError_t e = sisa::launch_pack_positions(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_pack_positions launch");
}

int sisa_attn_fwd(const sisa_view4* q, const sisa_view4* k, const sisa_view4* v, const sisa_view4* c,
                  const sisa_view4* b, const float* pos, const float* lam, int64_t B, int64_t H, int64_t L, int dtype,
                  const sisa_view4* o, float* lse, float* o32, int32_t* status, void* stream) {
  int rc;
  if ((rc = check_dims(B, H, L)) || (rc = check_dtype(dtype))) return rc;
  if ((rc = check_view(q, 2, "q")) || (rc = check_view(k, 2, "k")) || (rc = check_view(v, 2, "v")) ||
      (rc = check_view(c, 2, "c")) || (rc = check_view(b, 2, "b")) || (rc = check_view(o, 2, "o")))
    return rc;
  if (!pos || !lam || !lse) return fail(SISA_ERR_VALUE, "sisa_attn_fwd: null pos, lam or lse");
  if (!aligned16(pos) || (o32 && !aligned16(o32))) return fail(SISA_ERR_ALIGN, "pos/o32 must be 16-byte aligned");
  sisa::DeviceScope scope;
  if ((rc = scope.bind(q->data))) return rc;
  const CUtensorMapDataType dt = dtype == SISA_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  sisa::FwdParams p;
  memset(&p, 0, sizeof(p));
  if ((rc = map_view4(&p.tm_q, q, B, H, L, 64, 2, dt, 128, CU_TENSOR_MAP_SWIZZLE_128B, "q")) ||
      (rc = map_view4(&p.tm_k, k, B, H, L, 64, 2, dt, 64, CU_TENSOR_MAP_SWIZZLE_128B, "k")) ||
      (rc = map_view4(&p.tm_v, v, B, H, L, 64, 2, dt, 64, CU_TENSOR_MAP_SWIZZLE_128B, "v")) ||
      (rc = map_view4(&p.tm_c, c, B, H, L, 32, 2, dt, 128, CU_TENSOR_MAP_SWIZZLE_64B, "c")) ||
      (rc = map_view4(&p.tm_b, b, B, H, L, 32, 2, dt, 64, CU_TENSOR_MAP_SWIZZLE_64B, "b")) ||
      (rc = map_records(&p.tm_pos, pos, B * H, L, sisa_pos_len(L), "pos")) ||
      (rc = map_view4(&p.tm_ost, o, B, H, L, 64, 2, dt, 128, CU_TENSOR_MAP_SWIZZLE_128B, "o")) ||
      (o32 && (rc = map_rows3(&p.tm_o32, o32, B * H, L, 64, 4, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 32, 128,
                              CU_TENSOR_MAP_SWIZZLE_128B, "o32"))))
    return rc;
  p.pos = pos;
  p.lam = lam;
  p.o = static_cast<char*>(o->data); p.o_sb = o->stride_b; p.o_sh = o->stride_h; p.o_sl = o->stride_l;
  p.lse = lse; p.o32 = o32;
  p.B = (int)B; p.H = (int)H; p.L = (int)L; p.Lp = (int)sisa_pos_len(L); p.ntq = (int)((L + 127) / 128);
  p.status = status;
  cudaError_t e = sisa::launch_attn_fwd(p, dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_attn_fwd launch");
}

int sisa_attn_bwd(const sisa_view4* q, const sisa_view4* k, const sisa_view4* v, const sisa_view4* c,
                  const sisa_view4* b, const float* pos, const float* lam, const sisa_view4* o, const sisa_view4* dout,
                  const float* lse, const float* o32, int64_t B, int64_t H, int64_t L, int dtype, const sisa_view4* dq,
                  const sisa_view4* dk, const sisa_view4* dv, const sisa_view4* dc, const sisa_view4* db, float* dg,
                  float* dF, float* dlam, void* workspace, int32_t* status, void* stream) {
  int rc;
  if ((rc = check_dims(B, H, L)) || (rc = check_dtype(dtype))) return rc;
  if ((rc = check_view(q, 2, "q")) || (rc = check_view(k, 2, "k")) || (rc = check_view(v, 2, "v")) ||
      (rc = check_view(c, 2, "c")) || (rc = check_view(b, 2, "b")) || (rc = check_view(o, 2, "o")) ||
      (rc = check_view(dout, 2, "dout")) || (rc = check_view(dq, 2, "dq")) || (rc = check_view(dk, 2, "dk")) ||
      (rc = check_view(dv, 2, "dv")) || (rc = check_view(dc, 4, "dc")) || (rc = check_view(db, 4, "db")))
    return rc;
  if (!pos || !lam || !lse || !dg || !dlam || !workspace)
    return fail(SISA_ERR_VALUE, "sisa_attn_bwd: null pos, lam, lse, dg, dlam or workspace");
  if (!aligned16(pos) || !aligned16(workspace) || (o32 && !aligned16(o32)))
    return fail(SISA_ERR_ALIGN, "pos, o32 and workspace must be 16-byte aligned");
  sisa::DeviceScope scope;
  if ((rc = scope.bind(q->data))) return rc;
  const CUtensorMapDataType dt = dtype == SISA_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  sisa::BwdParams p;
  memset(&p, 0, sizeof(p));
  const CUtensorMapSwizzle s128 = CU_TENSOR_MAP_SWIZZLE_128B, s64 = CU_TENSOR_MAP_SWIZZLE_64B;
  char* ws = static_cast<char*>(workspace);
  const int64_t n = B * H * L;
  p.rstat = reinterpret_cast<float*>(ws);
  p.rg = reinterpret_cast<float*>(ws + B * H * sisa_pos_len(L) * 16);
  p.rf = p.rg + n;
  p.rl = p.rf + n;
  if ((rc = map_view4(&p.tm_q128, q, B, H, L, 64, 2, dt, 128, s128, "q")) ||
      (rc = map_view4(&p.tm_do128, dout, B, H, L, 64, 2, dt, 128, s128, "dout")) ||
      (rc = map_view4(&p.tm_c128, c, B, H, L, 32, 2, dt, 128, s64, "c")) ||
      (rc = map_view4(&p.tm_k64, k, B, H, L, 64, 2, dt, 64, s128, "k")) ||
      (rc = map_view4(&p.tm_v64, v, B, H, L, 64, 2, dt, 64, s128, "v")) ||
      (rc = map_view4(&p.tm_b64, b, B, H, L, 32, 2, dt, 64, s64, "b")) ||
      (rc = map_view4(&p.tm_k128, k, B, H, L, 64, 2, dt, 128, s128, "k")) ||
      (rc = map_view4(&p.tm_v128, v, B, H, L, 64, 2, dt, 128, s128, "v")) ||
      (rc = map_view4(&p.tm_b128, b, B, H, L, 32, 2, dt, 128, s64, "b")) ||
      (rc = map_view4(&p.tm_q64, q, B, H, L, 64, 2, dt, 64, s128, "q")) ||
      (rc = map_view4(&p.tm_do64, dout, B, H, L, 64, 2, dt, 64, s128, "dout")) ||
      (rc = map_view4(&p.tm_c64, c, B, H, L, 32, 2, dt, 64, s64, "c")) ||
      (rc = map_records(&p.tm_pos, pos, B * H, L, sisa_pos_len(L), "pos")) ||
      (rc = map_records(&p.tm_rstat, p.rstat, B * H, L, sisa_pos_len(L), "rstat")) ||
      (rc = o32 ? map_rows3(&p.tm_o, o32, B * H, L, 64, 4, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 32, 128, s128, "o32")
                : map_view4(&p.tm_o, o, B, H, L, 64, 2, dt, 128, s128, "o")) ||
      (rc = map_view4(&p.tm_dq, dq, B, H, L, 64, 2, dt, 128, s128, "dq")) ||
      (rc = map_view4(&p.tm_dc, dc, B, H, L, 32, 4, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 128, s128, "dc")) ||
      (rc = map_view4(&p.tm_dk, dk, B, H, L, 64, 2, dt, 128, s128, "dk")) ||
      (rc = map_view4(&p.tm_dv, dv, B, H, L, 64, 2, dt, 128, s128, "dv")) ||
      (rc = map_view4(&p.tm_db, db, B, H, L, 32, 4, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 128, s128, "db")))
    return rc;
  p.pos = pos;
  p.lam = lam;
  p.q = static_cast<const char*>(q->data); p.q_sb = q->stride_b; p.q_sh = q->stride_h; p.q_sl = q->stride_l;
  p.k = static_cast<const char*>(k->data); p.k_sb = k->stride_b; p.k_sh = k->stride_h; p.k_sl = k->stride_l;
  p.bm = static_cast<const char*>(b->data); p.b_sb = b->stride_b; p.b_sh = b->stride_h; p.b_sl = b->stride_l;
  p.o = static_cast<const char*>(o->data); p.o_sb = o->stride_b; p.o_sh = o->stride_h; p.o_sl = o->stride_l;
  p.dout = static_cast<const char*>(dout->data); p.do_sb = dout->stride_b; p.do_sh = dout->stride_h;
  p.do_sl = dout->stride_l;
  p.lse = lse; p.o32 = o32;
  p.dq = static_cast<char*>(dq->data); p.dq_sb = dq->stride_b; p.dq_sh = dq->stride_h; p.dq_sl = dq->stride_l;
  p.dk = static_cast<char*>(dk->data); p.dk_sb = dk->stride_b; p.dk_sh = dk->stride_h; p.dk_sl = dk->stride_l;
  p.dv = static_cast<char*>(dv->data); p.dv_sb = dv->stride_b; p.dv_sh = dv->stride_h; p.dv_sl = dv->stride_l;
  p.dc = static_cast<float*>(dc->data); p.dc_sb = dc->stride_b; p.dc_sh = dc->stride_h; p.dc_sl = dc->stride_l;
  p.db = static_cast<float*>(db->data); p.db_sb = db->stride_b; p.db_sh = db->stride_h; p.db_sl = db->stride_l;
  p.dg = dg; p.dF = dF; p.dlam = dlam;
  p.B = (int)B; p.H = (int)H; p.L = (int)L; p.Lp = (int)sisa_pos_len(L);
  p.ntq128 = (int)((L + 127) / 128); p.ntq64 = (int)((L + 63) / 64);
  p.has_f = dF != nullptr;
  p.status = status;
  cudaError_t e = sisa::launch_attn_bwd(p, dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_attn_bwd launch");
}

int sisa_prep_bwd(const void* proj, int64_t B, int64_t L, int64_t H, int64_t proj_sb, int64_t proj_sl, int dtype,
                  const float* z, int64_t z_sb, int64_t z_sl, const void* tot, const float* dc, const float* db,
                  const float* dg, const float* dF, void* dproj, int64_t dproj_sb, int64_t dproj_sl, float* dz,
                  void* workspace, int32_t* status, void* stream) {
  int rc;
  if ((rc = check_dims(B, H, L)) || (rc = check_dtype(dtype))) return rc;
  if (!proj || !tot || !dc || !db || !dg || !dproj || !workspace)
    return fail(SISA_ERR_VALUE, "sisa_prep_bwd: null pointer");
  if (z && !dz) return fail(SISA_ERR_VALUE, "sisa_prep_bwd: dz is null but z is given");
  int64_t off[9];
  layout(H, off);
  if (proj_sl < off[8] || dproj_sl < off[8]) return fail(SISA_ERR_VALUE, "proj/dproj row stride < NPAD");
  if (!aligned16(proj) || !aligned16(dproj) || proj_sl % 8 || proj_sb % 8 || dproj_sl % 8 || dproj_sb % 8)
    return fail(SISA_ERR_ALIGN, "proj/dproj must be 16-byte aligned with strides that are multiples of 8");
  if (!aligned16(dc) || !aligned16(db) || !aligned16(workspace))
    return fail(SISA_ERR_ALIGN, "dc, db and workspace must be 16-byte aligned");
  sisa::PrepBwdLaunch p{};
  p.proj = proj; p.proj_sb = proj_sb; p.proj_sl = proj_sl; p.dtype = dtype;
  p.z = z; p.z_sb = z_sb; p.z_sl = z_sl;
  p.B = B; p.L = L; p.H = H;
  p.col_b = off[3]; p.col_c = off[4]; p.col_th = off[5]; p.col_a = off[6]; p.ntot = off[7]; p.npad = off[8];
  p.tot = static_cast<const float*>(tot); p.dc = dc; p.db = db; p.dg = dg; p.dF = dF;
  p.dproj = dproj; p.dproj_sb = dproj_sb; p.dproj_sl = dproj_sl; p.dz = dz;
  p.bt = static_cast<double*>(workspace); p.status = status;
  cudaError_t e = sisa::launch_prep_bwd(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_prep_bwd launch");
}

int64_t sisa_decode_workspace(int64_t B, int64_t H, int64_t N) {
  return (int64_t)sisa::decode_splits(B, H, N) * B * H * 66 * 4;
}

// Shared by sisa_decode_attn (d_pos null, N keys) and sisa_decode_attn_dpos (N = *d_pos + 1 <= max_n keys).
static int decode_attn_impl(const sisa_view4* q, const sisa_view4* c, const float* g_q, const float* f_q,
                            const sisa_view4* k_cache, const sisa_view4* v_cache, const sisa_view4* b_cache,
                            const float* g_cache, const float* f_cache, int64_t gf_stride, const float* lam,
                            int64_t B, int64_t H, int64_t N, const int32_t* d_pos, int dtype, const sisa_view4* y,
                            void* workspace, int32_t* status, void* stream) {
  int rc;
  if ((rc = check_dims(B, H, N)) || (rc = check_dtype(dtype))) return rc;
  if ((rc = check_view(q, 2, "q")) || (rc = check_view(c, 2, "c")) || (rc = check_view(k_cache, 2, "k_cache")) ||
      (rc = check_view(v_cache, 2, "v_cache")) || (rc = check_view(b_cache, 2, "b_cache")) ||
      (rc = check_view(y, 2, "y")))
    return rc;
  if (!g_q || !g_cache || !lam || !workspace) return fail(SISA_ERR_VALUE, "sisa_decode_attn: null pointer");
  if ((f_q == nullptr) != (f_cache == nullptr))
    return fail(SISA_ERR_VALUE, "sisa_decode_attn: f_q and f_cache must both be given or both be null");
  if (gf_stride < N) return fail(SISA_ERR_VALUE, "g/F cache row stride %lld < N %lld", (long long)gf_stride,
                                 (long long)N);
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
  p.ws = static_cast<float*>(workspace);
  p.B = (int)B; p.H = (int)H; p.N = (int)N; p.splits = sisa::decode_splits(B, H, N);
  p.status = status;
  p.d_pos = d_pos;
  cudaError_t e = sisa::launch_decode(p, dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_decode_attn launch");
}

int sisa_decode_attn(const sisa_view4* q, const sisa_view4* c, const float* g_q, const float* f_q,
                     const sisa_view4* k_cache, const sisa_view4* v_cache, const sisa_view4* b_cache,
                     const float* g_cache, const float* f_cache, int64_t gf_stride, const float* lam, int64_t B,
                     int64_t H, int64_t N, int dtype, const sisa_view4* y, void* workspace, int32_t* status,
                     void* stream) {
  return decode_attn_impl(q, c, g_q, f_q, k_cache, v_cache, b_cache, g_cache, f_cache, gf_stride, lam, B, H, N,
                          nullptr, dtype, y, workspace, status, stream);
}

int sisa_decode_attn_dpos(const sisa_view4* q, const sisa_view4* c, const float* g_q, const float* f_q,
                          const sisa_view4* k_cache, const sisa_view4* v_cache, const sisa_view4* b_cache,
                          const float* g_cache, const float* f_cache, int64_t gf_stride, const float* lam,
                          int64_t B, int64_t H, const int32_t* d_pos, int64_t max_n, int dtype, const sisa_view4* y,
                          void* workspace, int32_t* status, void* stream) {
  if (!d_pos || (reinterpret_cast<uintptr_t>(d_pos) & 3u))
    return fail(SISA_ERR_VALUE, "sisa_decode_attn_dpos: d_pos must be a 4-byte aligned device pointer");
  return decode_attn_impl(q, c, g_q, f_q, k_cache, v_cache, b_cache, g_cache, f_cache, gf_stride, lam, B, H, max_n,
                          d_pos, dtype, y, workspace, status, stream);
}

// Shared by sisa_decode_prep (host position pos) and sisa_decode_prep_dpos (position *d_pos, checked on the
// device against [1, pos), where pos then carries max_pos).
static int decode_prep_impl(const void* proj, int64_t proj_sb, const float* z, int64_t z_sb, int64_t B, int64_t H,
                            int dtype, const sisa_view4* k_cache, const sisa_view4* v_cache,
                            const sisa_view4* b_cache, float* g_cache, float* f_cache, int64_t gf_stride,
                            int64_t pos, const int32_t* d_pos, float* phi, void* c_out, float* g_out, float* f_out,
                            int32_t* status, void* stream) {
  int rc;
  if ((rc = check_dims(B, H, pos + 1)) || (rc = check_dtype(dtype))) return rc;
  if ((rc = check_view(k_cache, 2, "k_cache")) || (rc = check_view(v_cache, 2, "v_cache")) ||
      (rc = check_view(b_cache, 2, "b_cache")))
    return rc;
  if (!proj || !g_cache || !phi || !c_out || !g_out) return fail(SISA_ERR_VALUE, "sisa_decode_prep: null pointer");
  if ((z == nullptr) != (f_cache == nullptr) || (z == nullptr) != (f_out == nullptr))
    return fail(SISA_ERR_VALUE, "sisa_decode_prep: z, f_cache and f_out must all be given or all be null");
  if (d_pos && (pos < 2 || pos > gf_stride))
    return fail(SISA_ERR_VALUE, "sisa_decode_prep_dpos: max_pos %lld outside [2, %lld]", (long long)pos,
                (long long)gf_stride);
  if (!d_pos && (pos < 1 || pos >= gf_stride))
    return fail(SISA_ERR_VALUE, "sisa_decode_prep: position %lld outside [1, %lld)", (long long)pos, (long long)gf_stride);
  int64_t off[9];
  if ((rc = sisa_fused_layout(H, off))) return rc;
  const auto al4 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 3u) == 0; };
  if (!al4(proj) || proj_sb < off[7] || proj_sb % 2 || !al4(c_out) || !al4(k_cache->data) || !al4(v_cache->data) ||
      !al4(b_cache->data) || (k_cache->stride_b | k_cache->stride_h | k_cache->stride_l) % 2 ||
      (v_cache->stride_b | v_cache->stride_h | v_cache->stride_l) % 2 ||
      (b_cache->stride_b | b_cache->stride_h | b_cache->stride_l) % 2)
    return fail(SISA_ERR_ALIGN, "sisa_decode_prep: operands need 4-byte alignment and even element strides");
  sisa::DecodePrepParams p{};
  p.proj = static_cast<const uint16_t*>(proj); p.proj_sb = proj_sb;
  p.z = z; p.z_sb = z_sb;
  p.col_k = (int)off[1]; p.col_v = (int)off[2]; p.col_b = (int)off[3]; p.col_c = (int)off[4];
  p.col_th = (int)off[5]; p.col_a = (int)off[6];
  p.k = static_cast<uint16_t*>(k_cache->data); p.k_sb = k_cache->stride_b; p.k_sh = k_cache->stride_h;
  p.k_sl = k_cache->stride_l;
  p.v = static_cast<uint16_t*>(v_cache->data); p.v_sb = v_cache->stride_b; p.v_sh = v_cache->stride_h;
  p.v_sl = v_cache->stride_l;
  p.bm = static_cast<uint16_t*>(b_cache->data); p.b_sb = b_cache->stride_b; p.b_sh = b_cache->stride_h;
  p.b_sl = b_cache->stride_l;
  p.g = g_cache; p.f = f_cache; p.gf_stride = gf_stride; p.phi = phi;
  p.c_out = static_cast<uint16_t*>(c_out); p.g_out = g_out; p.f_out = f_out;
  p.B = (int)B; p.H = (int)H;
  p.pos = d_pos ? 0 : pos;
  p.d_pos = d_pos; p.max_pos = d_pos ? pos : 0; p.status = status;
  cudaError_t e = sisa::launch_decode_prep(p, dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_decode_prep launch");
}

int sisa_decode_prep(const void* proj, int64_t proj_sb, const float* z, int64_t z_sb, int64_t B, int64_t H,
                     int dtype, const sisa_view4* k_cache, const sisa_view4* v_cache, const sisa_view4* b_cache,
                     float* g_cache, float* f_cache, int64_t gf_stride, int64_t pos, float* phi, void* c_out,
                     float* g_out, float* f_out, int32_t* status, void* stream) {
  return decode_prep_impl(proj, proj_sb, z, z_sb, B, H, dtype, k_cache, v_cache, b_cache, g_cache, f_cache, gf_stride,
                          pos, nullptr, phi, c_out, g_out, f_out, status, stream);
}

int sisa_decode_prep_dpos(const void* proj, int64_t proj_sb, const float* z, int64_t z_sb, int64_t B, int64_t H,
                          int dtype, const sisa_view4* k_cache, const sisa_view4* v_cache, const sisa_view4* b_cache,
                          float* g_cache, float* f_cache, int64_t gf_stride, const int32_t* d_pos, int64_t max_pos,
                          float* phi, void* c_out, float* g_out, float* f_out, int32_t* status, void* stream) {
  if (!d_pos || (reinterpret_cast<uintptr_t>(d_pos) & 3u))
    return fail(SISA_ERR_VALUE, "sisa_decode_prep_dpos: d_pos must be a 4-byte aligned device pointer");
  return decode_prep_impl(proj, proj_sb, z, z_sb, B, H, dtype, k_cache, v_cache, b_cache, g_cache, f_cache, gf_stride,
                          max_pos, d_pos, phi, c_out, g_out, f_out, status, stream);
}

// ------------------------------------------------------------------------------------ tensor maps of the GEMM
// Tensor map of one operand: rows x K, K-major (box 64 K x 128 rows) or MN-major (box 64 rows x 64 K).
static int map_operand(CUtensorMap* m, const void* ptr, int64_t ld, int mn, int64_t rows, int64_t K,
                       CUtensorMapDataType dt, const char* name) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(SISA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)(mn ? rows : K), (cuuint64_t)(mn ? K : rows)};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, mn ? 64u : 128u}, es[2] = {1, 1};
  if (enc(m, dt, 2, const_cast<void*>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS)
    return fail(SISA_ERR_ALIGN, "%s: cuTensorMapEncodeTiled failed", name);
  return SISA_OK;
}

// Tensor map of C: rows x N row-major in out_dtype; box 32 rows x 128 bytes, 128-byte swizzle.
static int map_output(CUtensorMap* m, void* ptr, int64_t ld, int64_t rows, int64_t N, int out_dtype) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(SISA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const int64_t osz = out_dtype == SISA_F32 ? 4 : 2;
  cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * osz)};
  cuuint32_t box[2] = {(cuuint32_t)(128 / osz), 32}, es[2] = {1, 1};
  const CUtensorMapDataType cdt = out_dtype == SISA_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                  : out_dtype == SISA_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                          : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if (enc(m, cdt, 2, ptr, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return fail(SISA_ERR_ALIGN, "c: cuTensorMapEncodeTiled failed");
  return SISA_OK;
}

int64_t sisa_lce_workspace(int64_t R, int64_t Vp) {
  const int64_t nseg = (Vp + 255) / 256;            // one (max, sum) record per row and 256-column tile
  return R * nseg * 8 + ((R * 4 + 255) / 256) * 256;
}

int sisa_lce_logits(const void* x, int64_t R, int64_t D, int64_t x_ld, const void* w, int64_t V, int64_t Vp,
                    int64_t w_ld, int dtype, const int64_t* labels, void* logits, int64_t logits_ld,
                    void* workspace, int32_t* status, void* stream) {
  int rc;
  if ((rc = check_dtype(dtype))) return rc;
  if (!x || !w || !labels || !logits || !workspace) return fail(SISA_ERR_VALUE, "sisa_lce_logits: null pointer");
  if (R < 1 || D < 64 || D % 64 || V < 1 || Vp % 128 || Vp < V || R > ((int64_t)1 << 30) || Vp > ((int64_t)1 << 30))
    return fail(SISA_ERR_VALUE, "sisa_lce_logits: need R >= 1, D a multiple of 64, Vp >= V a multiple of 128 "
                "(R=%lld D=%lld V=%lld Vp=%lld)", (long long)R, (long long)D, (long long)V, (long long)Vp);
  if (!aligned16(x) || !aligned16(w) || !aligned16(logits) || !aligned16(workspace) || x_ld % 8 || w_ld % 8 ||
      logits_ld % 8 || x_ld < D || w_ld < D || logits_ld < Vp)
    return fail(SISA_ERR_ALIGN, "sisa_lce_logits: rows must be 16-byte aligned (ld multiple of 8 and >= width)");
  sisa::DeviceScope scope;
  if ((rc = scope.bind(x))) return rc;
  const CUtensorMapDataType dt = dtype == SISA_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  sisa::GemmParams p;
  memset(&p, 0, sizeof(p));
  if ((rc = map_operand(&p.tm_a, x, x_ld, 0, R, D, dt, "x"))) return rc;
  if ((rc = map_operand(&p.tm_b, w, w_ld, 0, Vp, D, dt, "w"))) return rc;
  if ((rc = map_output(&p.tm_c, logits, logits_ld, R, Vp, dtype == SISA_F16 ? SISA_F16 : SISA_BF16))) return rc;
  const int64_t nseg = (Vp + 255) / 256;
  p.ldc = logits_ld;
  p.M = (int)R; p.N = (int)Vp; p.K = (int)D;
  p.num_m = (int)((R + 255) / 256);
  p.status = status;
  p.labels = labels;
  p.part = static_cast<float2*>(workspace);
  p.tgt = reinterpret_cast<float*>(static_cast<char*>(workspace) + R * nseg * 8);
  p.V = (int)V; p.n_part = (int)nseg;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, scope.device());
  cudaError_t e = sisa::launch_lce_logits_gemm(p, dtype, sms, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_lce_logits launch");
}

int sisa_lce_grad(void* logits, int64_t logits_ld, int64_t R, int64_t V, int64_t Vp, int dtype,
                  const int64_t* labels, int64_t ignore_index, const float* inv_n, float grad_scale,
                  int compute_grad, const void* workspace, float* loss_rows, int32_t* status, void* stream) {
  int rc;
  if ((rc = check_dtype(dtype))) return rc;
  if (!logits || !labels || !inv_n || !workspace || !loss_rows) return fail(SISA_ERR_VALUE, "sisa_lce_grad: null pointer");
  if (R < 1 || Vp % 128 || Vp < V || logits_ld < Vp || logits_ld % 8 || !aligned16(logits))
    return fail(SISA_ERR_VALUE, "sisa_lce_grad: bad shape or alignment");
  const int64_t nseg = (Vp + 255) / 256;
  sisa::LceGradParams p{};
  p.logits = static_cast<char*>(logits); p.ld = logits_ld;
  p.part = static_cast<const float2*>(workspace);
  p.tgt = reinterpret_cast<const float*>(static_cast<const char*>(workspace) + R * nseg * 8);
  p.labels = labels; p.inv_n = inv_n; p.gscale = grad_scale; p.loss_rows = loss_rows;
  p.ignore_index = ignore_index; p.R = (int)R; p.V = (int)V; p.Vp = (int)Vp; p.n_nblk = (int)nseg;
  p.compute_grad = compute_grad; p.status = status;
  cudaError_t e = sisa::launch_lce_grad(p, dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_lce_grad launch");
}

int sisa_lce_seed_scale(float* x, int64_t n, const float* seed, void* out, int out_dtype, int32_t* status,
                        void* stream) {
  (void)status;
  if (!x || !seed) return fail(SISA_ERR_VALUE, "sisa_lce_seed_scale: null pointer");
  if (n < 0) return fail(SISA_ERR_VALUE, "sisa_lce_seed_scale: n < 0");
  if (out_dtype != SISA_BF16 && out_dtype != SISA_F16 && out_dtype != SISA_F32)
    return fail(SISA_ERR_TYPE, "sisa_lce_seed_scale: out_dtype must be SISA_BF16, SISA_F16 or SISA_F32");
  if (!out && out_dtype != SISA_F32) return fail(SISA_ERR_VALUE, "sisa_lce_seed_scale: in place needs SISA_F32");
  if (!aligned16(x) || (out && !aligned16(out)))
    return fail(SISA_ERR_ALIGN, "sisa_lce_seed_scale: pointers must be 16-byte aligned");
  int rc;
  sisa::DeviceScope scope;
  if ((rc = scope.bind(x))) return rc;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, scope.device());
  const int code = out_dtype == SISA_F32 ? 2 : out_dtype == SISA_F16 ? 1 : 0;
  cudaError_t e = sisa::launch_seed_scale(x, n, seed, out, code, sms, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_lce_seed_scale launch");
}

// ------------------------------------------------------------------------------------ flat AdamW
int sisa_adamw_flat(float* param, const float* grad, float* m, float* v, int64_t n, const sisa_adam_seg* segs,
                    int nseg, float* step, double* partials, int npart, float beta1, float beta2, float eps,
                    float max_norm, int32_t* status, void* stream) {
  if (!param || !grad || !m || !v || !segs || !step || !partials)
    return fail(SISA_ERR_VALUE, "sisa_adamw_flat: null pointer");
  if (n < 0 || n % 4 || nseg < 1 || nseg > 8192 || npart < 1 || npart > 4096)
    return fail(SISA_ERR_VALUE, "sisa_adamw_flat: need n a multiple of 4, 1 <= nseg <= 8192, 1 <= npart <= 4096 "
                "(n=%lld nseg=%d npart=%d)", (long long)n, nseg, npart);
  if (!aligned16(param) || !aligned16(grad) || !aligned16(m) || !aligned16(v) || !aligned16(segs) ||
      !aligned16(partials))
    return fail(SISA_ERR_ALIGN, "sisa_adamw_flat: buffers must be 16-byte aligned");
  if (!(beta1 >= 0.f && beta1 < 1.f && beta2 >= 0.f && beta2 < 1.f && eps > 0.f))
    return fail(SISA_ERR_VALUE, "sisa_adamw_flat: need 0 <= beta1, beta2 < 1 and eps > 0");
  static_assert(sizeof(sisa_adam_seg) == sizeof(sisa::AdamSeg), "segment layout");
  int rc;
  sisa::DeviceScope scope;
  if ((rc = scope.bind(param))) return rc;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, scope.device());
  sisa::AdamParams p{};
  p.param = param; p.grad = grad; p.m = m; p.v = v; p.n4 = n / 4;
  p.segs = reinterpret_cast<const sisa::AdamSeg*>(segs); p.nseg = nseg;
  p.step = step; p.partials = partials; p.npart = npart; p.nblocks = 8 * sms;
  p.beta1 = beta1; p.beta2 = beta2; p.eps = eps; p.max_norm = max_norm; p.status = status;
  cudaError_t e = sisa::launch_adamw(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_adamw_flat launch");
}

int sisa_adamw_tensors(const sisa_adam_tensor* tensors, int ntensors, float* m, float* v, int64_t n_state,
                       float* step, double* partials, int npart, float beta1, float beta2, float eps,
                       float max_norm, int32_t* status, void* stream) {
  if (!tensors || !m || !v || !step || !partials) return fail(SISA_ERR_VALUE, "sisa_adamw_tensors: null pointer");
  if (ntensors < 0 || ntensors > sisa::kMaxAdamTensors || npart < 1 || npart > 4096 || n_state < 0 || n_state % 4)
    return fail(SISA_ERR_VALUE, "sisa_adamw_tensors: need 0 <= ntensors <= %d, 1 <= npart <= 4096, n_state a "
                "multiple of 4 (ntensors=%d npart=%d n_state=%lld)", sisa::kMaxAdamTensors, ntensors, npart,
                (long long)n_state);
  if (!aligned16(m) || !aligned16(v) || !aligned16(partials))
    return fail(SISA_ERR_ALIGN, "sisa_adamw_tensors: m, v and partials must be 16-byte aligned");
  if (!(beta1 >= 0.f && beta1 < 1.f && beta2 >= 0.f && beta2 < 1.f && eps > 0.f))
    return fail(SISA_ERR_VALUE, "sisa_adamw_tensors: need 0 <= beta1, beta2 < 1 and eps > 0");
  static_assert(sizeof(sisa_adam_tensor) == sizeof(sisa::AdamTensor), "tensor entry layout");
  int64_t end = 0;
  for (int k = 0; k < ntensors; ++k) {
    const sisa_adam_tensor& t = tensors[k];
    if (!t.param || !t.grad || t.n < 1 || t.offset % 4 || t.offset < end || t.offset + t.n > n_state)
      return fail(SISA_ERR_VALUE, "sisa_adamw_tensors: tensor %d: need param, grad, n >= 1 and an offset that is "
                  "a multiple of 4, past the previous tensor, with offset + n <= n_state", k);
    if ((reinterpret_cast<uintptr_t>(t.param) | reinterpret_cast<uintptr_t>(t.grad)) & 3u)
      return fail(SISA_ERR_ALIGN, "sisa_adamw_tensors: tensor %d: param and grad must be 4-byte aligned", k);
    end = t.offset + t.n;
  }
  if (ntensors == 0) return SISA_OK;
  int rc;
  sisa::DeviceScope scope;
  if ((rc = scope.bind(m))) return rc;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, scope.device());
  static sisa::AdamListParams p;          // 15 KB: kept off the stack; filled and launched under the lock
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  memset(&p, 0, sizeof(p));
  memcpy(p.t, tensors, sizeof(sisa::AdamTensor) * (size_t)ntensors);
  p.nt = ntensors;
  p.m = m; p.v = v; p.n4 = (end + 3) / 4;
  p.step = step; p.partials = partials; p.npart = npart; p.nblocks = 8 * sms;
  p.beta1 = beta1; p.beta2 = beta2; p.eps = eps; p.max_norm = max_norm; p.status = status;
  cudaError_t e = sisa::launch_adamw_list(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_adamw_tensors launch");
}

// ------------------------------------------------------------------------------------ weight copies
int sisa_row_copy_check(const sisa_row_copy* j) {
  if (!j) return fail(SISA_ERR_VALUE, "sisa_row_copy_check: null job");
  const int64_t lim = (int64_t)1 << 40;
  if (!j->dst || j->rows < 0 || j->cols < 8 || j->cols % 8 || j->block_rows < 1 || j->dst_block_stride < 0 ||
      j->rows > lim || j->cols > lim || j->dst_ld > lim || j->src_ld > lim)
    return fail(SISA_ERR_VALUE, "sisa_row_copy: need dst, rows >= 0, cols a positive multiple of 8, block_rows >= 1 "
                "(rows=%lld cols=%lld block_rows=%lld)", (long long)j->rows, (long long)j->cols,
                (long long)j->block_rows);
  if (!aligned16(j->dst) || j->dst_ld % 8 || j->dst_ld < j->cols ||
      (j->src && (!aligned16(j->src) || j->src_ld % 4 || j->src_ld < j->cols)))
    return fail(SISA_ERR_ALIGN, "sisa_row_copy: rows must be 16-byte aligned (dst_ld a multiple of 8, src_ld of 4, "
                "both >= cols)");
  return SISA_OK;
}

int sisa_copy_heads(const void* src, int64_t src_sb, int64_t src_sh, int64_t src_sl, void* dst, int64_t dst_sb,
                    int64_t dst_sh, int64_t dst_sl, int64_t B, int64_t H, int64_t L, int64_t width, void* stream) {
  if (!src || !dst) return fail(SISA_ERR_VALUE, "sisa_copy_heads: null pointer");
  if (B < 0 || H < 1 || L < 0 || width < 8 || width % 8 || H * (width / 8) > 256 || B > ((int64_t)1 << 31) ||
      L > ((int64_t)1 << 31))
    return fail(SISA_ERR_VALUE, "sisa_copy_heads: need B, L >= 0, H >= 1, width a positive multiple of 8 and "
                "H * width / 8 <= 256 (B=%lld H=%lld L=%lld width=%lld)", (long long)B, (long long)H, (long long)L,
                (long long)width);
  if (!aligned16(src) || !aligned16(dst) || src_sb % 8 || src_sh % 8 || src_sl % 8 || dst_sb % 8 || dst_sh % 8 ||
      dst_sl % 8)
    return fail(SISA_ERR_ALIGN, "sisa_copy_heads: pointers must be 16-byte aligned and strides multiples of 8");
  if (B == 0 || L == 0) return SISA_OK;
  int rc;
  sisa::DeviceScope scope;
  if ((rc = scope.bind(dst))) return rc;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, scope.device());
  const sisa::HeadsCopy p{src, src_sb, src_sh, src_sl, dst, dst_sb, dst_sh, dst_sl, B, H, L, width};
  cudaError_t e = sisa::launch_copy_heads(p, sms, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_copy_heads launch");
}

int sisa_embedding_bwd(const int64_t* ids, int64_t n, const float* grad, int64_t grad_ld, float* dw, int64_t V,
                       int64_t D, void* stream) {
  if ((n > 0 && (!ids || !grad)) || !dw) return fail(SISA_ERR_VALUE, "sisa_embedding_bwd: null pointer");
  if (n < 0 || n > SISA_EMBED_MAX_IDS || V < 1 || V > ((int64_t)1 << 31) - 1 || D < 4 || D % 4 || grad_ld < D)
    return fail(SISA_ERR_VALUE, "sisa_embedding_bwd: need 0 <= n <= %d, 1 <= V < 2^31, D a positive multiple of 4 "
                "and grad_ld >= D (n=%lld V=%lld D=%lld)", SISA_EMBED_MAX_IDS, (long long)n, (long long)V, (long long)D);
  if (!aligned16(dw) || (n > 0 && (!aligned16(grad) || grad_ld % 4 || reinterpret_cast<uintptr_t>(ids) % 8)))
    return fail(SISA_ERR_ALIGN, "sisa_embedding_bwd: dw and grad 16-byte aligned, grad_ld a multiple of 4, ids 8-byte "
                "aligned");
  int rc;
  sisa::DeviceScope scope;
  if ((rc = scope.bind(dw))) return rc;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, scope.device());
  const sisa::EmbedBwd p{ids, grad, dw, n, V, D, grad_ld, 0};
  cudaError_t e = sisa::launch_embed_bwd(p, sms, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_embedding_bwd launch");
}

int sisa_split_rows(const float* src, int64_t src_ld, float* dst0, float* dst1, int64_t dst_ld, int64_t rows,
                    int64_t cols, int64_t block, void* stream) {
  if (!src || !dst0 || !dst1) return fail(SISA_ERR_VALUE, "sisa_split_rows: null pointer");
  if (rows < 0 || cols < 0 || block < 1 || rows % block || cols % 4 || src_ld < cols || dst_ld < cols ||
      rows > ((int64_t)1 << 40) / (cols > 0 ? cols : 1))
    return fail(SISA_ERR_VALUE, "sisa_split_rows: need rows a multiple of block >= 1, cols a multiple of 4 and "
                "row strides >= cols (rows=%lld cols=%lld block=%lld)", (long long)rows, (long long)cols,
                (long long)block);
  if (!aligned16(src) || !aligned16(dst0) || !aligned16(dst1) || src_ld % 4 || dst_ld % 4)
    return fail(SISA_ERR_ALIGN, "sisa_split_rows: pointers must be 16-byte aligned and row strides multiples of 4");
  if (rows == 0 || cols == 0) return SISA_OK;
  int rc;
  sisa::DeviceScope scope;
  if ((rc = scope.bind(dst0))) return rc;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, scope.device());
  const sisa::SplitRows p{src, dst0, dst1, rows, cols, src_ld, dst_ld, block};
  cudaError_t e = sisa::launch_split_rows(p, sms, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_split_rows launch");
}

int sisa_copy_rows(const sisa_row_copy* jobs, int njobs, int64_t max_vectors, int dtype, int32_t* status,
                   void* stream) {
  (void)status;
  int rc;
  if ((rc = check_dtype(dtype))) return rc;
  if (njobs < 0 || njobs > 65535 || max_vectors < 0) return fail(SISA_ERR_VALUE, "sisa_copy_rows: need 0 <= njobs <= 65535");
  if (njobs == 0) return SISA_OK;
  if (!jobs || !aligned16(jobs)) return fail(SISA_ERR_ALIGN, "sisa_copy_rows: jobs must be a 16-byte aligned device array");
  static_assert(sizeof(sisa_row_copy) == sizeof(sisa::RowCopy), "job layout");
  sisa::DeviceScope scope;
  if ((rc = scope.bind(jobs))) return rc;
  cudaError_t e = sisa::launch_copy_rows(reinterpret_cast<const sisa::RowCopy*>(jobs), njobs, max_vectors,
                                         dtype == SISA_F16 ? 1 : 0, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_copy_rows launch");
}

// ------------------------------------------------------------------------------------ SwiGLU gate/up GEMM
int sisa_gemm_swiglu(const void* x, int64_t x_ld, const void* w, int64_t w_ld, void* gu, int64_t gu_ld, void* a,
                     int64_t a_ld, int64_t rows, int64_t d_ff, int64_t K, int dtype, int32_t* status, void* stream) {
  int rc;
  if ((rc = check_dtype(dtype))) return rc;
  if (!x || !w || !a) return fail(SISA_ERR_VALUE, "sisa_gemm_swiglu: null pointer");
  const int64_t lim = (int64_t)1 << 30;
  if (rows < 1 || d_ff < 8 || d_ff % 8 || K < 1 || rows > lim || 2 * d_ff > lim || K > lim)
    return fail(SISA_ERR_VALUE, "sisa_gemm_swiglu: need rows >= 1, d_ff a positive multiple of 8, K >= 1 "
                "(rows=%lld d_ff=%lld K=%lld)", (long long)rows, (long long)d_ff, (long long)K);
  if (!aligned16(x) || !aligned16(w) || !aligned16(a) || x_ld % 8 || w_ld % 8 || a_ld % 8 || x_ld < K ||
      w_ld < K || a_ld < d_ff || (gu && (!aligned16(gu) || gu_ld % 8 || gu_ld < 2 * d_ff)))
    return fail(SISA_ERR_ALIGN, "sisa_gemm_swiglu: rows must be 16-byte aligned (ld multiple of 8 and >= width)");
  sisa::DeviceScope scope;
  if ((rc = scope.bind(x))) return rc;
  const CUtensorMapDataType dt = dtype == SISA_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  sisa::GemmParams p;
  memset(&p, 0, sizeof(p));
  if ((rc = map_operand(&p.tm_a, x, x_ld, 0, rows, K, dt, "x"))) return rc;
  if ((rc = map_operand(&p.tm_b, w, w_ld, 0, 2 * d_ff, K, dt, "w"))) return rc;
  if (gu) {
    if ((rc = map_output(&p.tm_c, gu, gu_ld, rows, 2 * d_ff, dtype))) return rc;
  } else {
    p.skip_c = 1;
  }
  {
    EncodeTiledFn enc = encode_fn();
    cuuint64_t dims[2] = {(cuuint64_t)d_ff, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(a_ld * 2)};
    cuuint32_t box[2] = {32, 32}, es[2] = {1, 1};
    if (enc(&p.tm_c2, dt, 2, a, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return fail(SISA_ERR_ALIGN, "a: cuTensorMapEncodeTiled failed");
  }
  p.ldc = gu ? gu_ld : 0;
  p.M = (int)rows; p.N = (int)(2 * d_ff); p.K = (int)K;
  p.num_m = (int)((rows + 255) / 256);
  p.status = status;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, scope.device());
  cudaError_t e = sisa::launch_gemm_swiglu(p, dtype, sms, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_gemm_swiglu launch");
}

// ------------------------------------------------------------------------------------ GEMM
int64_t sisa_gemm_workspace(int64_t M, int64_t N, int64_t K, int out_dtype) {
  if (M < 1 || N < 1 || K < 1) return 0;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaGetLastError();
  const int out = out_dtype == SISA_F32 ? sisa::GEMM_OUT_F32 : out_dtype == SISA_BF16 ? sisa::GEMM_OUT_BF16
                                                                                        : sisa::GEMM_OUT_F16;
  return sisa::gemm_workspace_bytes(M, N, K, out, sms);
}

// The checks and the launch shared by sisa_gemm and sisa_gemm_bias_cols; the bias (if any) has been
// checked by the caller and covers columns [bias_c0, bias_c1).
static int gemm_impl(const char* name, const void* a, int64_t lda, int a_mn, const void* b, int64_t ldb, int b_mn,
                     void* c, int64_t ldc, int64_t M, int64_t N, int64_t K, int dtype, int out_dtype, int accumulate,
                     const void* bias, int bias_dtype, int64_t bias_c0, int64_t bias_c1, int bias_vec,
                     int bias_round, void* workspace, int64_t workspace_bytes, int32_t* status, void* stream) {
  int rc;
  if ((rc = check_dtype(dtype))) return rc;
  if (!a || !b || !c) return fail(SISA_ERR_VALUE, "%s: null pointer", name);
  if ((a_mn != 0 && a_mn != 1) || (b_mn != 0 && b_mn != 1))
    return fail(SISA_ERR_VALUE, "%s: a_mn and b_mn are 0 (K-major) or 1 (MN-major)", name);
  if (out_dtype != SISA_F32 && out_dtype != SISA_BF16 && out_dtype != SISA_F16)
    return fail(SISA_ERR_TYPE, "%s: out_dtype must be SISA_F32, SISA_BF16 or SISA_F16 (got %d)", name, out_dtype);
  if (accumulate && out_dtype != SISA_F32) return fail(SISA_ERR_VALUE, "%s: accumulate needs an fp32 output", name);
  const int64_t lim = (int64_t)1 << 30;
  if (M < 1 || N < 1 || K < 1 || M > lim || N > lim || K > lim)
    return fail(SISA_ERR_VALUE, "%s: need 1 <= M, N, K <= 2^30 (M=%lld N=%lld K=%lld)", name, (long long)M,
                (long long)N, (long long)K);
  const int64_t osz = out_dtype == SISA_F32 ? 4 : 2;
  if (!aligned16(a) || !aligned16(b) || !aligned16(c) || lda % 8 || ldb % 8 || (ldc * osz) % 16 ||
      lda < (a_mn ? M : K) || ldb < (b_mn ? N : K) || ldc < N)
    return fail(SISA_ERR_ALIGN, "%s: operands and C must be 16-byte aligned with row strides of whole "
                "16-byte units covering their rows (lda=%lld ldb=%lld ldc=%lld)", name, (long long)lda, (long long)ldb,
                (long long)ldc);
  if (workspace && (!aligned16(workspace) || workspace_bytes < 0))
    return fail(SISA_ERR_VALUE, "%s: workspace must be 16-byte aligned", name);
  sisa::DeviceScope scope;
  if ((rc = scope.bind(a))) return rc;
  const CUtensorMapDataType dt = dtype == SISA_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  sisa::GemmParams p;
  memset(&p, 0, sizeof(p));
  p.bias = bias;
  p.bias_dtype = bias_dtype == SISA_F32 ? 2 : bias_dtype == SISA_F16 ? 1 : 0;
  p.bias_c0 = (int)bias_c0; p.bias_c1 = (int)bias_c1; p.bias_vec = bias_vec; p.bias_round = bias_round;
  if (workspace && workspace_bytes > 0) { p.sema = static_cast<uint32_t*>(workspace); p.ws_bytes = workspace_bytes; }
  if ((rc = map_operand(&p.tm_a, a, lda, a_mn, M, K, dt, "a"))) return rc;
  if ((rc = map_operand(&p.tm_b, b, ldb, b_mn, N, K, dt, "b"))) return rc;
  if ((rc = map_output(&p.tm_c, c, ldc, M, N, out_dtype))) return rc;
  p.ldc = ldc;
  p.M = (int)M; p.N = (int)N; p.K = (int)K;
  p.num_m = (int)((M + 255) / 256);
  p.accumulate = accumulate ? 1 : 0;
  p.status = status;
  const int out = out_dtype == SISA_F32 ? sisa::GEMM_OUT_F32 : out_dtype == SISA_BF16 ? sisa::GEMM_OUT_BF16
                                                                                        : sisa::GEMM_OUT_F16;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, scope.device());
  int tile = -1;                             // chosen per problem; the variable forces a shape (tuning, tests)
  if (const char* t = getenv("SISA_GEMM_TILE")) {
    if (!strcmp(t, "wide")) tile = 1;
    else if (!strcmp(t, "narrow")) tile = 0;
  }
  cudaError_t e = sisa::launch_gemm(p, dtype, a_mn, b_mn, out, tile, sms, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, name);
}


int sisa_gemm(const void* a, int64_t lda, int a_mn, const void* b, int64_t ldb, int b_mn, void* c, int64_t ldc,
              int64_t M, int64_t N, int64_t K, int dtype, int out_dtype, int accumulate, const void* bias,
              int bias_dtype, void* workspace, int64_t workspace_bytes, int32_t* status, void* stream) {
  if (bias && ((bias_dtype != SISA_BF16 && bias_dtype != SISA_F16 && bias_dtype != SISA_F32) || !aligned16(bias)))
    return fail(SISA_ERR_VALUE, "sisa_gemm: bias must be 16-byte aligned SISA_BF16, SISA_F16 or SISA_F32");
  return gemm_impl("sisa_gemm", a, lda, a_mn, b, ldb, b_mn, c, ldc, M, N, K, dtype, out_dtype, accumulate, bias,
                   bias_dtype, 0, N, 1, 0, workspace, workspace_bytes, status, stream);
}

int sisa_gemm_bias_cols(const void* a, int64_t lda, int a_mn, const void* b, int64_t ldb, int b_mn, void* c,
                        int64_t ldc, int64_t M, int64_t N, int64_t K, int dtype, int out_dtype, int accumulate,
                        const void* bias, int bias_dtype, int64_t bias_col0, int64_t bias_ncols, int bias_round,
                        void* workspace, int64_t workspace_bytes, int32_t* status, void* stream) {
  if (!bias && bias_ncols > 0) return fail(SISA_ERR_VALUE, "sisa_gemm_bias_cols: null bias");
  if (bias_dtype != SISA_BF16 && bias_dtype != SISA_F16 && bias_dtype != SISA_F32)
    return fail(SISA_ERR_TYPE, "sisa_gemm_bias_cols: bias_dtype must be SISA_BF16, SISA_F16 or SISA_F32");
  const uintptr_t esz = bias_dtype == SISA_F32 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(bias) % esz)
    return fail(SISA_ERR_ALIGN, "sisa_gemm_bias_cols: bias must be aligned to its element size");
  if (bias_col0 < 0 || bias_ncols < 0 || bias_col0 > N || bias_ncols > N - bias_col0)
    return fail(SISA_ERR_VALUE, "sisa_gemm_bias_cols: columns [%lld, %lld) lie outside [0, N=%lld)",
                (long long)bias_col0, (long long)(bias_col0 + bias_ncols), (long long)N);
  if (bias_round != 0 && bias_round != 1)
    return fail(SISA_ERR_VALUE, "sisa_gemm_bias_cols: bias_round is 0 or 1");
  if (bias_round && out_dtype != dtype)
    return fail(SISA_ERR_VALUE, "sisa_gemm_bias_cols: bias_round needs a 16-bit output of the operands' type");
  if (bias_ncols == 0) bias = nullptr;      // no column takes a bias
  const int vec = aligned16(bias) && bias_col0 % 8 == 0;
  return gemm_impl("sisa_gemm_bias_cols", a, lda, a_mn, b, ldb, b_mn, c, ldc, M, N, K, dtype, out_dtype, accumulate,
                   bias, bias_dtype, bias_col0, bias_col0 + bias_ncols, vec, bias_round, workspace, workspace_bytes,
                   status, stream);
}

// ------------------------------------------------------------------------------------ norm, SwiGLU
static int check_edtype(int dt, const char* what) {
  if (dt != SISA_BF16 && dt != SISA_F16 && dt != SISA_F32)
    return fail(SISA_ERR_TYPE, "%s: dtype must be SISA_BF16, SISA_F16 or SISA_F32", what);
  return SISA_OK;
}

int64_t sisa_rmsnorm_bwd_workspace(int64_t rows, int64_t d) {
  return rows < 1 || d < 1 ? 0 : sisa::norm_bwd_partials(rows, 0) * sisa::norm_part_cols(d, 0) * 4;
}
int64_t sisa_norm_bwd_workspace(int64_t rows, int64_t d, int64_t n_proj) {
  return rows < 1 || d < 1 || n_proj < 0 ? 0 : sisa::norm_bwd_partials(rows, n_proj) * sisa::norm_part_cols(d, n_proj) * 4;
}

static bool norm_shape_ok(int64_t rows, int64_t d) { return rows >= 1 && d >= 1 && d <= (1 << 20) && rows <= ((int64_t)1 << 34); }

// A row operand: null is allowed when `optional`; else its type and stride are checked.
static int check_rows_arg(const void* ptr, int64_t ld, int dt, int64_t d, bool optional, const char* what) {
  if (!ptr) return optional ? SISA_OK : fail(SISA_ERR_VALUE, "%s: null pointer", what);
  int rc;
  if ((rc = check_edtype(dt, what))) return rc;
  if (ld < d) return fail(SISA_ERR_VALUE, "%s: row stride %lld < d %lld", what, (long long)ld, (long long)d);
  return SISA_OK;
}

static int check_proj(int64_t n_proj, int64_t d, const char* what) {
  if (n_proj < 0 || n_proj > 32 || n_proj * d * 4 > 200 * 1024)
    return fail(SISA_ERR_VALUE, "%s: n_proj %lld with d %lld (at most 32 columns and 200 KB of weights)", what,
                (long long)n_proj, (long long)d);
  return SISA_OK;
}

int sisa_norm_fwd(const sisa_norm_fwd_args* a, int32_t* status, void* stream) {
  if (!a) return fail(SISA_ERR_VALUE, "sisa_norm_fwd: null args");
  if (!norm_shape_ok(a->rows, a->d))
    return fail(SISA_ERR_VALUE, "sisa_norm_fwd: bad shape (rows %lld, d %lld)", (long long)a->rows, (long long)a->d);
  if (a->n_out < 1 || a->n_out > 2) return fail(SISA_ERR_VALUE, "sisa_norm_fwd: n_out must be 1 or 2");
  int rc;
  if ((rc = check_rows_arg(a->x, a->x_ld, a->x_dtype, a->d, false, "sisa_norm_fwd x")) ||
      (rc = check_rows_arg(a->res, a->res_ld, a->res_dtype, a->d, true, "sisa_norm_fwd res")) ||
      (rc = check_rows_arg(a->xsum, a->xsum_ld, a->x_dtype, a->d, true, "sisa_norm_fwd xsum")) ||
      (rc = check_rows_arg(a->y[0], a->y_ld[0], a->y_dtype[0], a->d, false, "sisa_norm_fwd y[0]")) ||
      (a->n_out > 1 && (rc = check_rows_arg(a->y[1], a->y_ld[1], a->y_dtype[1], a->d, false, "sisa_norm_fwd y[1]"))) ||
      (rc = check_proj(a->n_proj, a->d, "sisa_norm_fwd")))
    return rc;
  if (!a->weight || !a->rstd) return fail(SISA_ERR_VALUE, "sisa_norm_fwd: null weight or rstd");
  if (a->xsum && !a->res) return fail(SISA_ERR_VALUE, "sisa_norm_fwd: xsum without res");
  if (a->n_proj > 0 && (!a->proj_w || !a->proj_b || !a->proj_out))
    return fail(SISA_ERR_VALUE, "sisa_norm_fwd: n_proj > 0 needs proj_w, proj_b and proj_out");
  sisa::NormFwd p{};
  p.x = a->x; p.xs = a->x_ld; p.xdt = a->x_dtype;
  p.res = a->res; p.ress = a->res_ld; p.resdt = a->res ? a->res_dtype : 2;
  p.xsum = a->xsum; p.xsums = a->xsum_ld;
  p.w = a->weight; p.rows = a->rows; p.d = a->d; p.eps = a->eps;
  p.nout = a->n_out;
  for (int k = 0; k < 2; ++k) {
    const bool on = k < a->n_out;
    p.y[k] = on ? a->y[k] : nullptr; p.ys[k] = on ? a->y_ld[k] : 0; p.ydt[k] = on ? a->y_dtype[k] : 2;
  }
  p.rstd = a->rstd;
  p.pw = a->proj_w; p.pb = a->proj_b; p.np = (int)a->n_proj; p.pz = a->proj_out;
  p.status = status;
  cudaError_t e = sisa::launch_norm_fwd(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_norm_fwd launch");
}

int sisa_norm_bwd(const sisa_norm_bwd_args* a, int32_t* status, void* stream) {
  if (!a) return fail(SISA_ERR_VALUE, "sisa_norm_bwd: null args");
  if (!norm_shape_ok(a->rows, a->d))
    return fail(SISA_ERR_VALUE, "sisa_norm_bwd: bad shape (rows %lld, d %lld)", (long long)a->rows, (long long)a->d);
  int rc;
  if ((rc = check_rows_arg(a->v, a->v_ld, a->v_dtype, a->d, false, "sisa_norm_bwd v")) ||
      (rc = check_rows_arg(a->dy[0], a->dy_ld[0], a->dy_dtype[0], a->d, true, "sisa_norm_bwd dy[0]")) ||
      (rc = check_rows_arg(a->dy[1], a->dy_ld[1], a->dy_dtype[1], a->d, true, "sisa_norm_bwd dy[1]")) ||
      (rc = check_rows_arg(a->dv_in, a->dv_in_ld, a->dv_in_dtype, a->d, true, "sisa_norm_bwd dv_in")) ||
      (rc = check_rows_arg(a->dx, a->dx_ld, a->dx_dtype, a->d, false, "sisa_norm_bwd dx")) ||
      (rc = check_rows_arg(a->dres, a->dres_ld, a->dres_dtype, a->d, true, "sisa_norm_bwd dres")) ||
      (rc = check_proj(a->n_proj, a->d, "sisa_norm_bwd")))
    return rc;
  if (!a->weight || !a->rstd) return fail(SISA_ERR_VALUE, "sisa_norm_bwd: null weight or rstd");
  if (a->n_proj > 0 && (!a->proj_w || !a->dproj_out))
    return fail(SISA_ERR_VALUE, "sisa_norm_bwd: n_proj > 0 needs proj_w and dproj_out");
  if ((a->dweight || a->dproj_w || a->dproj_b) && !a->workspace)
    return fail(SISA_ERR_VALUE, "sisa_norm_bwd: weight gradients need the workspace");
  if (a->n_proj == 0 && (a->dproj_w || a->dproj_b))
    return fail(SISA_ERR_VALUE, "sisa_norm_bwd: dproj_w / dproj_b without a projection");
  sisa::NormBwd p{};
  p.v = a->v; p.vs = a->v_ld; p.vdt = a->v_dtype;
  p.w = a->weight; p.rstd = a->rstd; p.rows = a->rows; p.d = a->d;
  for (int k = 0; k < 2; ++k) { p.dy[k] = a->dy[k]; p.dys[k] = a->dy_ld[k]; p.dydt[k] = a->dy[k] ? a->dy_dtype[k] : 2; }
  p.dvin = a->dv_in; p.dvins = a->dv_in_ld; p.dvindt = a->dv_in ? a->dv_in_dtype : 2;
  p.pw = a->proj_w; p.np = (int)a->n_proj; p.dz = a->dproj_out;
  p.dx = a->dx; p.dxs = a->dx_ld; p.dxdt = a->dx_dtype;
  p.dres = a->dres; p.dress = a->dres_ld; p.dresdt = a->dres ? a->dres_dtype : 2;
  p.dw = a->dweight; p.dpw = a->dproj_w; p.dpb = a->dproj_b;
  p.part = static_cast<float*>(a->workspace);
  p.status = status;
  cudaError_t e = sisa::launch_norm_bwd(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_norm_bwd launch");
}

int sisa_rmsnorm_fwd(const void* x, int64_t x_ld, int x_dtype, const float* w, int64_t rows, int64_t d, float eps,
                     void* y, int64_t y_ld, int y_dtype, float* rstd, int32_t* status, void* stream) {
  sisa_norm_fwd_args a{};
  a.x = x; a.x_ld = x_ld; a.x_dtype = x_dtype; a.weight = w; a.rows = rows; a.d = d; a.eps = eps;
  a.n_out = 1; a.y[0] = y; a.y_ld[0] = y_ld; a.y_dtype[0] = y_dtype; a.rstd = rstd;
  return sisa_norm_fwd(&a, status, stream);
}

int sisa_rmsnorm_bwd(const void* dy, int64_t dy_ld, int dy_dtype, const void* x, int64_t x_ld, int x_dtype,
                     const float* w, const float* rstd, int64_t rows, int64_t d, void* dx, int64_t dx_ld, int dx_dtype,
                     float* dw, void* workspace, int32_t* status, void* stream) {
  if (!dy) return fail(SISA_ERR_VALUE, "sisa_rmsnorm_bwd: null pointer");
  sisa_norm_bwd_args a{};
  a.v = x; a.v_ld = x_ld; a.v_dtype = x_dtype; a.weight = w; a.rstd = rstd; a.rows = rows; a.d = d;
  a.dy[0] = dy; a.dy_ld[0] = dy_ld; a.dy_dtype[0] = dy_dtype;
  a.dx = dx; a.dx_ld = dx_ld; a.dx_dtype = dx_dtype; a.dweight = dw; a.workspace = workspace;
  return sisa_norm_bwd(&a, status, stream);
}

static int check_swiglu(int64_t rows, int64_t f, int dtype, const char* what) {
  int rc;
  if ((rc = check_edtype(dtype, what))) return rc;
  if (rows < 1 || f < 1 || rows * ((f + 7) / 8) >= ((int64_t)1 << 31))
    return fail(SISA_ERR_VALUE, "%s: bad shape (rows %lld, f %lld)", what, (long long)rows, (long long)f);
  return SISA_OK;
}

int sisa_swiglu_fwd(const void* g, int64_t g_ld, const void* u, int64_t u_ld, int64_t rows, int64_t f, int dtype,
                    void* a, int64_t a_ld, int32_t* status, void* stream) {
  (void)status;
  int rc;
  if ((rc = check_swiglu(rows, f, dtype, "sisa_swiglu_fwd"))) return rc;
  if (!g || !u || !a || g_ld < f || u_ld < f || a_ld < f) return fail(SISA_ERR_VALUE, "sisa_swiglu_fwd: null pointer or stride");
  sisa::SwiGluFwd p{g, g_ld, u, u_ld, rows, f, a, a_ld, dtype};
  cudaError_t e = sisa::launch_swiglu_fwd(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_swiglu_fwd launch");
}

int sisa_swiglu_bwd(const void* da, int64_t da_ld, const void* g, int64_t g_ld, const void* u, int64_t u_ld,
                    int64_t rows, int64_t f, int dtype, void* dg, int64_t dg_ld, void* du, int64_t du_ld,
                    int32_t* status, void* stream) {
  (void)status;
  int rc;
  if ((rc = check_swiglu(rows, f, dtype, "sisa_swiglu_bwd"))) return rc;
  if (!da || !g || !u || !dg || !du || da_ld < f || g_ld < f || u_ld < f || dg_ld < f || du_ld < f)
    return fail(SISA_ERR_VALUE, "sisa_swiglu_bwd: null pointer or stride");
  sisa::SwiGluBwd p{da, da_ld, g, g_ld, u, u_ld, rows, f, dg, dg_ld, du, du_ld, dtype};
  cudaError_t e = sisa::launch_swiglu_bwd(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? SISA_OK : cuda_fail(e, "sisa_swiglu_bwd launch");
}

}  // extern "C"
