/* sisa_b200.h - C ABI of the B200 (sm_100a) SISA hot path.
 *
 * Every entry point takes raw device pointers, int64 shapes and element strides, a cudaStream_t
 * (passed as void*) and a device int32 status word, and returns an int error code (SISA_OK = 0).
 * Nothing in this library allocates device memory, synchronises the host or throws across the
 * ABI: the caller owns every output and workspace buffer, and the work is ordered only by the
 * stream that is passed in. Kernels never trap; run-time conditions are OR-ed into *status
 * (SISA_ST_* bits) and left for the caller to read. Entry points that need a current context (to
 * encode TMA tensor maps) make the device that owns their data current for the length of the call
 * and give the calling thread back its previous context before they return.
 *
 * Reference interfaces (tlstngud/sisa, paths inside that project) that each entry point
 * replaces are cited beside it.
 */
#ifndef SISA_B200_H
#define SISA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- device status bits (OR-ed into the caller's int32 status word) ---- */
#define SISA_ST_NONFINITE   1  /* NaN/inf reached a score, lse or a block total (fused_prep.py:502-523) */
#define SISA_ST_NONMONOTONE 2  /* g rose by more than 1e-3 between neighbours (attention.py:123-125,675-683) */
#define SISA_ST_TIMEOUT     4  /* a bounded device wait gave up; results are invalid */
#define SISA_ST_BAD_SEED    8  /* linear-CE backward seed differs from the promised grad_scale (linear_ce.py:202-206) */
#define SISA_ST_BAD_POS    16  /* a decode position read on the device lay outside the cache; nothing was written */

/* ---- return codes ---- */
#define SISA_OK              0
#define SISA_ERR_VALUE       1  /* shape / layout / argument error (Python: ValueError) */
#define SISA_ERR_TYPE        2  /* dtype error (Python: TypeError) */
#define SISA_ERR_ALIGN       3  /* pointer or stride alignment the kernels cannot take (ValueError) */
#define SISA_ERR_CUDA        4  /* a CUDA runtime/driver call failed (RuntimeError) */
#define SISA_ERR_UNSUPPORTED 5  /* device is not sm_100 (RuntimeError) */

/* ---- element types of low-precision operands ---- */
#define SISA_BF16 0
#define SISA_F16  1
#define SISA_F32  2   /* only where an entry point says so */

/* A (B, H, L, X) view: element strides of the first three axes; the last axis is contiguous. */
typedef struct sisa_view4 {
  void* data;
  int64_t stride_b;
  int64_t stride_h;
  int64_t stride_l;
} sisa_view4;

/* Library version string and the message of the last error returned on this host thread. */
const char* sisa_version(void);
const char* sisa_last_error(void);

/* 0 when `device` is an sm_100 GPU this library was built for (else SISA_ERR_UNSUPPORTED). */
int sisa_device_check(int device);

/* Column layout of the fused projection for n_head heads (d_head 64, d_state 32):
 * out[0..8] = start columns Q, K, V, B, C, TH, A, then NTOT and NPAD.
 * Replaces sisa.kernels.fused_prep.fused_layout (src/sisa/kernels/fused_prep.py:71-96). */
int sisa_fused_layout(int64_t n_head, int64_t* out9);

/* Row length Lp of the position planes: L rounded up to a multiple of 4, so that every plane starts
 * on a 16-byte boundary (the tensor-memory-access loads need 16-byte strides). */
int64_t sisa_pos_len(int64_t L);

/* Workspace sizes in bytes for the entry points below (caller allocates; 256-byte aligned). */
int64_t sisa_prep_fwd_workspace(int64_t B, int64_t H, int64_t L);   /* per-block scan prefixes, fp32 */
int64_t sisa_prep_bwd_workspace(int64_t B, int64_t H, int64_t L);   /* fp64 block totals + fp32 per-token d Phi */
int64_t sisa_attn_bwd_workspace(int64_t B, int64_t H, int64_t L);   /* per-row statistics */

/* Fused preparation, forward (src/sisa/kernels/fused_prep.py:247-352, launched at :527-564):
 *   g = cumsum(-softplus(alpha)), F = cumsum(logsigmoid(z)), Phi = cumsum(theta),
 *   c_rot/b_rot = pair rotation R(Phi) of the C/B columns (fp32 math, one rounding).
 * proj: (B, L, NPAD) in `dtype` with element strides proj_sb, proj_sl (column stride 1).
 * z: (B, L, H) fp32 with strides z_sb, z_sl (head stride 1), or NULL for no forget gate.
 * c_rot, b_rot: (B, H, L, 32) contiguous, `dtype`.
 * pos: (B, H, 4, Lp) fp32 contiguous planes, Lp = sisa_pos_len(L): plane 0 g, plane 1 F, plane 2 rowf,
 *   plane 3 colf, where rowf/colf are the decay factors relative to the start/end of the position's
 *   64-row block. Entries [L, Lp) of each plane are not written. (The reference keeps g and F as
 *   separate (B, H, L) tensors; one planar record lets one bulk copy fetch all four per key tile.)
 * workspace: sisa_prep_fwd_workspace(B, H, L) bytes. */
int sisa_prep_fwd(const void* proj, int64_t B, int64_t L, int64_t H, int64_t proj_sb, int64_t proj_sl,
                  int dtype, const float* z, int64_t z_sb, int64_t z_sl,
                  void* c_rot, void* b_rot, float* pos, void* workspace,
                  int32_t* status, void* stream);

/* Position records for the unfused entry point (src/sisa/kernels/attention.py:129-153):
 * pos planes {g, fgate (0 if NULL), rowf, colf}, (B, H, 4, Lp) as above, from g (B, H, L) and
 * fgate (B, H, L) fp32 with the given element strides; sets SISA_ST_NONMONOTONE when g rises by
 * more than 1e-3. */
int sisa_pack_positions(const float* g, int64_t g_sb, int64_t g_sh, int64_t g_sl,
                        const float* fgate, int64_t f_sb, int64_t f_sh, int64_t f_sl,
                        int64_t B, int64_t H, int64_t L, float* pos, int32_t* status, void* stream);

/* Exact SISA attention forward on tcgen05 (src/sisa/kernels/attention.py:177-296, host 686-727):
 *   s_ij = q_i.k_j/8 + lam_h exp(g_i-g_j) (c_i.b_j) + (F_i - F_j), j <= i;  o = softmax(s) v.
 * q, k, v: (B, H, L, 64) views in `dtype`; c, b: (B, H, L, 32) views in `dtype`.
 * pos: (B, H, 4, Lp) planes from sisa_prep_fwd / sisa_pack_positions. lam: (H,) fp32.
 * o: (B, H, L, 64) view in `dtype`. lse: (B, H, L) fp32 contiguous, log2 units.
 * o32: (B, H, L, 64) fp32 contiguous o'' for the exact-delta backward (the self-normalised output,
 *   already snapped to o where the two agree to 2^-15), or NULL when no backward follows. All views: 16-byte aligned rows, strides multiple of 8. */
int sisa_attn_fwd(const sisa_view4* q, const sisa_view4* k, const sisa_view4* v,
                  const sisa_view4* c, const sisa_view4* b, const float* pos, const float* lam,
                  int64_t B, int64_t H, int64_t L, int dtype,
                  const sisa_view4* o, float* lse, float* o32, int32_t* status, void* stream);

/* Exact-delta backward on tcgen05 (src/sisa/kernels/attention.py:300-663, host 730-784):
 * dq, dk, dv: (B, H, L, 64) views in `dtype` (may alias columns of a fused d_proj);
 * dc, db: (B, H, L, 32) fp32 views; dg, dF: (B, H, L) fp32 contiguous (dF may be NULL when
 * the forward had no forget gate); dlam: (H,) fp32, summed in fp64 and rounded once.
 * workspace: sisa_attn_bwd_workspace(B, H, L) bytes. Deterministic (no atomics on data). */
int sisa_attn_bwd(const sisa_view4* q, const sisa_view4* k, const sisa_view4* v,
                  const sisa_view4* c, const sisa_view4* b, const float* pos, const float* lam,
                  const sisa_view4* o, const sisa_view4* dout, const float* lse, const float* o32,
                  int64_t B, int64_t H, int64_t L, int dtype,
                  const sisa_view4* dq, const sisa_view4* dk, const sisa_view4* dv,
                  const sisa_view4* dc, const sisa_view4* db, float* dg, float* dF, float* dlam,
                  void* workspace, int32_t* status, void* stream);

/* Fused preparation, backward (src/sisa/kernels/fused_prep.py:385-494, launched at :622-633):
 * reverse scans in fp64 -> d alpha, dz, d theta; inverse rotation of dc/db; zero padding columns.
 * dproj: (B, L, NPAD) `dtype` with strides dproj_sb, dproj_sl; only the B, C, TH, A and padding
 * columns are written here (the Q, K, V columns come from sisa_attn_bwd).
 * dc, db: (B, H, L, 32) fp32 contiguous; dg, dF: (B, H, L) fp32 (dF NULL without z).
 * dz: (B, L, H) fp32 contiguous (ignored without z). tot: the forward's workspace (per-block scan prefixes).
 * workspace: sisa_prep_bwd_workspace(B, H, L) bytes. */
int sisa_prep_bwd(const void* proj, int64_t B, int64_t L, int64_t H, int64_t proj_sb, int64_t proj_sl,
                  int dtype, const float* z, int64_t z_sb, int64_t z_sl, const void* tot,
                  const float* dc, const float* db, const float* dg, const float* dF,
                  void* dproj, int64_t dproj_sb, int64_t dproj_sl, float* dz,
                  void* workspace, int32_t* status, void* stream);

/* Chunked linear + cross-entropy over a tied LM head (src/sisa/kernels/linear_ce.py:60-196).
 * sisa_lce_logits: logits (R, Vp) = x (R, D) . w (Vp, D)^T on tcgen05 CTA pairs (the sisa_gemm kernel with
 *   a log-sum-exp epilogue), stored in `dtype` (rounded as under autocast) at logits (row stride
 *   logits_ld), plus per (row, 256-column tile) online max/sum-exp over the first V columns and the
 *   label's logit, kept in `workspace` (sisa_lce_workspace(R, Vp) bytes, 16-byte aligned). D a multiple
 *   of 64, Vp >= V a multiple of 128 (the reference's padding), w rows [V, Vp) zero.
 * sisa_lce_grad: per row lse, loss_rows[r] = lse - logit[label] (0 for ignore_index), and, when
 *   compute_grad, G = (softmax - onehot) * (*inv_n) * grad_scale written over the logits in place
 *   (padding columns 0). inv_n is a device scalar (1 / number of non-ignored rows).
 * The gradient GEMMs dx = G . w and dw += G^T . x are sisa_gemm calls. */
int64_t sisa_lce_workspace(int64_t R, int64_t Vp);
int sisa_lce_logits(const void* x, int64_t R, int64_t D, int64_t x_ld, const void* w, int64_t V, int64_t Vp,
                    int64_t w_ld, int dtype, const int64_t* labels, void* logits, int64_t logits_ld,
                    void* workspace, int32_t* status, void* stream);
int sisa_lce_grad(void* logits, int64_t logits_ld, int64_t R, int64_t V, int64_t Vp, int dtype,
                  const int64_t* labels, int64_t ignore_index, const float* inv_n, float grad_scale,
                  int compute_grad, const void* workspace, float* loss_rows, int32_t* status, void* stream);
/* The backward of the linear-CE (src/sisa/kernels/linear_ce.py:200-217, grad_output * dx / dW):
 * out[i] = x[i] * (*seed) in out_dtype (SISA_BF16, SISA_F16 or SISA_F32), or x scaled in place when out
 * is NULL (SISA_F32). In place with a seed of exactly 1 nothing is written. seed is a device scalar. */
int sisa_lce_seed_scale(float* x, int64_t n, const float* seed, void* out, int out_dtype, int32_t* status,
                        void* stream);

/* C (+)= A . B^T (+ bias) on CTA pairs of tcgen05 tensor cores: the linear-CE gradient GEMMs (the
 * torch.matmul calls of src/sisa/kernels/linear_ce.py:170-178) and the model's linears under autocast
 * (F.linear of src/sisa/modeling.py:39-49, 213-222, 255). A is M x K and B is N x K in `dtype`
 * (SISA_BF16 / SISA_F16), each K-major (element (r, k) at r * ld + k; a_mn / b_mn = 0) or MN-major
 * (element (r, k) at k * ld + r; = 1); C is M x N row-major in out_dtype (SISA_F32, SISA_BF16 or
 * SISA_F16) with fp32 accumulation and one rounding; accumulate = 1 (fp32 C only) adds to C. bias
 * (optional, N values of bias_dtype) is added in fp32 before the rounding. workspace (optional,
 * sisa_gemm_workspace(M, N, K, out_dtype) bytes on the current device, 0 when no split is wanted; used
 * by one stream at a time) lets a small fp32 problem split K across CTA pairs: each slice writes an
 * fp32 partial and the last slice of a tile sums them in slice order (deterministic). Pointers 16-byte
 * aligned, row strides in elements covering a row and whole 16-byte units; 1 <= M, N, K <= 2^30.
 * Waits are bounded (SISA_ST_TIMEOUT). */
int64_t sisa_gemm_workspace(int64_t M, int64_t N, int64_t K, int out_dtype);
int sisa_gemm(const void* a, int64_t lda, int a_mn, const void* b, int64_t ldb, int b_mn, void* c, int64_t ldc,
              int64_t M, int64_t N, int64_t K, int dtype, int out_dtype, int accumulate, const void* bias,
              int bias_dtype, void* workspace, int64_t workspace_bytes, int32_t* status, void* stream);

/* sisa_gemm with a bias that covers only some columns: bias holds bias_ncols values of bias_dtype for
 * columns [bias_col0, bias_col0 + bias_ncols) of C, and the other columns get none; output tiles that
 * do not meet those columns skip the bias entirely. bias_round = 1 rounds each bias value to C's
 * 16-bit type (which must be `dtype`) before the fp32 add: the cast autocast applies to a linear's
 * bias. The bias needs only the alignment of its element type (it may be NULL when bias_ncols = 0).
 * This is the fused projection's F.linear(x, W_cat, b_cat) (src/sisa/modeling.py:213-222,
 * fused_prep.py:99-122), where b_cat is zero except the H alpha columns: the alpha bias is passed as it
 * is stored instead of a full b_cat. */
int sisa_gemm_bias_cols(const void* a, int64_t lda, int a_mn, const void* b, int64_t ldb, int b_mn, void* c,
                        int64_t ldc, int64_t M, int64_t N, int64_t K, int dtype, int out_dtype, int accumulate,
                        const void* bias, int bias_dtype, int64_t bias_col0, int64_t bias_ncols, int bias_round,
                        void* workspace, int64_t workspace_bytes, int32_t* status, void* stream);

/* The SwiGLU MLP's gate and up projections with the activation in the epilogue (src/sisa/modeling.py:39-49:
 * w_gate x, w_up x and silu(.) * (.), which the reference runs as two GEMMs and two elementwise kernels).
 * w (2 d_ff, K): the gate and up weights interleaved in blocks of 8 rows (gate rows 8b .. 8b + 7, then
 * up rows 8b .. 8b + 7, b = 0 .. d_ff / 8 - 1), K-major like x (rows, K), both in `dtype`. Outputs:
 * gu (rows, 2 d_ff), the projections in the same interleaved column order rounded to `dtype` (what the
 * backward reads), and a (rows, d_ff) = silu(g) * u computed in fp32 from the rounded g, u with one
 * rounding (sisa_swiglu_fwd's arithmetic). d_ff a multiple of 8; 16-byte aligned rows. gu NULL: only a
 * is stored (inference, where nothing reads the projections again). */
int sisa_gemm_swiglu(const void* x, int64_t x_ld, const void* w, int64_t w_ld, void* gu, int64_t gu_ld, void* a,
                     int64_t a_ld, int64_t rows, int64_t d_ff, int64_t K, int dtype, int32_t* status, void* stream);

/* AdamW with global-norm gradient clipping over flat fp32 buffers: the training step's
 * torch.nn.utils.clip_grad_norm_(params, max_norm) followed by torch.optim.AdamW (the reference's
 * examples/train_minimal.py:253-301; decoupled weight decay, bias-corrected steps), for parameters laid
 * out in one buffer. param, grad, m, v: n fp32 each (n a multiple of 4), 16-byte aligned. segs: nseg
 * device records sorted by start, [start, end) multiples of 4, each with its group's lr and weight
 * decay; elements outside every segment are left alone. step: device float, advanced by 1 (the
 * bias corrections use the new value). partials: npart doubles of workspace (the norm's fixed-order
 * partial sums: deterministic). max_norm <= 0 disables clipping. A non-finite norm sets
 * SISA_ST_NONFINITE. */
typedef struct sisa_adam_seg {
  int64_t start, end;
  float lr, weight_decay;
} sisa_adam_seg;
int sisa_adamw_flat(float* param, const float* grad, float* m, float* v, int64_t n, const sisa_adam_seg* segs,
                    int nseg, float* step, double* partials, int npart, float beta1, float beta2, float eps,
                    float max_norm, int32_t* status, void* stream);

/* The same AdamW with clipping over separate parameter tensors (the training step's own tensors,
 * gradients as autograd hands them over): tensors[k] = {param, grad, offset, n, lr, weight_decay}, param
 * and grad n fp32 values each (16-byte aligned for the fast path; 4-byte aligned, e.g. a gradient in a
 * DDP bucket, is accepted and read element by element); offset (a multiple of 4, increasing with k) is the
 * tensor's first element in the moment buffers m and v (n_state fp32 each, zero-initialised by the
 * caller). tensors is a HOST array of at most 384 entries: it is passed to the kernels by value, so a
 * captured CUDA graph replays it. The norm covers the listed gradients; tensors left out (no gradient)
 * are not updated. Other arguments as for sisa_adamw_flat. */
typedef struct sisa_adam_tensor {
  float* param;
  const float* grad;
  int64_t offset, n;
  float lr, weight_decay;
} sisa_adam_tensor;
int sisa_adamw_tensors(const sisa_adam_tensor* tensors, int ntensors, float* m, float* v, int64_t n_state,
                       float* step, double* partials, int npart, float beta1, float beta2, float eps,
                       float max_norm, int32_t* status, void* stream);

/* Compute-dtype copies of fp32 weights, many at once (the autocast casts of the weights that the
 * reference's linears make on every forward, src/sisa/modeling.py:39-49,213-222): job j copies source
 * rows r = 0 .. rows-1 (cols fp32 values each, row stride src_ld) to destination row
 * (r / block_rows) * dst_block_stride + r % block_rows (row stride dst_ld) in `dtype`, rounding to
 * nearest even; a job with src NULL zero-fills its destination rows. cols a multiple of 8, src and dst
 * 16-byte aligned, src_ld a multiple of 4 and dst_ld of 8, both >= cols, block_rows >= 1.
 * sisa_row_copy_check: checks one job on the host (no CUDA call).
 * sisa_copy_rows: `jobs` holds njobs checked jobs in DEVICE memory (so a captured CUDA graph can replay
 * the launch); max_vectors is the largest rows * cols / 8 among them. */
/* sisa_copy_heads: dst[b, h, t, 0:width] = src[b, h, t, 0:width] for 16-bit elements (bf16 / fp16), b < B,
 * h < H, t < L, with element strides (sb, sh, sl) on each side: the prompt's keys, values and rotated
 * B~ (views of the fused projection / the preparation output) into a decode cache's buffers, as
 * LayerState.append of the reference's generation.py:58-95 does with torch copies. width a multiple of
 * 8, H * width / 8 <= 256, pointers 16-byte aligned and every stride a multiple of 8. */
int sisa_copy_heads(const void* src, int64_t src_sb, int64_t src_sh, int64_t src_sl, void* dst, int64_t dst_sb,
                    int64_t dst_sh, int64_t dst_sl, int64_t B, int64_t H, int64_t L, int64_t width, void* stream);

/* sisa_split_rows: two fp32 matrices out of one buffer that interleaves them in blocks of `block`
 * rows (block 0 of matrix 0, block 0 of matrix 1, block 1 of matrix 0, ...): dst_h[r, :] =
 * src[(r / block) 2 block + h block + r % block, :] for r < rows, h = 0, 1. The gate and up weight
 * gradients out of the one dW GEMM over their 8-row-interleaved weight (the two weight gradients of
 * src/sisa/modeling.py:39-49). rows a multiple of block, cols a multiple of 4, pointers 16-byte
 * aligned, row strides multiples of 4 and >= cols. */
int sisa_split_rows(const float* src, int64_t src_ld, float* dst0, float* dst1, int64_t dst_ld, int64_t rows,
                    int64_t cols, int64_t block, void* stream);

/* The token embedding's weight gradient (the backward of nn.Embedding in src/sisa/modeling.py, whose
 * weight the tied LM head shares): dw[v, :] = sum of grad[i, :] over the positions i < n with
 * ids[i] = v, summed in increasing i (the same bits on every run; no sort, no atomics), every row of
 * dw written (zero where no id falls). ids outside [0, V) add nothing. Each of the kernel's blocks scans
 * all ids, so n is bounded: n <= SISA_EMBED_MAX_IDS. grad: n rows of D fp32 values, row stride grad_ld;
 * dw: V x D fp32 contiguous. D a multiple of 4, dw and grad 16-byte aligned, grad_ld a multiple of 4. */
#define SISA_EMBED_MAX_IDS 262144
int sisa_embedding_bwd(const int64_t* ids, int64_t n, const float* grad, int64_t grad_ld, float* dw, int64_t V,
                       int64_t D, void* stream);

typedef struct sisa_row_copy {
  const float* src;
  void* dst;
  int64_t rows, cols, src_ld, dst_ld;
  int64_t block_rows, dst_block_stride;
} sisa_row_copy;
int sisa_row_copy_check(const sisa_row_copy* job);
int sisa_copy_rows(const sisa_row_copy* jobs, int njobs, int64_t max_vectors, int dtype, int32_t* status,
                   void* stream);

/* Fused RMSNorm and SwiGLU activation of the model's blocks (src/sisa/modeling.py:25-49). Element
 * types SISA_BF16, SISA_F16 or SISA_F32; row strides (x_ld ...) in elements, unit inner stride.
 * sisa_rmsnorm_fwd: rstd[r] = rsqrt(mean_c x[r,c]^2 + eps), y = (x * rstd) * w, fp32 arithmetic,
 *   one rounding to y's type. w (d,) fp32.
 * sisa_rmsnorm_bwd: dx = rstd (g - xh mean(g xh)) with xh = x rstd, g = dy w; when dw is not null also
 *   dw = sum over rows of dy xh (fp32, fixed reduction order; needs sisa_rmsnorm_bwd_workspace bytes).
 * sisa_swiglu_fwd: a = silu(g) u; sisa_swiglu_bwd: dg = da u silu'(g), du = da silu(g) (fp32
 *   arithmetic, one rounding). rows * ceil(f / 8) < 2^31.
 * These wait on nothing; status may be null. */
int64_t sisa_rmsnorm_bwd_workspace(int64_t rows, int64_t d);
int sisa_rmsnorm_fwd(const void* x, int64_t x_ld, int x_dtype, const float* w, int64_t rows, int64_t d, float eps,
                     void* y, int64_t y_ld, int y_dtype, float* rstd, int32_t* status, void* stream);
int sisa_rmsnorm_bwd(const void* dy, int64_t dy_ld, int dy_dtype, const void* x, int64_t x_ld, int x_dtype,
                     const float* w, const float* rstd, int64_t rows, int64_t d, void* dx, int64_t dx_ld, int dx_dtype,
                     float* dw, void* workspace, int32_t* status, void* stream);

/* RMSNorm at a block boundary with the work eager PyTorch runs around it as separate kernels
 * (src/sisa/modeling.py:275-276 with :25-36, :167-168 and the autocast casts before the linears):
 *   v = x + res (res optional; rounded to x's type, as the reference's residual add; written to xsum),
 *   rstd = rsqrt(mean(v^2) + eps), h = (v rstd) w rounded to x's type (the reference's RMSNorm output),
 *   y[k] = h in y_dtype[k] for k < n_out (n_out 1 or 2: one copy per consumer, so that each consumer's
 *   gradient arrives separately and is summed in fp32 as the reference sums them),
 *   proj_out = h proj_w^T + proj_b in fp32 when n_proj > 0 (the attention's forget projection;
 *   proj_w (n_proj, d) and proj_b (n_proj,) fp32, n_proj <= 32, n_proj * d * 4 <= 200 KB).
 * Backward: G = sum_k dy[k] (null entries skipped) + dproj_out proj_w; dv = rstd (G w - xh mean(G w xh))
 *   + dv_in (the gradient v gets from its other consumers; may be null), with xh = v rstd; dv is
 *   stored as dx and, when dres is not null, also in dres's type (the residual's gradient); and, each
 *   when not null, dweight = sum_r G xh, dproj_w = sum_r dproj_out^T h, dproj_b = sum_r dproj_out, from
 *   per-row-split partial sums in a fixed order (deterministic; sisa_norm_bwd_workspace bytes). */
typedef struct sisa_norm_fwd_args {
  const void* x; int64_t x_ld; int x_dtype;
  const void* res; int64_t res_ld; int res_dtype;
  void* xsum; int64_t xsum_ld;
  const float* weight;
  int64_t rows, d;
  float eps;
  int n_out;
  void* y[2]; int64_t y_ld[2]; int y_dtype[2];
  float* rstd;
  const float* proj_w; const float* proj_b; int64_t n_proj; float* proj_out;
} sisa_norm_fwd_args;

typedef struct sisa_norm_bwd_args {
  const void* v; int64_t v_ld; int v_dtype;     /* the normalised rows: x, or xsum with a residual add */
  const float* weight; const float* rstd;
  int64_t rows, d;
  const void* dy[2]; int64_t dy_ld[2]; int dy_dtype[2];
  const void* dv_in; int64_t dv_in_ld; int dv_in_dtype;
  const float* proj_w; int64_t n_proj; const float* dproj_out;
  void* dx; int64_t dx_ld; int dx_dtype;
  void* dres; int64_t dres_ld; int dres_dtype;
  float* dweight; float* dproj_w; float* dproj_b;
  void* workspace;
} sisa_norm_bwd_args;

int64_t sisa_norm_bwd_workspace(int64_t rows, int64_t d, int64_t n_proj);
int sisa_norm_fwd(const sisa_norm_fwd_args* args, int32_t* status, void* stream);
int sisa_norm_bwd(const sisa_norm_bwd_args* args, int32_t* status, void* stream);
int sisa_swiglu_fwd(const void* g, int64_t g_ld, const void* u, int64_t u_ld, int64_t rows, int64_t f, int dtype,
                    void* a, int64_t a_ld, int32_t* status, void* stream);
int sisa_swiglu_bwd(const void* da, int64_t da_ld, const void* g, int64_t g_ld, const void* u, int64_t u_ld,
                    int64_t rows, int64_t f, int dtype, void* dg, int64_t dg_ld, void* du, int64_t du_ld,
                    int32_t* status, void* stream);

/* Incremental decode: one new query row per (batch, head) against N cached keys
 * (src/sisa/modeling.py:224-238 via src/sisa/functional.py:69-103, src/sisa/generation.py:58-95):
 *   s_j = q.k_j/8 + lam_h exp(min(g_q - g_j, 0)) (c.b_j) + (F_q - F_j), y = softmax(s) v, in fp32.
 * q: (B, H, 1, 64) and c: (B, H, 1, 32) views in `dtype`; g_q, f_q: (B, H) fp32 contiguous (f_q may be
 * NULL, then f_cache must be NULL too). k_cache, v_cache: (B, H, >=N, 64) and b_cache: (B, H, >=N, 32) views;
 * g_cache, f_cache: fp32 with element (b, h, j) at (b*H + h)*gf_stride + j. y: (B, H, 1, 64) view.
 * workspace: sisa_decode_workspace(B, H, N) bytes (split-K partials). */
int64_t sisa_decode_workspace(int64_t B, int64_t H, int64_t N);
int sisa_decode_attn(const sisa_view4* q, const sisa_view4* c, const float* g_q, const float* f_q,
                     const sisa_view4* k_cache, const sisa_view4* v_cache, const sisa_view4* b_cache,
                     const float* g_cache, const float* f_cache, int64_t gf_stride, const float* lam,
                     int64_t B, int64_t H, int64_t N, int dtype, const sisa_view4* y, void* workspace,
                     int32_t* status, void* stream);

/* Allocation-free variant of sisa_decode_attn (no counterpart in the reference): identical arguments
 * except that there is no workspace. For callers that cannot allocate device memory when they decode:
 * host programs that bind only this C ABI and have no device allocator, and serving loops held to a
 * fixed, pre-reserved memory budget. The split-K partials live in a fixed 4.3 MB array owned by the
 * library on every GPU that loads it; B*H may not exceed 16384 (SISA_ERR_VALUE otherwise). The first
 * call on a device looks up the array's address (cudaGetSymbolAddress, with that device current) and
 * keeps it; a cudaDeviceReset makes that address stale. Calls that overlap on the GPU share the array
 * and race. The caller's current device is unchanged on return. */
int sisa_decode_attn_noalloc(const sisa_view4* q, const sisa_view4* c, const float* g_q, const float* f_q,
                             const sisa_view4* k_cache, const sisa_view4* v_cache, const sisa_view4* b_cache,
                             const float* g_cache, const float* f_cache, int64_t gf_stride, const float* lam,
                             int64_t B, int64_t H, int64_t N, int dtype, const sisa_view4* y,
                             int32_t* status, void* stream);

/* One decode step's layer input from the fused projection row of the new token (the single-token case
 * of src/sisa/modeling.py:171-199 with the recurrences continued from the cache, generation.py:58-95):
 * per (batch b, head h), with proj the (B, NPAD) row in `dtype` (columns as sisa_fused_layout) and z the
 * (B, H) fp32 forget logits (z_sb row stride; may be null together with f_cache and f_out):
 *   g = g_cache[pos-1] - softplus(alpha), F = f_cache[pos-1] + logsigmoid(z), Phi = phi + theta (16 pairs),
 *   c~ = R(Phi) c, b~ = R(Phi) b (fp32, torch's separate products, one rounding).
 * Writes k, v, b~ into the caches at position pos, g and F into g_cache/f_cache[pos] and g_out/f_out
 * (B, H), c~ into c_out (B, H, 32) contiguous, and advances phi (B, H, 16) fp32 contiguous in place.
 * 1 <= pos < gf_stride; the caches are (B, H, >pos, 64 or 32) views with even element strides. q is the
 * Q columns of proj, passed to sisa_decode_attn as a view. */
int sisa_decode_prep(const void* proj, int64_t proj_sb, const float* z, int64_t z_sb, int64_t B, int64_t H,
                     int dtype, const sisa_view4* k_cache, const sisa_view4* v_cache, const sisa_view4* b_cache,
                     float* g_cache, float* f_cache, int64_t gf_stride, int64_t pos, float* phi, void* c_out,
                     float* g_out, float* f_out, int32_t* status, void* stream);

/* Device-position forms of sisa_decode_prep and sisa_decode_attn, for a decode step that is captured
 * once as a CUDA graph and replayed for every new token. The reference runs the same step eagerly from
 * its generate() loop (src/sisa/generation.py:177-189 calling modeling.py:224-238); its per-token host
 * work is what the graph removes. The arguments are those of the host-position forms, except:
 *   sisa_decode_prep_dpos: the position is *d_pos (int32 in device memory, read when the kernel runs);
 *     max_pos (2 <= max_pos <= gf_stride, at most the caches' position count) bounds it: a position
 *     outside [1, max_pos) sets SISA_ST_BAD_POS and writes nothing.
 *   sisa_decode_attn_dpos: attends over N = *d_pos + 1 cached keys; max_n bounds N (a position outside
 *     [1, max_n) sets SISA_ST_BAD_POS and y is zero) and sizes the split count and the workspace,
 *     sisa_decode_workspace(B, H, max_n) bytes.
 * The caller advances *d_pos between steps (inside the graph). */
int sisa_decode_prep_dpos(const void* proj, int64_t proj_sb, const float* z, int64_t z_sb, int64_t B, int64_t H,
                          int dtype, const sisa_view4* k_cache, const sisa_view4* v_cache, const sisa_view4* b_cache,
                          float* g_cache, float* f_cache, int64_t gf_stride, const int32_t* d_pos, int64_t max_pos,
                          float* phi, void* c_out, float* g_out, float* f_out, int32_t* status, void* stream);
int sisa_decode_attn_dpos(const sisa_view4* q, const sisa_view4* c, const float* g_q, const float* f_q,
                          const sisa_view4* k_cache, const sisa_view4* v_cache, const sisa_view4* b_cache,
                          const float* g_cache, const float* f_cache, int64_t gf_stride, const float* lam,
                          int64_t B, int64_t H, const int32_t* d_pos, int64_t max_n, int dtype, const sisa_view4* y,
                          void* workspace, int32_t* status, void* stream);

/* Diagnostic: one block runs the library's bounded-wait handshake (a producer warp, consumer warps
 * waiting on an mbarrier, a tensor-memory allocation freed at the end) with the wait limit limit_ns
 * (1e3..1e9 ns) in place of the library's 2 s. With producer_arrives = 0 nothing ever arrives, so the
 * consumers' waits run out: SISA_ST_TIMEOUT is OR-ed into *status, *result (device int32) receives the
 * number of consumer warps that gave up (2), and the kernel returns with the context usable. With
 * producer_arrives = 1, *result is 0. The reference asserts on the device instead
 * (src/sisa/kernels/fused_prep.py:502-523 via torch._assert_async), which ends the CUDA context. */
int sisa_selftest_wait(int producer_arrives, int64_t limit_ns, int32_t* status, int32_t* result, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SISA_B200_H */
