"""Fused SISA layer core on the sm_100a kernels (mirrors src/sisa/kernels/fused_prep.py of tlstngud/sisa).

``sisa_fused(proj, z, lam, n_head) -> y``: the preparation kernel (g, F, Phi scans and the rotation of
C/B) plus the tcgen05 attention forward; backward runs the exact-delta attention backward, whose dq,
dk, dv land directly in the Q/K/V columns of d_proj, then the reverse-scan kernel that fills the B, C,
theta, alpha and padding columns of d_proj and dz.
"""
from __future__ import annotations

import torch

from .gemm import matmul_t
from .. import ops

__all__ = ["sisa_fused", "fused_layout", "concat_fused_weights", "fused_projection", "prefill_layer"]

D_HEAD = 64
D_STATE = 32


def fused_layout(n_head: int, d_head: int = D_HEAD, d_state: int = D_STATE) -> dict:
    """Column offsets of the fused projection (src/sisa/kernels/fused_prep.py:71-96):
    ``[Q H*64 | K H*64 | V H*64 | B H*32 | C H*32 | TH H*16 | A H | zero padding to a multiple of 16]``."""
    if d_head != D_HEAD or d_state != D_STATE:
        raise ValueError(f"the fused kernels support d_head={D_HEAD} and d_state={D_STATE} only")
    return ops.fused_layout(n_head)


def concat_fused_weights(W_Q, W_K, W_V, W_B, W_C, W_theta, W_alpha, b_alpha):
    """``(W_cat, b_cat)`` with ``proj = F.linear(x, W_cat, b_cat)`` (src/sisa/kernels/fused_prep.py:99-122).
    Padding rows and every bias entry except the alpha columns are zero; differentiable."""
    H = W_alpha.shape[0]
    off = fused_layout(H)
    pad = off["NPAD"] - off["NTOT"]
    d = W_Q.shape[1]
    ws = [W_Q, W_K, W_V, W_B, W_C, W_theta, W_alpha]
    bs = [torch.zeros(off["A"], device=b_alpha.device, dtype=b_alpha.dtype), b_alpha]
    if pad:
        ws.append(torch.zeros(pad, d, device=W_Q.device, dtype=W_Q.dtype))
        bs.append(torch.zeros(pad, device=b_alpha.device, dtype=b_alpha.dtype))
    W = torch.cat(ws, 0)
    if W.shape[0] != off["NPAD"]:
        raise ValueError(f"concatenated weight has {W.shape[0]} rows, expected {off['NPAD']} for n_head={H}")
    return W, torch.cat(bs, 0)


def take_fresh(owner, slot: str, key: tuple, train: bool):
    """The compute-dtype weight copy kept on ``owner`` under ``slot`` if it may be used now, else None.
    Entries are ``(key, tensor, fresh)``. Outside training the key decides. In a training forward
    (``train``: gradients enabled where the linear was called) the copy must also be fresh, i.e. written
    by the model's refresh for this forward; the mark is taken with the use."""
    hit = owner.__dict__.get(slot)
    if hit is None or hit[0] != key:
        return None
    if hit[2]:
        owner.__dict__[slot] = (hit[0], hit[1], False)
        return hit[1]
    return None if train else hit[1]


def wcat_key(weights, dtype) -> tuple:
    """The key under which the compute-dtype concatenation of ``weights`` is kept (``_wcat_train``)."""
    return (dtype,) + tuple((w.data_ptr(), w._version, w.dtype) for w in weights)


def _cached_wcat(owner, weights, dtype, train: bool = False) -> torch.Tensor:
    """The concatenation of ``weights`` (plus zero padding rows to NPAD) in ``dtype``, kept on ``owner``;
    it never enters the autograd graph. Outside training it is reused while every weight keeps its
    storage, version and dtype. In a training forward only a copy that the model's one-launch refresh
    has just written is used (kernels/weights.py), else it is rebuilt: fused optimizers update the
    weights without advancing their versions."""
    key = wcat_key(weights, dtype)
    hit = take_fresh(owner, "_wcat_train", key, train)
    if hit is not None:
        return hit
    H = weights[-1].shape[0]
    off = fused_layout(H)
    d = weights[0].shape[1]
    wc = torch.empty((off["NPAD"], d), dtype=dtype, device=weights[0].device)
    row = 0
    with torch.no_grad():
        for w in weights:
            wc[row:row + w.shape[0]].copy_(w)
            row += w.shape[0]
        wc[row:].zero_()
    owner.__dict__["_wcat_train"] = (key, wc, False)
    return wc


_ONES: dict[tuple, torch.Tensor] = {}


def _ones_row(n: int, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """A (1, n) row of ones, kept per (n, dtype, device) (the training shapes repeat)."""
    key = (n, dtype, device)
    t = _ONES.get(key)
    if t is None:
        if len(_ONES) >= 64:
            _ONES.clear()
        t = _ONES[key] = torch.ones((1, n), dtype=dtype, device=device)
    return t


class _FusedProjFn(torch.autograd.Function):
    """``proj = x W_cat^T + b_cat`` in the compute dtype from the seven projection weights, ``b_cat`` zero
    except the alpha columns: the call ``F.linear`` makes under autocast (inputs in the compute dtype, bias
    added in the GEMM epilogue before the one rounding), here on the CTA-pair tcgen05 GEMM with its bias
    epilogue. ``W_cat`` comes from :func:`_cached_wcat` instead of a differentiable ``torch.cat``; the
    backward runs the two plain linear-backward GEMMs (cuBLAS) once for the concatenation, dW with an
    fp32 output, hands each weight its rows of dW as a view, and reduces only the H alpha columns for
    the bias gradient."""

    @staticmethod
    def forward(ctx, x, b_alpha, owner, dtype, train, *weights):
        H = b_alpha.shape[0]
        col_a = fused_layout(H)["A"]
        xc = x.to(dtype)
        wc = _cached_wcat(owner, weights, dtype, train)
        d = xc.shape[-1]
        x2 = xc.reshape(-1, d)
        out = torch.empty((x2.shape[0], wc.shape[0]), dtype=dtype, device=x.device)
        if x2.shape[0]:
            # b_cat is zero outside the alpha columns: the alpha bias goes to the GEMM as stored, rounded
            # to the compute dtype in the epilogue (autocast's cast of the bias)
            matmul_t(x2 if x2.stride(-1) == 1 else x2.contiguous(), wc, out, bias=b_alpha.contiguous(),
                     bias_col0=col_a, bias_round=True)
        out = out.view(*xc.shape[:-1], wc.shape[0])
        ctx.save_for_backward(xc, wc)
        ctx.col_a, ctx.H = col_a, H
        ctx.rows = [w.shape[0] for w in weights]
        ctx.dtypes = (x.dtype, b_alpha.dtype, [w.dtype for w in weights])
        return out

    @staticmethod
    def backward(ctx, g):
        xc, wc = ctx.saved_tensors
        g2 = g.reshape(-1, g.shape[-1])
        dx = db = None
        if ctx.needs_input_grad[0]:
            dx = (g2 @ wc).view(xc.shape).to(ctx.dtypes[0])
        if ctx.needs_input_grad[1]:
            # the alpha columns' sum over rows as a GEMV against a row of ones (fp32 accumulation, the
            # result in the gradient's dtype like the sum autograd takes): torch's reduction of this
            # strided 12-column slice took 13 us per layer
            ones = _ones_row(g2.shape[0], g2.dtype, g2.device)
            db = torch.mm(ones, g2[:, ctx.col_a:ctx.col_a + ctx.H]).view(ctx.H).to(ctx.dtypes[1])
        dws = [None] * len(ctx.rows)
        if any(ctx.needs_input_grad[5:]):
            # dW in fp32 straight from the GEMM: each fp32 weight takes its rows as a view, no casts
            dw = torch.mm(g2.t(), xc.reshape(-1, xc.shape[-1]), out_dtype=torch.float32)
            row = 0
            for i, (n, dt) in enumerate(zip(ctx.rows, ctx.dtypes[2])):
                if ctx.needs_input_grad[5 + i]:
                    dws[i] = dw[row:row + n].to(dt)
                row += n
        return (dx, db, None, None, None, *dws)


def fused_projection(x: torch.Tensor, weights, b_alpha: torch.Tensor, dtype: torch.dtype, owner) -> torch.Tensor:
    """``F.linear(x, W_cat, b_cat)`` under autocast to ``dtype`` (fused_prep.py:99-122) from the projection
    weights ``[W_Q, W_K, W_V, W_B, W_C, W_theta, W_alpha]`` and the alpha bias. The compute-dtype
    concatenation is kept on ``owner`` (see :func:`_cached_wcat`)."""
    return _FusedProjFn.apply(x, b_alpha, owner, dtype, torch.is_grad_enabled(), *weights)


def prep_forward(proj: torch.Tensor, z: torch.Tensor | None, H: int):
    """Run the preparation kernels: returns (c_rot, b_rot, pos, tot)."""
    return ops.prep_fwd(proj, z, H)


class _SISAFusedFn(torch.autograd.Function):
    """The layer core on the ``sisa_b200`` operators: forward = prep_fwd + attn_fwd, backward = fused_bwd."""

    @staticmethod
    def forward(ctx, proj, z, lam, H):
        B, L, _ = proj.shape
        off = fused_layout(H)
        c_rot, b_rot, pos, tot = ops.prep_fwd(proj, z, H)
        q, k, v = ops.heads(proj, off["Q"], H, 64), ops.heads(proj, off["K"], H, 64), ops.heads(proj, off["V"], H, 64)
        o, lse, o32 = ops.attn_fwd(q, k, v, c_rot, b_rot, pos, lam, any(ctx.needs_input_grad))
        ctx.save_for_backward(proj, z, lam, c_rot, b_rot, pos, tot, o, lse, o32)
        ctx.H = H
        return o.transpose(1, 2).reshape(B, L, H * D_HEAD)

    @staticmethod
    def backward(ctx, dy):
        proj, z, lam, c_rot, b_rot, pos, tot, o, lse, o32 = ctx.saved_tensors
        dproj, dz, dlam = ops.fused_bwd(proj, z, lam, c_rot, b_rot, pos, tot, o, lse, o32, dy, ctx.H)
        return dproj, (dz if z is not None else None), dlam, None


def prefill_layer(proj: torch.Tensor, z: torch.Tensor, lam: torch.Tensor, n_head: int):
    """The layer core over a whole prompt without autograd, keeping what a decode cache needs: the
    preparation kernel and the tcgen05 forward (no o'' - nothing will run a backward), on the fused
    projection ``proj`` (B, L, NPAD) and forget logits ``z`` (B, L, H) fp32.

    The reference fills its cache through the unfused path instead (src/sisa/modeling.py:226-232: seven
    projections, torch recurrences and rotations). Returns ``y`` (B, L, H*64) and the cache entries:
    k, v (views of proj's K/V columns), b~ (B, H, L, 32) as the kernels rotated it, g and F (views of the
    position planes) and Phi at the last position (B, H, 16) fp32."""
    H = int(n_head)
    B, L, _ = proj.shape
    off = fused_layout(H)
    c_rot, b_rot, pos, _ = ops.prep_fwd(proj, z, H)
    q, k, v = ops.heads(proj, off["Q"], H, 64), ops.heads(proj, off["K"], H, 64), ops.heads(proj, off["V"], H, 64)
    o, _, _ = ops.attn_fwd(q, k, v, c_rot, b_rot, pos, lam, False)
    theta = proj[..., off["TH"]:off["TH"] + H * (D_STATE // 2)]
    phi_last = theta.float().sum(dim=1).view(B, H, D_STATE // 2)
    y = o.transpose(1, 2).reshape(B, L, H * D_HEAD)
    return y, (k, v, b_rot, pos[:, :, 0, :L], pos[:, :, 1, :L], phi_last)


def sisa_fused(proj: torch.Tensor, z: torch.Tensor | None, lam: torch.Tensor, n_head: int) -> torch.Tensor:
    """Fused SISA layer core (src/sisa/kernels/fused_prep.py:637-683).

    Args:
        proj: ``(B, L, NPAD)`` bf16/fp16 output of ``F.linear(x_norm, W_cat, b_cat)`` (fused_layout columns),
            ``stride(-1) == 1`` and ``stride(1) == NPAD``.
        z: ``(B, L, H)`` fp32 forget-gate logits (``stride(2) == 1``) or None.
        lam: ``(H,)`` fp32 ``softplus(lambda_raw)``.
        n_head: number of heads (d_head 64, d_state 32).

    Returns ``y`` ``(B, L, H*64)`` in ``proj.dtype``; differentiable w.r.t. proj, z and lam. The gradient
    of the padding columns is exactly zero.
    """
    H = int(n_head)
    if proj.dim() != 3:
        raise ValueError(f"proj must be (B, L, NPAD), got shape {tuple(proj.shape)}")
    off = fused_layout(H)
    B, L, NP = proj.shape
    if NP != off["NPAD"]:
        raise ValueError(f"proj has {NP} columns, expected NPAD={off['NPAD']} for n_head={H}")
    if proj.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"proj must be bf16 or fp16, got {proj.dtype}")
    if not proj.is_cuda:
        raise ValueError("proj must be a CUDA tensor")
    if L < 1:
        raise ValueError("sequence length must be >= 1")
    if proj.stride(-1) != 1 or proj.stride(1) != NP or proj.stride(0) % 8 or ops.base_misaligned(proj):
        proj = proj.contiguous()
    if z is not None:
        if z.shape != (B, L, H):
            raise ValueError(f"z must have shape {(B, L, H)}, got {tuple(z.shape)}")
        if z.dtype != torch.float32:
            raise TypeError(f"z must be fp32, got {z.dtype}")
        if z.stride(2) != 1:
            z = z.contiguous()
    if lam.shape != (H,):
        raise ValueError(f"lam must have shape {(H,)}, got {tuple(lam.shape)}")
    lam = lam.float().contiguous()
    return _SISAFusedFn.apply(proj, z, lam, H)

