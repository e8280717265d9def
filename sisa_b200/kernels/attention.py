"""Exact SISA attention on the sm_100a kernels, standalone form (mirrors src/sisa/kernels/attention.py:788-877).

``sisa_attention_cuda(q, k, v, c, b, g, lam, fgate=None) -> o`` with
``s_ij = q_i.k_j/8 + lam_h exp(g_i - g_j)(c_i.b_j) + (fgate_i - fgate_j)``, j <= i. The position
records {g, F, rowf, colf} are packed (and g's monotonicity checked) by one small kernel, then the
tcgen05 forward runs; backward is the exact-delta two-kernel backward. Deterministic.
"""
from __future__ import annotations

import torch

from .. import ops

__all__ = ["sisa_attention_cuda"]

D_HEAD = 64
D_STATE = 32


def _aligned(t: torch.Tensor) -> torch.Tensor:
    """A view the kernels can take: contiguous last axis, 16-byte rows and strides."""
    unit = 16 // t.element_size()
    if t.stride(-1) != 1 or ops.base_misaligned(t) or any(s % unit for s in t.stride()[:-1]):
        return t.contiguous()
    return t


def pack_positions(g: torch.Tensor, fgate: torch.Tensor | None) -> torch.Tensor:
    return ops.pack_positions(g, fgate)


class _SISAAttentionFn(torch.autograd.Function):
    """Unfused attention on the ``sisa_b200`` operators: pack_positions + attn_fwd, backward attn_bwd."""

    @staticmethod
    def forward(ctx, q, k, v, c, b, g, lam, fgate):
        pos = ops.pack_positions(g, fgate)
        o, lse, o32 = ops.attn_fwd(q, k, v, c, b, pos, lam, any(ctx.needs_input_grad))
        ctx.save_for_backward(q, k, v, c, b, pos, lam, o, lse, o32)
        ctx.has_f = fgate is not None
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, c, b, pos, lam, o, lse, o32 = ctx.saved_tensors
        do = _aligned(do.to(q.dtype))
        dq, dk, dv, dc, db, dg, dlam, dF = ops.attn_bwd(q, k, v, c, b, pos, lam, o, do, lse, o32, ctx.has_f)
        return dq, dk, dv, dc, db, dg, dlam, (dF if ctx.has_f else None)


def _prepare_inputs(q, k, v, c, b, g, lam, fgate):
    """Validation with the reference's exception types (src/sisa/kernels/attention.py:812-850)."""
    if q.dim() != 4 or q.shape[-1] != D_HEAD or c.dim() != 4 or c.shape[-1] != D_STATE:
        raise ValueError(f"the cuda kernels support d_head=64 and d_state=32 only; got q {tuple(q.shape)}, "
                         f"c {tuple(c.shape)}")
    if q.dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"q must be bf16 or fp16 for the cuda kernels, got {q.dtype}")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError(f"q/k/v dtypes differ: {q.dtype}, {k.dtype}, {v.dtype}")
    tensors = [q, k, v, c, b, g, lam] + ([fgate] if fgate is not None else [])
    if not (q.is_cuda and all(t.device == q.device for t in tensors)):
        raise ValueError("all inputs must be on the same CUDA device")
    B, H, L, _ = q.shape
    if L < 1:
        raise ValueError("sequence length must be >= 1")
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f"k/v shapes {tuple(k.shape)}/{tuple(v.shape)} != q shape {tuple(q.shape)}")
    if c.shape != (B, H, L, D_STATE) or b.shape != (B, H, L, D_STATE):
        raise ValueError(f"c/b must have shape {(B, H, L, D_STATE)}, got {tuple(c.shape)}/{tuple(b.shape)}")
    if g.dtype != torch.float32:
        raise TypeError(f"g must be fp32, got {g.dtype}")
    if g.shape != (B, H, L):
        raise ValueError(f"g must have shape {(B, H, L)}, got {tuple(g.shape)}")
    if fgate is not None:
        if fgate.dtype != torch.float32:
            raise TypeError(f"fgate must be fp32, got {fgate.dtype}")
        if fgate.shape != g.shape:
            raise ValueError(f"fgate shape {tuple(fgate.shape)} != g shape {tuple(g.shape)}")
    if lam.shape != (H,):
        raise ValueError(f"lam must have shape {(H,)}, got {tuple(lam.shape)}")
    lam = lam.float().contiguous()
    if c.dtype != q.dtype:
        c = c.to(q.dtype)
    if b.dtype != q.dtype:
        b = b.to(q.dtype)
    q, k, v, c, b = (_aligned(t) for t in (q, k, v, c, b))
    return q, k, v, c, b, g, lam, fgate


def sisa_attention_cuda(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, c: torch.Tensor, b: torch.Tensor,
                        g: torch.Tensor, lam: torch.Tensor, fgate: torch.Tensor | None = None) -> torch.Tensor:
    """Exact SISA attention on the sm_100a kernels, differentiable w.r.t. every tensor argument.

    Args:
        q, k, v: ``(B, H, L, 64)`` bf16 or fp16, any strides with a contiguous last axis.
        c, b: ``(B, H, L, 32)`` rotated SSM read/write vectors (cast to q.dtype; the gradient flows back in
            their own dtype).
        g: ``(B, H, L)`` fp32 cumulative log-decay, non-increasing (checked per the check mode).
        lam: ``(H,)`` fp32. fgate: ``(B, H, L)`` fp32 cumulative log forget gate, or None.

    Returns ``(B, H, L, 64)`` in q.dtype stored in ``(B, L, H, 64)`` memory (``o.transpose(1, 2).reshape``
    is a view).
    """
    q, k, v, c, b, g, lam, fgate = _prepare_inputs(q, k, v, c, b, g, lam, fgate)
    return _SISAAttentionFn.apply(q, k, v, c, b, g, lam, fgate)
