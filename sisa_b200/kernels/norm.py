"""Fused RMSNorm and SwiGLU activation for the model's blocks (reference: src/sisa/modeling.py:26-49).

``rms_norm(x, weight, eps)`` computes ``((x.float() * rsqrt(mean(x.float()^2) + eps)) * weight.float())
.to(x.dtype)`` in one sm_100a kernel (the eager form is six), and its backward in two (dx per row, dw
from fixed-order partial sums, deterministic). ``swiglu(g, u)`` computes ``silu(g) * u`` and its
backward in one kernel each, in fp32 with one rounding. Both raise if the CUDA library is missing;
the callers choose them only for CUDA tensors on the ``cuda`` path.
"""
from __future__ import annotations

import torch

from .. import _lib

F32 = 2


def _code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return F32
    return _lib.dtype_code(dt)


def _rows(x: torch.Tensor) -> torch.Tensor:
    """(rows, d) view with unit inner stride (copies only if the layout needs it)."""
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    return x2


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        lib = _lib.load()
        x2 = _rows(x)
        rows, d = x2.shape
        w = weight.float().contiguous()
        y = torch.empty((rows, d), dtype=x.dtype, device=x.device)
        rstd = torch.empty((rows,), dtype=torch.float32, device=x.device)
        rc = lib.sisa_rmsnorm_fwd(x2.data_ptr(), x2.stride(0), _code(x.dtype), w.data_ptr(), rows, d, float(eps),
                                  y.data_ptr(), d, _code(y.dtype), rstd.data_ptr(), None, _lib.stream_ptr(x.device))
        _lib.check(rc, "sisa_rmsnorm_fwd")
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape, ctx.wdtype = x.shape, weight.dtype
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        lib = _lib.load()
        x2, w, rstd = ctx.saved_tensors
        rows, d = x2.shape
        dy2 = _rows(dy)
        dx = torch.empty((rows, d), dtype=x2.dtype, device=x2.device)
        need_w = ctx.needs_input_grad[1]
        dw = torch.empty((d,), dtype=torch.float32, device=x2.device) if need_w else None
        ws = (torch.empty((lib.sisa_rmsnorm_bwd_workspace(rows, d),), dtype=torch.uint8, device=x2.device)
              if need_w else None)
        rc = lib.sisa_rmsnorm_bwd(dy2.data_ptr(), dy2.stride(0), _code(dy2.dtype), x2.data_ptr(), x2.stride(0),
                                  _code(x2.dtype), w.data_ptr(), rstd.data_ptr(), rows, d, dx.data_ptr(), d,
                                  _code(dx.dtype), dw.data_ptr() if need_w else None,
                                  ws.data_ptr() if need_w else None, None, _lib.stream_ptr(x2.device))
        _lib.check(rc, "sisa_rmsnorm_bwd")
        return dx.view(ctx.shape), (dw.to(ctx.wdtype) if need_w else None), None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm of the last axis in fp32, output in x's dtype (modeling.py:26-36), on the sm_100a kernels."""
    return _RMSNormFn.apply(x, weight, eps)


class _SwiGLUFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, g, u):
        lib = _lib.load()
        g2, u2 = _rows(g), _rows(u)
        rows, f = g2.shape
        a = torch.empty((rows, f), dtype=g.dtype, device=g.device)
        rc = lib.sisa_swiglu_fwd(g2.data_ptr(), g2.stride(0), u2.data_ptr(), u2.stride(0), rows, f, _code(g.dtype),
                                 a.data_ptr(), f, None, _lib.stream_ptr(g.device))
        _lib.check(rc, "sisa_swiglu_fwd")
        ctx.save_for_backward(g2, u2)
        ctx.shape = g.shape
        return a.view(g.shape)

    @staticmethod
    def backward(ctx, da):
        lib = _lib.load()
        g2, u2 = ctx.saved_tensors
        rows, f = g2.shape
        da2 = _rows(da.to(g2.dtype))
        dg = torch.empty_like(g2)
        du = torch.empty_like(u2)
        rc = lib.sisa_swiglu_bwd(da2.data_ptr(), da2.stride(0), g2.data_ptr(), g2.stride(0), u2.data_ptr(),
                                 u2.stride(0), rows, f, _code(g2.dtype), dg.data_ptr(), f, du.data_ptr(), f, None,
                                 _lib.stream_ptr(g2.device))
        _lib.check(rc, "sisa_swiglu_bwd")
        return dg.view(ctx.shape), du.view(ctx.shape)


def swiglu(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """silu(g) * u (g, u of one dtype and shape), on the sm_100a kernels."""
    if g.shape != u.shape or g.dtype != u.dtype:
        raise ValueError(f"swiglu: g {tuple(g.shape)} {g.dtype} and u {tuple(u.shape)} {u.dtype} must match")
    return _SwiGLUFn.apply(g, u)
