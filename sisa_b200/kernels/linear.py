"""``F.linear(x, W)`` under autocast for the model's plain linears (W_O, w_down): the same bf16/fp16
product, with the weight's compute-dtype copy written by the model's one-launch refresh of all its
weight copies (kernels/weights.py) or kept between inference calls while the weight is unchanged, and
the weight gradient computed in fp32 by the GEMM (instead of a low-precision gradient cast to the fp32
parameter's dtype afterwards). The GEMMs are plain library GEMMs (cuBLAS
through ``torch.mm``); nothing is fused into them.
"""
from __future__ import annotations

import torch
from torch import Tensor

__all__ = ["linear_cast", "supports"]


def supports(x: Tensor, weight: Tensor, dtype: torch.dtype) -> bool:
    """CUDA input, a 16-bit compute dtype that differs from the weight's (the autocast case)."""
    return x.is_cuda and dtype in (torch.bfloat16, torch.float16) and weight.dtype != dtype


def weight_key(weight: Tensor, dtype: torch.dtype) -> tuple:
    """The key under which the compute-dtype copy of ``weight`` is kept (``_lp_<name>``)."""
    return (dtype, weight.data_ptr(), weight._version, weight.dtype)


def _cached(owner, name: str, weight: Tensor, dtype: torch.dtype, train: bool = False) -> Tensor:
    """The compute-dtype copy kept on ``owner`` under ``_lp_<name>``, used as ``kernels.fused.take_fresh``
    allows and rebuilt otherwise."""
    from .fused import take_fresh

    key = weight_key(weight, dtype)
    slot = "_lp_" + name
    hit = take_fresh(owner, slot, key, train)
    if hit is None:
        with torch.no_grad():
            hit = weight.to(dtype).contiguous()
        owner.__dict__[slot] = (key, hit, False)
    return hit


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, owner, name, dtype, train):
        w = _cached(owner, name, weight, dtype, train)
        x2 = x.reshape(-1, x.shape[-1]).to(dtype)
        y = torch.mm(x2, w.t())
        ctx.save_for_backward(x2, w)
        ctx.meta = (x.shape, x.dtype, weight.dtype)
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        x_shape, x_dtype, w_dtype = ctx.meta
        dy2 = dy.reshape(-1, dy.shape[-1]).to(w.dtype)
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = torch.mm(dy2, w).view(x_shape).to(x_dtype)
        if ctx.needs_input_grad[1]:
            dw = torch.mm(dy2.t(), x2, out_dtype=torch.float32).to(w_dtype)
        return dx, dw, None, None, None, None


def linear_cast(x: Tensor, weight: Tensor, dtype: torch.dtype, owner, name: str) -> Tensor:
    """``x W^T`` in ``dtype`` (no bias), the weight's ``dtype`` copy kept on ``owner`` under ``name``."""
    with torch.autocast(x.device.type, enabled=False):
        return _LinearFn.apply(x, weight, owner, name, dtype, torch.is_grad_enabled())
