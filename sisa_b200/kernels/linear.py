"""``F.linear(x, W)`` under autocast for the model's plain linears (W_O, w_down): the same bf16/fp16
product, with the weight's compute-dtype copy kept while the weight is unchanged (instead of a cast on
every forward) and the weight gradient computed in fp32 by the GEMM (instead of a low-precision
gradient cast to the fp32 parameter's dtype afterwards). The GEMMs are plain library GEMMs (cuBLAS
through ``torch.mm``); nothing is fused into them.
"""
from __future__ import annotations

import torch
from torch import Tensor

__all__ = ["linear_cast", "supports"]


def supports(x: Tensor, weight: Tensor, dtype: torch.dtype) -> bool:
    """CUDA input, a 16-bit compute dtype that differs from the weight's (the autocast case)."""
    return x.is_cuda and dtype in (torch.bfloat16, torch.float16) and weight.dtype != dtype


def _cached(owner, name: str, weight: Tensor, dtype: torch.dtype) -> Tensor:
    key = (dtype, weight.data_ptr(), weight._version, weight.dtype)
    slot = "_lp_" + name
    hit = owner.__dict__.get(slot)
    if hit is None or hit[0] != key:
        with torch.no_grad():
            hit = (key, weight.to(dtype).contiguous())
        owner.__dict__[slot] = hit
    return hit[1]


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, owner, name, dtype):
        w = _cached(owner, name, weight, dtype)
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
        return dx, dw, None, None, None


def linear_cast(x: Tensor, weight: Tensor, dtype: torch.dtype, owner, name: str) -> Tensor:
    """``x W^T`` in ``dtype`` (no bias), the weight's ``dtype`` copy kept on ``owner`` under ``name``."""
    with torch.autocast(x.device.type, enabled=False):
        return _LinearFn.apply(x, weight, owner, name, dtype)
