"""The SwiGLU MLP's gate and up projections as one tcgen05 GEMM with the activation in its epilogue
(``sisa_gemm_swiglu``): ``silu(h W_gate^T) * (h W_up^T)`` of src/sisa/modeling.py:39-49 under autocast.

The two weights are kept as one compute-dtype copy with their rows interleaved in blocks of 8 (gate rows
8b .. 8b + 7, then the up rows of the same features), so that every epilogue warp holds the gate and up
values of its features. The forward writes the activation ``a`` and, in the same interleaved column
order, the rounded gate and up outputs the backward needs. The backward runs the SwiGLU derivative kernel
on that layout, then the plain GEMMs ``dh = dgu W_il`` and ``dW_il = dgu^T h`` (cuBLAS through
``torch.mm``), and hands each weight its rows of ``dW_il``.
"""
from __future__ import annotations

import torch
from torch import Tensor

from .. import _lib, backends

__all__ = ["gate_up_swiglu", "interleave_gate_up", "supports"]

BLOCK = 8          # rows per interleave block (one 16-byte vector of a 16-bit type)


def supports(h: Tensor, d_ff: int, dtype: torch.dtype) -> bool:
    """Whether the fused kernel takes this input: CUDA, a 16-bit compute dtype, widths of whole 16-byte
    vectors."""
    return h.is_cuda and dtype in (torch.bfloat16, torch.float16) and d_ff % BLOCK == 0 and h.shape[-1] % 8 == 0


def interleave_gate_up(w_gate: Tensor, w_up: Tensor, dtype: torch.dtype) -> Tensor:
    """``(2 d_ff, d)`` in ``dtype``: block b of 8 gate rows, then block b of 8 up rows, for every b."""
    d_ff, d = w_gate.shape
    w = torch.empty((d_ff // BLOCK, 2, BLOCK, d), dtype=dtype, device=w_gate.device)
    with torch.no_grad():
        w[:, 0].copy_(w_gate.view(d_ff // BLOCK, BLOCK, d))
        w[:, 1].copy_(w_up.view(d_ff // BLOCK, BLOCK, d))
    return w.view(2 * d_ff, d)


def gate_up_key(w_gate: Tensor, w_up: Tensor, dtype: torch.dtype) -> tuple:
    """The key under which the interleaved compute-dtype copy is kept (``_gate_up_il``)."""
    return (dtype,) + tuple((w.data_ptr(), w._version, w.dtype) for w in (w_gate, w_up))


def _cached(owner, w_gate: Tensor, w_up: Tensor, dtype: torch.dtype, train: bool = False) -> Tensor:
    """The interleaved copy kept on ``owner`` (outside the autograd graph), used as
    ``kernels.fused.take_fresh`` allows and rebuilt otherwise."""
    from .fused import take_fresh

    key = gate_up_key(w_gate, w_up, dtype)
    hit = take_fresh(owner, "_gate_up_il", key, train)
    if hit is None:
        hit = interleave_gate_up(w_gate, w_up, dtype)
        owner.__dict__["_gate_up_il"] = (key, hit, False)
    return hit


class _GateUpFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w_gate, w_up, owner, dtype, train):
        d = h.shape[-1]
        d_ff = w_gate.shape[0]
        h2 = h.reshape(-1, d).to(dtype).contiguous()
        rows = h2.shape[0]
        w_il = _cached(owner, w_gate, w_up, dtype, train)
        gu = torch.empty((rows, 2 * d_ff), dtype=dtype, device=h.device)
        a = torch.empty((rows, d_ff), dtype=dtype, device=h.device)
        if rows:
            dev = h.device
            _lib.check(_lib.load().sisa_gemm_swiglu(h2.data_ptr(), d, w_il.data_ptr(), d, gu.data_ptr(), 2 * d_ff,
                                                    a.data_ptr(), d_ff, rows, d_ff, d, _lib.dtype_code(dtype),
                                                    backends.status_word(dev).data_ptr(), _lib.stream_ptr(dev)),
                       "sisa_gemm_swiglu")
            backends.after_call(dev)
        ctx.save_for_backward(h2, w_il, gu)
        ctx.meta = (h.shape, h.dtype, w_gate.dtype, w_up.dtype)
        return a.view(*h.shape[:-1], d_ff)

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, da):
        h2, w_il, gu = ctx.saved_tensors
        h_shape, h_dtype, g_dtype, u_dtype = ctx.meta
        rows, d = h2.shape
        d_ff = w_il.shape[0] // 2
        dgu = torch.empty_like(gu)
        if rows:
            da2 = da.reshape(rows, d_ff).to(gu.dtype).contiguous()
            # the interleaved layout as (rows * d_ff / 8) rows of 8 features: gate at +0, up at +8 of a
            # 16-element stride
            n = rows * (d_ff // BLOCK)
            es = gu.element_size()
            _lib.check(_lib.load().sisa_swiglu_bwd(da2.data_ptr(), BLOCK, gu.data_ptr(), 2 * BLOCK,
                                                   gu.data_ptr() + BLOCK * es, 2 * BLOCK, n, BLOCK,
                                                   _lib.dtype_code(gu.dtype), dgu.data_ptr(), 2 * BLOCK,
                                                   dgu.data_ptr() + BLOCK * es, 2 * BLOCK, None,
                                                   _lib.stream_ptr(gu.device)), "sisa_swiglu_bwd")
        dh = dwg = dwu = None
        if ctx.needs_input_grad[0]:
            dh = torch.mm(dgu, w_il).view(h_shape).to(h_dtype)
        if ctx.needs_input_grad[1] or ctx.needs_input_grad[2]:
            dw = torch.mm(dgu.t(), h2, out_dtype=torch.float32).view(d_ff // BLOCK, 2, BLOCK, d)
            if ctx.needs_input_grad[1] and ctx.needs_input_grad[2]:
                # one launch takes both weights' rows out of the interleaved dW (sisa_split_rows)
                dwg = torch.empty((d_ff, d), dtype=torch.float32, device=dw.device)
                dwu = torch.empty_like(dwg)
                _lib.check(_lib.load().sisa_split_rows(dw.data_ptr(), d, dwg.data_ptr(), dwu.data_ptr(), d, d_ff, d,
                                                       BLOCK, _lib.stream_ptr(dw.device)), "sisa_split_rows")
                dwg, dwu = dwg.to(g_dtype), dwu.to(u_dtype)
            elif ctx.needs_input_grad[1]:
                dwg = dw[:, 0].reshape(d_ff, d).to(g_dtype)
            else:
                dwu = dw[:, 1].reshape(d_ff, d).to(u_dtype)
        return dh, dwg, dwu, None, None, None


def _gate_up_inference(h: Tensor, w_gate: Tensor, w_up: Tensor, dtype: torch.dtype, owner) -> Tensor:
    """The forward alone: only the activation is stored (the projections are what a backward would read)."""
    d = h.shape[-1]
    d_ff = w_gate.shape[0]
    h2 = h.reshape(-1, d).to(dtype).contiguous()
    rows = h2.shape[0]
    w_il = _cached(owner, w_gate, w_up, dtype, False)
    a = torch.empty((rows, d_ff), dtype=dtype, device=h.device)
    if rows:
        dev = h.device
        _lib.check(_lib.load().sisa_gemm_swiglu(h2.data_ptr(), d, w_il.data_ptr(), d, None, 0, a.data_ptr(), d_ff,
                                                rows, d_ff, d, _lib.dtype_code(dtype),
                                                backends.status_word(dev).data_ptr(), _lib.stream_ptr(dev)),
                   "sisa_gemm_swiglu")
        backends.after_call(dev)
    return a.view(*h.shape[:-1], d_ff)


def gate_up_swiglu(h: Tensor, w_gate: Tensor, w_up: Tensor, dtype: torch.dtype, owner) -> Tensor:
    """``silu(h W_gate^T) * (h W_up^T)`` in ``dtype`` (the autocast computation of modeling.py:39-49 up to
    the activation's single rounding), on the fused GEMM. ``owner`` keeps the interleaved weight copy.
    Without a gradient to compute, the projections are not stored at all."""
    if not supports(h, w_gate.shape[0], dtype):
        raise ValueError(f"gate_up_swiglu needs a CUDA input, a bf16/fp16 compute dtype and widths divisible by 8; "
                         f"got {h.device}, {dtype}, d_ff={w_gate.shape[0]}, d={h.shape[-1]}")
    with torch.autocast(h.device.type, enabled=False):
        if not torch.is_grad_enabled() or not (h.requires_grad or w_gate.requires_grad or w_up.requires_grad):
            return _gate_up_inference(h, w_gate, w_up, dtype, owner)
        return _GateUpFn.apply(h, w_gate, w_up, owner, dtype, torch.is_grad_enabled())
