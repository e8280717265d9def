"""Chunked linear + cross-entropy over a tied LM head on the sm_100a kernels (the interface of
src/sisa/kernels/linear_ce.py).

``linear_cross_entropy(hidden, weight, labels)`` is the mean over non-ignored rows of
``cross_entropy(hidden @ weight.T, labels)`` with the logits rounded to the compute dtype, and it never
holds more than one chunk of logits. Everything happens in one operator, ``sisa_b200::lce``, during the
forward: per chunk of token rows the tcgen05 logits kernel (``sisa_lce_logits``) writes the chunk's
logits with per-tile online max / sum-exp partials, ``sisa_lce_grad`` turns them into the per-row loss
and overwrites the chunk with G = (softmax - onehot) * scale, and the CTA-pair tcgen05 GEMM
(``sisa_gemm``) takes dX = G W and dW += G^T X in fp32 (later chunks add into dW with TMA reduce-adds). The backward only scales the stored gradients by its seed, unless the caller
promised the seed (``grad_scale``), in which case G was already scaled and the backward checks the
promise on the device.

The operator needs CUDA tensors and a bf16/fp16 compute dtype (autocast's, else the input's). CPU
tensors take the plain formula :func:`reference_linear_cross_entropy`; an fp32 compute dtype on CUDA is
rejected rather than silently computed another way.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

from .. import _lib, backends
from .gemm import matmul_t

__all__ = ["linear_cross_entropy", "reference_linear_cross_entropy", "chunk_rows"]

VOCAB_ALIGN = 128          # vocabulary rows of the padded weight copy (the reference's padding)
LOGITS_BUDGET = 1 << 30    # bytes one chunk of logits may take
ROW_ALIGN = 128            # chunk rows are whole M tiles of the logits kernel


def chunk_rows(n_rows: int, vocab_padded: int, elem_bytes: int, requested: int | None = None) -> int:
    """Rows per chunk. ``requested`` wins; otherwise the fewest chunks whose logits fit the budget, made
    equal in size and rounded up to whole 128-row tiles (the reference's rule, linear_ce.py:116-124, which
    sets the peak memory)."""
    if requested:
        return max(1, min(n_rows, int(requested)))
    fit = max(ROW_ALIGN, LOGITS_BUDGET // (vocab_padded * elem_bytes))
    chunks = -(-n_rows // fit)
    even = -(-n_rows // chunks)
    return min(n_rows, -(-even // ROW_ALIGN) * ROW_ALIGN)


def reference_linear_cross_entropy(hidden: Tensor, weight: Tensor, labels: Tensor, ignore_index: int = -100) -> Tensor:
    """The plain formula ``F.cross_entropy(F.linear(hidden, weight).float(), labels, ignore_index)``
    (src/sisa/kernels/linear_ce.py:220-224)."""
    logits = F.linear(hidden, weight)
    return F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), labels.reshape(-1), ignore_index=ignore_index)


@torch.library.custom_op("sisa_b200::lce", mutates_args=())
def _lce(x: Tensor, w_pad: Tensor, labels: Tensor, vocab: int, ignore_index: int, rows: int, need_dx: bool,
         need_dw: bool, grad_scale: float) -> tuple[Tensor, Tensor, Tensor]:
    """Loss and gradients of one call. ``x`` (N, D) and ``w_pad`` (Vp, D) in the compute dtype, ``w_pad``
    zero beyond row ``vocab``; ``labels`` (N,) int64. Returns the fp32 loss, dX (N, D) fp32 and dW (Vp, D)
    fp32 (each empty when not asked for), both scaled by ``grad_scale``."""
    lib = _lib.load()
    N, D = x.shape
    Vp = w_pad.shape[0]
    dev = x.device
    code = _lib.dtype_code(x.dtype)
    st = backends.status_word(dev)
    sp = _lib.stream_ptr(dev)
    valid = (labels != ignore_index).sum()
    inv_valid = valid.to(torch.float32).reciprocal().reshape(1)
    per_row = torch.empty(N, dtype=torch.float32, device=dev)
    chunk = torch.empty((rows, Vp), dtype=x.dtype, device=dev)
    dx = torch.empty((N, D) if need_dx else (0,), dtype=torch.float32, device=dev)
    dw = torch.empty((Vp, D) if need_dw else (0,), dtype=torch.float32, device=dev)
    ws = None
    for start in range(0, N, rows):
        stop = min(N, start + rows)
        g = chunk[:stop - start]
        xs, ls = x[start:stop], labels[start:stop]
        # The chunk's per-row records (max / sum per 256 logit columns, the label's logit) live in the
        # chunk's own rows of dX, which its dX GEMM overwrites only after the gradient pass has read them;
        # when they do not fit there (or no dX is asked for), in a buffer of their own.
        need = lib.sisa_lce_workspace(stop - start, Vp)
        if need_dx and need <= (stop - start) * D * 4:
            ws_ptr = dx[start:stop].data_ptr()
        else:
            if ws is None or ws.numel() < need:
                ws = torch.empty(lib.sisa_lce_workspace(rows, Vp), dtype=torch.uint8, device=dev)
            ws_ptr = ws.data_ptr()
        _lib.check(lib.sisa_lce_logits(xs.data_ptr(), stop - start, D, xs.stride(0), w_pad.data_ptr(), vocab, Vp,
                                       w_pad.stride(0), code, ls.data_ptr(), g.data_ptr(), g.stride(0), ws_ptr,
                                       st.data_ptr(), sp), "sisa_lce_logits")
        _lib.check(lib.sisa_lce_grad(g.data_ptr(), g.stride(0), stop - start, vocab, Vp, code, ls.data_ptr(),
                                     ignore_index, inv_valid.data_ptr(), grad_scale, int(need_dx or need_dw),
                                     ws_ptr, per_row[start:stop].data_ptr(), st.data_ptr(), sp),
                   "sisa_lce_grad")
        if need_dx:
            matmul_t(g, w_pad.t(), dx[start:stop])
        if need_dw:
            matmul_t(g.t(), xs.t(), dw, accumulate=start > 0)
    backends.after_call(dev)
    return per_row.sum() / valid, dx, dw


@_lce.register_fake
def _(x, w_pad, labels, vocab, ignore_index, rows, need_dx, need_dw, grad_scale):
    N, D = x.shape
    f32 = dict(dtype=torch.float32)
    return (x.new_empty((), **f32), x.new_empty((N, D) if need_dx else (0,), **f32),
            x.new_empty((w_pad.shape[0], D) if need_dw else (0,), **f32))


class _LinearCE(torch.autograd.Function):
    """Loss in the forward together with the unscaled (or promised-scale) gradients; the backward scales.

    Eagerly the backward hands out the gradient buffers themselves, multiplied by the seed in place (not
    at all for a seed of 1, decided on the device), rather than fresh products, so a second backward
    through the same graph (``retain_graph=True``) is refused. Traced by torch.compile it returns the
    products ``seed * buffer`` as new tensors."""

    @staticmethod
    def forward(ctx, hidden, weight, labels, ignore_index, rows, cdtype, grad_scale):
        D = hidden.shape[-1]
        V = weight.shape[0]
        x = hidden.reshape(-1, D).to(cdtype).contiguous()
        Vp = -(-V // VOCAB_ALIGN) * VOCAB_ALIGN
        w_pad = torch.empty((Vp, D), dtype=cdtype, device=weight.device)
        w_pad[:V].copy_(weight.detach())            # the autocast rounding of the weight
        w_pad[V:].zero_()
        need_dx, need_dw = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        loss, dx, dw = _lce(x, w_pad, labels.reshape(-1).to(torch.int64).contiguous(), V, int(ignore_index),
                            chunk_rows(x.shape[0], Vp, x.element_size(), rows), need_dx, need_dw,
                            1.0 if grad_scale is None else float(grad_scale))
        ctx.save_for_backward(dx, dw)
        ctx.handed = False
        ctx.meta = (hidden.shape, hidden.dtype, weight.dtype, V, grad_scale)
        return loss

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, seed):
        dx, dw = ctx.saved_tensors
        h_shape, h_dtype, w_dtype, V, grad_scale = ctx.meta
        dev = seed.device
        if grad_scale is not None:
            # the gradients already carry the promised seed; a different one sets a status bit
            mismatch = (seed.float() != float(grad_scale)).to(torch.int32) * _lib.ST_BAD_SEED
            backends.status_word(dev).bitwise_or_(mismatch.reshape(1))
            backends.after_call(dev)
        if torch.compiler.is_compiling():
            scale = None if grad_scale is not None else seed.float()
            dh = dW = None
            if ctx.needs_input_grad[0]:
                dh = (dx if scale is None else dx * scale).view(h_shape).to(h_dtype)
            if ctx.needs_input_grad[1]:
                dW = (dw[:V] if scale is None else dw[:V] * scale).to(w_dtype)
            return dh, dW, None, None, None, None, None
        if ctx.handed:
            raise RuntimeError("linear_cross_entropy: backward ran twice through one graph; its gradient buffers "
                               "went to the first call (retain_graph is not supported)")
        ctx.handed = True
        if grad_scale is not None:
            seed32 = torch.ones(1, dtype=torch.float32, device=dev)
        else:
            seed32 = seed.detach().to(torch.float32).reshape(1).contiguous()
        lib = _lib.load()
        st, sp = backends.status_word(dev).data_ptr(), _lib.stream_ptr(dev)

        def scaled(buf, n, dtype):
            if n == 0:
                return torch.empty(0, dtype=dtype, device=dev)
            if dtype in (torch.bfloat16, torch.float16):
                out = torch.empty(n, dtype=dtype, device=dev)
                _lib.check(lib.sisa_lce_seed_scale(buf.data_ptr(), n, seed32.data_ptr(), out.data_ptr(),
                                                   _lib.dtype_code(dtype), st, sp), "sisa_lce_seed_scale")
                return out
            _lib.check(lib.sisa_lce_seed_scale(buf.data_ptr(), n, seed32.data_ptr(), None, _lib.F32, st, sp),
                       "sisa_lce_seed_scale")
            return buf.reshape(-1)[:n].to(dtype)

        dh = dW = None
        if ctx.needs_input_grad[0]:
            dh = scaled(dx, dx.numel(), h_dtype).view(h_shape)
        if ctx.needs_input_grad[1]:
            dW = scaled(dw, V * dw.shape[1], w_dtype).view(V, dw.shape[1])
        return dh, dW, None, None, None, None, None


def _compute_dtype(x: Tensor) -> torch.dtype:
    if torch.is_autocast_enabled(x.device.type):
        return torch.get_autocast_dtype(x.device.type)
    return x.dtype


def linear_cross_entropy(hidden: Tensor, weight: Tensor, labels: Tensor, ignore_index: int = -100, *,
                         chunk_tokens: int | None = None, grad_scale: float | None = None) -> Tensor:
    """Mean cross-entropy of ``hidden @ weight.T`` against ``labels`` without materialising all logits
    (src/sisa/kernels/linear_ce.py:228-259).

    Args:
        hidden: ``(..., D)``, D a multiple of 64; weight: ``(V, D)`` (receives dL/dW); labels: ``(...)``
            aligned with hidden's rows (not shifted here). Rows labelled ``ignore_index`` get no loss and
            no gradient.
        chunk_tokens: rows per chunk (default: equal chunks under a 1 GiB logits buffer).
        grad_scale: a promise that the backward is seeded with exactly this value; the gradients are then
            scaled once inside the kernels, and a different seed sets ``SISA_ST_BAD_SEED``.

    Returns the fp32 loss (NaN when every row is ignored, as ``F.cross_entropy``).
    """
    if not hidden.is_cuda:
        return reference_linear_cross_entropy(hidden, weight, labels, ignore_index)
    cdtype = _compute_dtype(hidden)
    if cdtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"the cuda linear-CE kernels take a bf16/fp16 compute dtype (enable autocast or pass "
                        f"low-precision inputs), got {cdtype}; reference_linear_cross_entropy computes it in fp32")
    D = hidden.shape[-1]
    if weight.dim() != 2 or weight.shape[1] != D:
        raise ValueError(f"weight must be (V, {D}), got {tuple(weight.shape)}")
    if labels.numel() * D != hidden.numel():
        raise ValueError(f"labels have {labels.numel()} elements, expected one per hidden row ({hidden.numel() // D})")
    if D % 64:
        raise ValueError(f"the cuda linear-CE kernel needs a hidden size that is a multiple of 64, got {D}")
    with torch.autocast(hidden.device.type, enabled=False):
        return _LinearCE.apply(hidden, weight, labels, ignore_index, chunk_tokens, cdtype, grad_scale)
