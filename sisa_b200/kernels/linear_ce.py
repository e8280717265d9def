"""Chunked linear + cross-entropy for a tied LM head on the sm_100a kernels
(mirrors src/sisa/kernels/linear_ce.py).

``linear_cross_entropy(hidden, weight, labels)`` returns the loss of
``F.cross_entropy(F.linear(hidden, weight).float(), labels, ignore_index=-100)`` (mean over non-ignored
rows) and computes the gradients for ``hidden`` and ``weight`` during the forward pass, chunk by chunk:
the tcgen05 logits kernel (``sisa_lce_logits``) writes a chunk of compute-dtype logits together with
per-tile online max/sum-exp partials, ``sisa_lce_grad`` turns them into the loss rows and overwrites the
chunk with G = (softmax - onehot) / N_valid, and two plain cuBLAS GEMMs give dX = G W and dW += G^T X
(fp32 outputs). Only one chunk of logits exists at a time (by default balanced chunks under 1 GiB).

CPU tensors or an fp32 compute dtype use the eager formula, as the reference does.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .. import _lib, backends

__all__ = ["linear_cross_entropy", "reference_linear_cross_entropy"]

_CHUNK_MB = 1024
_VPAD = 256


def _compute_dtype(x):
    try:
        if torch.is_autocast_enabled(x.device.type):
            return torch.get_autocast_dtype(x.device.type)
    except (TypeError, RuntimeError):
        pass
    return x.dtype


def _pick_chunk(N, Vp, chunk_tokens, elt):
    """Rows per chunk: explicit, or balanced chunks under the 1 GiB logits budget rounded to 128 rows
    (linear_ce.py:116-124)."""
    if chunk_tokens:
        return max(1, min(N, int(chunk_tokens)))
    tmax = max(128, (_CHUNK_MB << 20) // (Vp * elt))
    n_chunks = -(-N // tmax)
    t = -(-N // n_chunks)
    return min(N, -(-t // 128) * 128)


def _padded_weight(w, dtype):
    V, D = w.shape
    Vp = -(-V // _VPAD) * _VPAD
    out = torch.empty((Vp, D), dtype=dtype, device=w.device)
    out[:V].copy_(w.detach())
    if Vp > V:
        out[V:].zero_()
    return out


class _LinearCrossEntropyFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, w, labels, opts):
        ignore_index, chunk_tokens, cdtype, need_dh, need_dw, grad_scale = opts
        lib = _lib.load()
        need_grad = need_dh or need_dw
        D = h.shape[-1]
        V = w.shape[0]
        dev = h.device
        x = h.reshape(-1, D)
        N = x.shape[0]
        lab = labels.reshape(-1)
        if lab.dtype != torch.int64:
            lab = lab.long()
        lab = lab.contiguous()
        xb = (x if x.dtype == cdtype else x.to(cdtype)).contiguous()
        wp = _padded_weight(w, cdtype)
        Vp = wp.shape[0]
        n_valid = (lab != ignore_index).sum()
        inv_n = torch.reciprocal(n_valid.to(torch.float32)).reshape(1)
        loss_rows = torch.empty(N, dtype=torch.float32, device=dev)
        T = _pick_chunk(N, Vp, chunk_tokens, wp.element_size())
        buf = torch.empty((T, Vp), dtype=cdtype, device=dev)
        ws = torch.empty(lib.sisa_lce_workspace(T, Vp), dtype=torch.uint8, device=dev)
        dx = torch.empty((N, D), dtype=torch.float32, device=dev) if need_dh else None
        dw = torch.empty((Vp, D), dtype=torch.float32, device=dev) if need_dw else None
        gs = 1.0 if grad_scale is None else float(grad_scale)
        st = backends.status_word(dev)
        sp = _lib.stream_ptr(dev)
        code = _lib.dtype_code(cdtype)
        first = True
        for s in range(0, N, T):
            e = min(N, s + T)
            R = e - s
            lg = buf[:R]
            xc = xb[s:e]
            rc = lib.sisa_lce_logits(xc.data_ptr(), R, D, xc.stride(0), wp.data_ptr(), V, Vp, wp.stride(0), code,
                                     lab[s:e].data_ptr(), lg.data_ptr(), lg.stride(0), ws.data_ptr(), st.data_ptr(), sp)
            _lib.check(rc, "sisa_lce_logits")
            rc = lib.sisa_lce_grad(lg.data_ptr(), lg.stride(0), R, V, Vp, code, lab[s:e].data_ptr(), ignore_index,
                                   inv_n.data_ptr(), gs, int(need_grad), ws.data_ptr(), loss_rows[s:e].data_ptr(),
                                   st.data_ptr(), sp)
            _lib.check(rc, "sisa_lce_grad")
            if need_dh:
                torch.mm(lg, wp, out_dtype=torch.float32, out=dx[s:e])
            if need_dw:
                if first:
                    torch.mm(lg.t(), xc, out_dtype=torch.float32, out=dw)
                else:
                    torch.addmm(dw, lg.t(), xc, out_dtype=torch.float32, out=dw)
            first = False
        backends.after_call(dev)
        loss = loss_rows.sum() / n_valid
        ctx.h_shape, ctx.h_dtype, ctx.w_dtype, ctx.grad_scale, ctx.V = h.shape, h.dtype, w.dtype, grad_scale, V
        ctx.save_for_backward(dx, dw)
        return loss

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, g):
        dx, dw = ctx.saved_tensors
        if ctx.grad_scale is not None:
            # G was pre-scaled by the promised seed; a different seed sets the status bit
            bad = (g.to(torch.float32) != float(ctx.grad_scale)).to(torch.int32) * _lib.ST_BAD_SEED
            st = backends.status_word(g.device)
            st.bitwise_or_(bad.reshape(1))
            backends.after_call(g.device)
            dh = dx.view(ctx.h_shape) if dx is not None else None
            dW = dw[:ctx.V] if dw is not None else None
        else:
            g = g.to(torch.float32)
            dh = torch.mul(dx, g).view(ctx.h_shape) if dx is not None else None
            dW = torch.mul(dw[:ctx.V], g) if dw is not None else None
        if dh is not None and dh.dtype != ctx.h_dtype:
            dh = dh.to(ctx.h_dtype)
        if dW is not None and dW.dtype != ctx.w_dtype:
            dW = dW.to(ctx.w_dtype)
        return dh, dW, None, None


def reference_linear_cross_entropy(hidden, weight, labels, ignore_index: int = -100):
    """The eager formula: ``F.cross_entropy(F.linear(hidden, weight).float(), labels, ignore_index)``."""
    logits = F.linear(hidden, weight)
    return F.cross_entropy(logits.view(-1, logits.size(-1)).float(), labels.reshape(-1), ignore_index=ignore_index)


@torch.compiler.disable
def linear_cross_entropy(hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor, ignore_index: int = -100,
                         *, chunk_tokens: int | None = None, grad_scale: float | None = None) -> torch.Tensor:
    """Mean cross-entropy of ``hidden @ weight.T`` against ``labels`` (src/sisa/kernels/linear_ce.py:228-259).

    Args:
        hidden: ``(..., D)``; weight: ``(V, D)`` (receives dL/dW); labels: ``(...)`` aligned with hidden rows
            (no shifting here), ``ignore_index`` rows get no loss and no gradient.
        chunk_tokens: rows per chunk (default: balanced chunks under a 1 GiB logits buffer).
        grad_scale: promise that backward is seeded with exactly this value; G is then pre-scaled and a
            different seed sets ``SISA_ST_BAD_SEED`` (raised by the check mode).
    """
    cdtype = _compute_dtype(hidden)
    if cdtype not in (torch.bfloat16, torch.float16) or not hidden.is_cuda:
        return reference_linear_cross_entropy(hidden, weight, labels, ignore_index)
    if weight.dim() != 2 or weight.shape[1] != hidden.shape[-1]:
        raise ValueError(f"weight must be (V, {hidden.shape[-1]}), got {tuple(weight.shape)}")
    if labels.numel() != hidden.numel() // hidden.shape[-1]:
        raise ValueError(f"labels have {labels.numel()} elements, expected one per hidden row "
                         f"({hidden.numel() // hidden.shape[-1]})")
    if hidden.shape[-1] % 64:
        raise ValueError(f"the cuda linear-CE kernel needs a hidden size that is a multiple of 64, got {hidden.shape[-1]}")
    ge = torch.is_grad_enabled()
    opts = (ignore_index, chunk_tokens, cdtype, bool(ge and hidden.requires_grad), bool(ge and weight.requires_grad),
            grad_scale)
    return _LinearCrossEntropyFn.apply(hidden, weight, labels, opts)
