"""Fused RMSNorm and SwiGLU activation for the model's blocks (reference: src/sisa/modeling.py:25-49).

``rms_norm(x, weight, eps)`` computes ``((x.float() * rsqrt(mean(x.float()^2) + eps)) * weight.float())
.to(x.dtype)`` in one sm_100a kernel (the eager form is six), and its backward in three (dx per row, dw
from fixed-order partial sums, deterministic). ``block_norm`` is the same norm with what the blocks do
around it folded in: the residual add before it, one output copy per consumer in the dtype that
consumer casts to, and the attention's fp32 forget projection of the output (section comment of
csrc/norm.cu). ``swiglu(g, u)`` computes ``silu(g) * u`` and its backward in one kernel each, in fp32
with one rounding. All raise if the CUDA library is missing; the callers choose them only for CUDA
tensors on the ``cuda`` path.
"""
from __future__ import annotations

import ctypes

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


class _BlockNormFn(torch.autograd.Function):
    """Outputs, in order: ``x + res`` (with ``res`` and ``keep_sum``), one normalised copy per entry of
    ``out_dtypes``, and ``z`` (with a projection). Each output's gradient arrives separately and the
    backward kernel sums them in fp32, as autograd sums the gradients of the reference's casts."""

    @staticmethod
    def forward(ctx, x, res, weight, proj_w, proj_b, eps, out_dtypes, keep_sum):
        lib = _lib.load()
        shape, dev = x.shape, x.device
        x2 = _rows(x)
        rows, d = x2.shape
        a = _lib.NormFwdArgs()
        a.x, a.x_ld, a.x_dtype = x2.data_ptr(), x2.stride(0), _code(x.dtype)
        res2 = xsum = None
        if res is not None:
            if res.shape != shape:
                raise ValueError(f"block_norm: res {tuple(res.shape)} must match x {tuple(shape)}")
            res2 = _rows(res)
            xsum = torch.empty((rows, d), dtype=x.dtype, device=dev)
            a.res, a.res_ld, a.res_dtype = res2.data_ptr(), res2.stride(0), _code(res.dtype)
            a.xsum, a.xsum_ld = xsum.data_ptr(), d
        w = weight.float().contiguous()
        a.weight, a.rows, a.d, a.eps = w.data_ptr(), rows, d, float(eps)
        ys = [torch.empty((rows, d), dtype=dt, device=dev) for dt in out_dtypes]
        a.n_out = len(ys)
        for k, y in enumerate(ys):
            a.y[k], a.y_ld[k], a.y_dtype[k] = y.data_ptr(), d, _code(y.dtype)
        rstd = torch.empty((rows,), dtype=torch.float32, device=dev)
        a.rstd = rstd.data_ptr()
        pw = z = None
        if proj_w is not None:
            pw, pb = proj_w.float().contiguous(), proj_b.float().contiguous()
            z = torch.empty((rows, pw.shape[0]), dtype=torch.float32, device=dev)
            a.proj_w, a.proj_b, a.n_proj, a.proj_out = pw.data_ptr(), pb.data_ptr(), pw.shape[0], z.data_ptr()
        _lib.check(lib.sisa_norm_fwd(ctypes.byref(a), None, _lib.stream_ptr(dev)), "sisa_norm_fwd")
        ctx.save_for_backward(xsum if res is not None else x2, w, rstd, pw)
        ctx.set_materialize_grads(False)
        ctx.shape, ctx.x_dtype = shape, x.dtype
        ctx.res_dtype = None if res is None else res.dtype
        ctx.has_sum = res is not None and keep_sum
        ctx.n_out = len(ys)
        ctx.wdtype = weight.dtype
        ctx.pdtypes = None if proj_w is None else (proj_w.dtype, proj_b.dtype)
        outs = ([xsum.view(shape)] if ctx.has_sum else []) + [y.view(shape) for y in ys]
        if z is not None:
            outs.append(z.view(*shape[:-1], z.shape[-1]))
        return tuple(outs)

    @staticmethod
    def backward(ctx, *grads):
        lib = _lib.load()
        v, w, rstd, pw = ctx.saved_tensors
        rows, d = v.shape
        dev = v.device
        i = 0
        dsum = None
        if ctx.has_sum:
            dsum, i = grads[0], 1
        dys = [g for g in grads[i:i + ctx.n_out] if g is not None]
        dz = grads[i + ctx.n_out] if ctx.pdtypes is not None else None
        a = _lib.NormBwdArgs()
        a.v, a.v_ld, a.v_dtype = v.data_ptr(), v.stride(0), _code(v.dtype)
        a.weight, a.rstd, a.rows, a.d = w.data_ptr(), rstd.data_ptr(), rows, d
        keep = []
        for k, g in enumerate(dys):
            g2 = _rows(g)
            keep.append(g2)
            a.dy[k], a.dy_ld[k], a.dy_dtype[k] = g2.data_ptr(), g2.stride(0), _code(g2.dtype)
        if dsum is not None:
            ds2 = _rows(dsum)
            keep.append(ds2)
            a.dv_in, a.dv_in_ld, a.dv_in_dtype = ds2.data_ptr(), ds2.stride(0), _code(ds2.dtype)
        n_proj = 0
        if dz is not None:
            n_proj = pw.shape[0]
            dz2 = dz.reshape(rows, n_proj).float().contiguous()
            keep.append(dz2)
            a.proj_w, a.n_proj, a.dproj_out = pw.data_ptr(), n_proj, dz2.data_ptr()
        dx = torch.empty((rows, d), dtype=ctx.x_dtype, device=dev)
        a.dx, a.dx_ld, a.dx_dtype = dx.data_ptr(), d, _code(dx.dtype)
        dres = None
        if ctx.res_dtype is not None and ctx.needs_input_grad[1]:
            dres = torch.empty((rows, d), dtype=ctx.res_dtype, device=dev)
            a.dres, a.dres_ld, a.dres_dtype = dres.data_ptr(), d, _code(dres.dtype)
        dw = dpw = dpb = None
        if ctx.needs_input_grad[2]:
            dw = torch.empty((d,), dtype=torch.float32, device=dev)
            a.dweight = dw.data_ptr()
        if n_proj and (ctx.needs_input_grad[3] or ctx.needs_input_grad[4]):
            dpw = torch.empty((n_proj, d), dtype=torch.float32, device=dev)
            dpb = torch.empty((n_proj,), dtype=torch.float32, device=dev)
            a.dproj_w, a.dproj_b = dpw.data_ptr(), dpb.data_ptr()
        ws = None
        if dw is not None or dpw is not None:
            ws = torch.empty((lib.sisa_norm_bwd_workspace(rows, d, n_proj),), dtype=torch.uint8, device=dev)
            a.workspace = ws.data_ptr()
        _lib.check(lib.sisa_norm_bwd(ctypes.byref(a), None, _lib.stream_ptr(dev)), "sisa_norm_bwd")
        shape = ctx.shape
        return (dx.view(shape), None if dres is None else dres.view(shape),
                None if dw is None else dw.to(ctx.wdtype),
                None if dpw is None else dpw.to(ctx.pdtypes[0]), None if dpb is None else dpb.to(ctx.pdtypes[1]),
                None, None, None)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm of the last axis in fp32, output in x's dtype (modeling.py:25-36), on the sm_100a kernels."""
    return _BlockNormFn.apply(x, None, weight, None, None, eps, (x.dtype,), False)[0]


def block_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, *, res: torch.Tensor | None = None,
               out_dtypes=None, proj: tuple[torch.Tensor, torch.Tensor] | None = None,
               keep_sum: bool = True) -> tuple[torch.Tensor, ...]:
    """RMSNorm of ``v = x + res`` (or of ``x``) with its consumers' casts and the forget projection folded in.

    Returns ``(v,)`` (when ``res`` is given and ``keep_sum``), then ``h`` in each dtype of ``out_dtypes``
    (default: x's dtype), then ``z = h proj_w^T + proj_b`` in fp32 (when ``proj`` is given). ``h`` is the
    reference's RMSNorm output ``((v.float() * rstd) * weight.float()).to(v.dtype)``, stored in each
    requested dtype by one rounding, which is the cast the next linear applies under autocast
    (modeling.py:25-36, 167-168, 275-276)."""
    out_dtypes = tuple(out_dtypes or (x.dtype,))
    if not 1 <= len(out_dtypes) <= 2:
        raise ValueError("block_norm: one or two output dtypes")
    pw, pb = proj if proj is not None else (None, None)
    return _BlockNormFn.apply(x, res, weight, pw, pb, eps, out_dtypes, keep_sum)


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
