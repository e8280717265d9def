"""Fused SISA layer core on the sm_100a kernels (mirrors src/sisa/kernels/fused_prep.py of tlstngud/sisa).

``sisa_fused(proj, z, lam, n_head) -> y``: the preparation kernel (g, F, Phi scans and the rotation of
C/B) plus the tcgen05 attention forward; backward runs the exact-delta attention backward, whose dq,
dk, dv land directly in the Q/K/V columns of d_proj, then the reverse-scan kernel that fills the B, C,
theta, alpha and padding columns of d_proj and dz.
"""
from __future__ import annotations

import torch

from .. import _lib, backends

__all__ = ["sisa_fused", "fused_layout", "concat_fused_weights", "fused_projection", "prefill_layer"]

D_HEAD = 64
D_STATE = 32


def fused_layout(n_head: int, d_head: int = D_HEAD, d_state: int = D_STATE) -> dict:
    """Column offsets of the fused projection (src/sisa/kernels/fused_prep.py:71-96):
    ``[Q H*64 | K H*64 | V H*64 | B H*32 | C H*32 | TH H*16 | A H | zero padding to a multiple of 16]``."""
    if d_head != D_HEAD or d_state != D_STATE:
        raise ValueError(f"the fused kernels support d_head={D_HEAD} and d_state={D_STATE} only")
    H = int(n_head)
    o = {"Q": 0, "K": H * 64, "V": 2 * H * 64, "B": 3 * H * 64, "C": 3 * H * 64 + H * 32,
         "TH": 3 * H * 64 + 2 * H * 32}
    o["A"] = o["TH"] + H * 16
    o["NTOT"] = o["A"] + H
    o["NPAD"] = (o["NTOT"] + 15) // 16 * 16
    return o


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


class _FusedProjFn(torch.autograd.Function):
    """``proj = x W_cat^T + b_cat`` in the compute dtype, where ``b_cat`` is zero except the alpha
    columns. The forward is the call ``F.linear`` makes under autocast (inputs cast to the compute dtype,
    bias added in the GEMM epilogue before the one rounding); the backward runs the same two GEMMs as
    autograd's linear backward, but forms the bias gradient from the H alpha columns only, where
    autograd reduces all NPAD columns of the output gradient."""

    @staticmethod
    def forward(ctx, x, weight, b_alpha, col_a, dtype):
        H = b_alpha.shape[0]
        xc, wc = x.to(dtype), weight.to(dtype)
        bias = torch.zeros((weight.shape[0],), dtype=dtype, device=x.device)
        bias[col_a:col_a + H] = b_alpha.to(dtype)
        with torch.autocast(x.device.type, enabled=False):
            out = torch.nn.functional.linear(xc, wc, bias)
        ctx.save_for_backward(xc, wc)
        ctx.col_a, ctx.H = col_a, H
        ctx.dtypes = (x.dtype, weight.dtype, b_alpha.dtype)
        return out

    @staticmethod
    def backward(ctx, g):
        xc, wc = ctx.saved_tensors
        g2 = g.reshape(-1, g.shape[-1])
        dx = dw = db = None
        if ctx.needs_input_grad[0]:
            dx = (g2 @ wc).view(xc.shape).to(ctx.dtypes[0])
        if ctx.needs_input_grad[1]:
            dw = (g2.t() @ xc.reshape(-1, xc.shape[-1])).to(ctx.dtypes[1])
        if ctx.needs_input_grad[2]:
            db = g2[:, ctx.col_a:ctx.col_a + ctx.H].sum(0).to(ctx.dtypes[2])
        return dx, dw, db, None, None


def fused_projection(x: torch.Tensor, weight: torch.Tensor, b_alpha: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """``F.linear(x, W_cat, b_cat)`` under autocast to ``dtype`` (fused_prep.py:99-122) with ``b_cat`` built
    from ``b_alpha``; the same values, and a backward that reduces only the alpha columns for the bias."""
    col_a = fused_layout(b_alpha.shape[0])["A"]
    return _FusedProjFn.apply(x, weight, b_alpha, col_a, dtype)


def _heads(t: torch.Tensor, col: int, H: int, w: int) -> torch.Tensor:
    B, L, _ = t.shape
    return t[..., col:col + H * w].view(B, L, H, w).transpose(1, 2)


def _ws(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)


def prep_forward(proj: torch.Tensor, z: torch.Tensor | None, H: int):
    """Run the preparation kernels: returns (c_rot, b_rot, pos, tot)."""
    lib = _lib.load()
    B, L, _ = proj.shape
    dev = proj.device
    c_rot = torch.empty((B, H, L, D_STATE), device=dev, dtype=proj.dtype)
    b_rot = torch.empty_like(c_rot)
    pos = _lib.pos_planes(B, H, L, dev)
    tot = _ws(lib.sisa_prep_fwd_workspace(B, H, L), dev)
    st = backends.status_word(dev)
    rc = lib.sisa_prep_fwd(proj.data_ptr(), B, L, H, proj.stride(0), proj.stride(1), _lib.dtype_code(proj.dtype),
                           _lib.ptr(z), z.stride(0) if z is not None else 0, z.stride(1) if z is not None else 0,
                           c_rot.data_ptr(), b_rot.data_ptr(), pos.data_ptr(), tot.data_ptr(), st.data_ptr(),
                           _lib.stream_ptr(dev))
    _lib.check(rc, "sisa_prep_fwd")
    return c_rot, b_rot, pos, tot


class _SISAFusedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, proj, z, lam, H):
        lib = _lib.load()
        B, L, _ = proj.shape
        dev = proj.device
        off = fused_layout(H)
        c_rot, b_rot, pos, tot = prep_forward(proj, z, H)
        q, k, v = _heads(proj, off["Q"], H, 64), _heads(proj, off["K"], H, 64), _heads(proj, off["V"], H, 64)
        o = torch.empty_strided((B, H, L, D_HEAD), (L * H * D_HEAD, D_HEAD, H * D_HEAD, 1), device=dev,
                                dtype=proj.dtype)
        lse = torch.empty((B, H, L), device=dev, dtype=torch.float32)
        need = any(ctx.needs_input_grad)
        o32 = torch.empty((B, H, L, D_HEAD), device=dev, dtype=torch.float32) if need else None
        st = backends.status_word(dev)
        vq, vk, vv, vc, vb, vo = (_lib.view4(t) for t in (q, k, v, c_rot, b_rot, o))
        rc = lib.sisa_attn_fwd(_lib.vref(vq), _lib.vref(vk), _lib.vref(vv), _lib.vref(vc), _lib.vref(vb),
                               pos.data_ptr(), lam.data_ptr(), B, H, L, _lib.dtype_code(proj.dtype), _lib.vref(vo),
                               lse.data_ptr(), _lib.ptr(o32), st.data_ptr(), _lib.stream_ptr(dev))
        _lib.check(rc, "sisa_attn_fwd")
        backends.after_call(dev)
        ctx.save_for_backward(proj, z, lam, c_rot, b_rot, pos, tot, o, lse, o32)
        ctx.H = H
        return o.transpose(1, 2).reshape(B, L, H * D_HEAD)

    @staticmethod
    def backward(ctx, dy):
        lib = _lib.load()
        proj, z, lam, c_rot, b_rot, pos, tot, o, lse, o32 = ctx.saved_tensors
        H = ctx.H
        B, L, NP = proj.shape
        dev = proj.device
        off = fused_layout(H)
        dy = dy.contiguous()
        if dy.dtype != proj.dtype:
            dy = dy.to(proj.dtype)
        do = dy.view(B, L, H, D_HEAD).transpose(1, 2)
        dproj = torch.empty_like(proj)
        q, k, v = _heads(proj, off["Q"], H, 64), _heads(proj, off["K"], H, 64), _heads(proj, off["V"], H, 64)
        dq, dk, dv = _heads(dproj, off["Q"], H, 64), _heads(dproj, off["K"], H, 64), _heads(dproj, off["V"], H, 64)
        f32 = dict(device=dev, dtype=torch.float32)
        dc = torch.empty((B, H, L, D_STATE), **f32)
        db = torch.empty((B, H, L, D_STATE), **f32)
        dg = torch.empty((B, H, L), **f32)
        dF = torch.empty((B, H, L), **f32) if z is not None else None
        dlam = torch.empty((H,), **f32)
        ws = _ws(lib.sisa_attn_bwd_workspace(B, H, L), dev)
        st = backends.status_word(dev)
        views = [_lib.view4(t) for t in (q, k, v, c_rot, b_rot, o, do, dq, dk, dv, dc, db)]
        r = [_lib.vref(x) for x in views]
        rc = lib.sisa_attn_bwd(r[0], r[1], r[2], r[3], r[4], pos.data_ptr(), lam.data_ptr(), r[5], r[6],
                               lse.data_ptr(), _lib.ptr(o32), B, H, L, _lib.dtype_code(proj.dtype),
                               r[7], r[8], r[9], r[10], r[11], dg.data_ptr(), _lib.ptr(dF), dlam.data_ptr(),
                               ws.data_ptr(), st.data_ptr(), _lib.stream_ptr(dev))
        _lib.check(rc, "sisa_attn_bwd")
        dz = torch.empty((B, L, H), **f32) if z is not None else None
        bt = _ws(lib.sisa_prep_bwd_workspace(B, H, L), dev)
        rc = lib.sisa_prep_bwd(proj.data_ptr(), B, L, H, proj.stride(0), proj.stride(1),
                               _lib.dtype_code(proj.dtype), _lib.ptr(z), z.stride(0) if z is not None else 0,
                               z.stride(1) if z is not None else 0, tot.data_ptr(), dc.data_ptr(), db.data_ptr(),
                               dg.data_ptr(), _lib.ptr(dF), dproj.data_ptr(), dproj.stride(0), dproj.stride(1),
                               _lib.ptr(dz), bt.data_ptr(), st.data_ptr(), _lib.stream_ptr(dev))
        _lib.check(rc, "sisa_prep_bwd")
        backends.after_call(dev)
        return dproj, dz, dlam, None


def prefill_layer(proj: torch.Tensor, z: torch.Tensor, lam: torch.Tensor, n_head: int):
    """The layer core over a whole prompt without autograd, keeping what a decode cache needs: the
    preparation kernel and the tcgen05 forward (no o'' - nothing will run a backward), on the fused
    projection ``proj`` (B, L, NPAD) and forget logits ``z`` (B, L, H) fp32.

    The reference fills its cache through the unfused path instead (src/sisa/modeling.py:226-232: seven
    projections, torch recurrences and rotations). Returns ``y`` (B, L, H*64) and the cache entries:
    k, v (views of proj's K/V columns), b~ (B, H, L, 32) as the kernels rotated it, g and F (views of the
    position planes) and Phi at the last position (B, H, 16) fp32."""
    lib = _lib.load()
    H = int(n_head)
    B, L, _ = proj.shape
    dev = proj.device
    off = fused_layout(H)
    c_rot, b_rot, pos, _ = prep_forward(proj, z, H)
    q, k, v = _heads(proj, off["Q"], H, 64), _heads(proj, off["K"], H, 64), _heads(proj, off["V"], H, 64)
    o = torch.empty_strided((B, H, L, D_HEAD), (L * H * D_HEAD, D_HEAD, H * D_HEAD, 1), device=dev, dtype=proj.dtype)
    lse = torch.empty((B, H, L), device=dev, dtype=torch.float32)
    st = backends.status_word(dev)
    vq, vk, vv, vc, vb, vo = (_lib.view4(t) for t in (q, k, v, c_rot, b_rot, o))
    rc = lib.sisa_attn_fwd(_lib.vref(vq), _lib.vref(vk), _lib.vref(vv), _lib.vref(vc), _lib.vref(vb),
                           pos.data_ptr(), lam.data_ptr(), B, H, L, _lib.dtype_code(proj.dtype), _lib.vref(vo),
                           lse.data_ptr(), None, st.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(rc, "sisa_attn_fwd")
    backends.after_call(dev)
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
    if proj.stride(-1) != 1 or proj.stride(1) != NP or proj.stride(0) % 8 or proj.data_ptr() % 16:
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

