"""The sm_100a kernels as PyTorch custom operators (namespace ``sisa_b200``).

Each operator is one launch sequence of the C ABI (``include/sisa_b200.h``) on torch's current
stream, with every output allocated here. They are registered through ``torch.library`` together with
fake (shape-only) implementations, so torch.compile can trace a model on the cuda path without graph
breaks; the autograd functions of :mod:`sisa_b200.kernels` are built from them. An output a call does
not produce is returned as an empty tensor. The reference wraps its Triton launchers in plain Python
autograd functions, which compiled graphs break around (its README.md:473-476).

The operators read the check mode (:mod:`sisa_b200.backends`): in ``"sync"`` mode each one raises for
a status bit its kernels set.
"""
from __future__ import annotations

import torch
from torch import Tensor

from . import _lib, backends

__all__ = ["prep_fwd", "pack_positions", "attn_fwd", "attn_bwd", "fused_bwd", "fused_layout", "heads",
           "base_misaligned"]

D_HEAD = 64
D_STATE = 32


def fused_layout(n_head: int) -> dict:
    """Column offsets of the fused projection (src/sisa/kernels/fused_prep.py:71-96):
    ``[Q H*64 | K H*64 | V H*64 | B H*32 | C H*32 | TH H*16 | A H | zero padding to a multiple of 16]``."""
    H = int(n_head)
    o = {"Q": 0, "K": H * 64, "V": 2 * H * 64, "B": 3 * H * 64, "C": 3 * H * 64 + H * 32,
         "TH": 3 * H * 64 + 2 * H * 32}
    o["A"] = o["TH"] + H * 16
    o["NTOT"] = o["A"] + H
    o["NPAD"] = (o["NTOT"] + 15) // 16 * 16
    return o


def heads(t: Tensor, col: int, H: int, w: int) -> Tensor:
    """The (B, H, L, w) view of columns [col, col + H*w) of a (B, L, N) tensor."""
    B, L, _ = t.shape
    return t[..., col:col + H * w].view(B, L, H, w).transpose(1, 2)


def _bytes(n: int, device) -> Tensor:
    return torch.empty(max(int(n), 16), dtype=torch.uint8, device=device)


def _o_like(B: int, H: int, L: int, dtype, device) -> Tensor:
    """(B, H, L, 64) with (B, L, H, 64) storage, so that the heads-concatenated output is a view."""
    return torch.empty_strided((B, H, L, D_HEAD), (L * H * D_HEAD, D_HEAD, H * D_HEAD, 1), dtype=dtype, device=device)


def base_misaligned(t: Tensor) -> bool:
    """Whether ``t`` starts off a 16-byte boundary (the TMA tensor maps need 16-byte aligned bases).
    A traced graph has no storage to look at, so under torch.compile this reports False and the C ABI's
    own check (SISA_ERR_ALIGN, raised as ValueError) stays the guard."""
    if torch.compiler.is_compiling():
        return False
    return t.data_ptr() % 16 != 0


def _none_if_empty(t: Tensor | None) -> Tensor | None:
    return None if t is None or t.numel() == 0 else t


def _zero_plane_padding(pos: Tensor, L: int) -> None:
    """The position planes' alignment padding (columns L..Lp-1) is never read; zero it so that every
    output of the operators is defined."""
    if pos.shape[-1] > L:
        pos[..., L:].zero_()


# ------------------------------------------------------------------------------------------------ prep
@torch.library.custom_op("sisa_b200::prep_fwd", mutates_args=())
def prep_fwd(proj: Tensor, z: Tensor | None, n_head: int) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """``sisa_prep_fwd``: the g / F / Phi scans and the rotation of C and B from the fused projection
    ``proj`` (B, L, NPAD) and forget logits ``z`` (B, L, H) fp32 or None. Returns c~, b~ (B, H, L, 32)
    in proj.dtype, the planar position records (B, H, 4, Lp) fp32 and the block-total workspace."""
    lib = _lib.load()
    B, L, _ = proj.shape
    H = int(n_head)
    dev = proj.device
    c_rot = torch.empty((B, H, L, D_STATE), device=dev, dtype=proj.dtype)
    b_rot = torch.empty_like(c_rot)
    pos = _lib.pos_planes(B, H, L, dev)
    tot = _bytes(lib.sisa_prep_fwd_workspace(B, H, L), dev)
    st = backends.status_word(dev)
    rc = lib.sisa_prep_fwd(proj.data_ptr(), B, L, H, proj.stride(0), proj.stride(1), _lib.dtype_code(proj.dtype),
                           _lib.ptr(z), z.stride(0) if z is not None else 0, z.stride(1) if z is not None else 0,
                           c_rot.data_ptr(), b_rot.data_ptr(), pos.data_ptr(), tot.data_ptr(), st.data_ptr(),
                           _lib.stream_ptr(dev))
    _lib.check(rc, "sisa_prep_fwd")
    _zero_plane_padding(pos, L)
    return c_rot, b_rot, pos, tot


@prep_fwd.register_fake
def _(proj, z, n_head):
    B, L, _ = proj.shape
    H = int(n_head)
    lp = (L + 3) // 4 * 4
    c = proj.new_empty((B, H, L, D_STATE))
    return c, torch.empty_like(c), proj.new_empty((B, H, 4, lp), dtype=torch.float32), \
        proj.new_empty((max(B * H * ((L + 63) // 64) * 18 * 4, 16),), dtype=torch.uint8)


@torch.library.custom_op("sisa_b200::pack_positions", mutates_args=())
def pack_positions(g: Tensor, fgate: Tensor | None) -> Tensor:
    """``sisa_pack_positions``: planar position records (B, H, 4, Lp) fp32 from g and fgate (B, H, L)
    fp32 (fgate may be None); a g that rises by more than 1e-3 sets SISA_ST_NONMONOTONE."""
    lib = _lib.load()
    B, H, L = g.shape
    pos = _lib.pos_planes(B, H, L, g.device)
    st = backends.status_word(g.device)
    fs = fgate.stride() if fgate is not None else (0, 0, 0)
    rc = lib.sisa_pack_positions(g.data_ptr(), *g.stride(), _lib.ptr(fgate), *fs, B, H, L, pos.data_ptr(),
                                 st.data_ptr(), _lib.stream_ptr(g.device))
    _lib.check(rc, "sisa_pack_positions")
    _zero_plane_padding(pos, L)
    return pos


@pack_positions.register_fake
def _(g, fgate):
    B, H, L = g.shape
    return g.new_empty((B, H, 4, (L + 3) // 4 * 4))


# ------------------------------------------------------------------------------------------------ attention
@torch.library.custom_op("sisa_b200::attn_fwd", mutates_args=())
def attn_fwd(q: Tensor, k: Tensor, v: Tensor, c: Tensor, b: Tensor, pos: Tensor, lam: Tensor,
             keep_o32: bool) -> tuple[Tensor, Tensor, Tensor]:
    """``sisa_attn_fwd``: o (B, H, L, 64) in q.dtype stored as (B, L, H, 64), lse (B, H, L) fp32 in log2
    units and, with ``keep_o32``, the self-normalised fp32 output o'' the backward needs (else empty)."""
    lib = _lib.load()
    B, H, L, _ = q.shape
    dev = q.device
    o = _o_like(B, H, L, q.dtype, dev)
    lse = torch.empty((B, H, L), device=dev, dtype=torch.float32)
    o32 = torch.empty((B, H, L, D_HEAD), device=dev, dtype=torch.float32) if keep_o32 else \
        torch.empty(0, device=dev, dtype=torch.float32)
    st = backends.status_word(dev)
    vs = [_lib.view4(t) for t in (q, k, v, c, b, o)]
    r = [_lib.vref(x) for x in vs]
    rc = lib.sisa_attn_fwd(r[0], r[1], r[2], r[3], r[4], pos.data_ptr(), lam.data_ptr(), B, H, L,
                           _lib.dtype_code(q.dtype), r[5], lse.data_ptr(), _lib.ptr(_none_if_empty(o32)),
                           st.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(rc, "sisa_attn_fwd")
    backends.after_call(dev)
    return o, lse, o32


@attn_fwd.register_fake
def _(q, k, v, c, b, pos, lam, keep_o32):
    B, H, L, _ = q.shape
    o = torch.empty_strided((B, H, L, D_HEAD), (L * H * D_HEAD, D_HEAD, H * D_HEAD, 1), dtype=q.dtype,
                            device=q.device)
    o32 = q.new_empty((B, H, L, D_HEAD) if keep_o32 else (0,), dtype=torch.float32)
    return o, q.new_empty((B, H, L), dtype=torch.float32), o32


def _attn_bwd_into(q, k, v, c, b, pos, lam, o, do, lse, o32, dq, dk, dv, dF) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """``sisa_attn_bwd`` with dq, dk, dv written into the given views; returns dc, db, dg, dlam."""
    lib = _lib.load()
    B, H, L, _ = q.shape
    dev = q.device
    f32 = dict(device=dev, dtype=torch.float32)
    dc = torch.empty((B, H, L, D_STATE), **f32)
    db = torch.empty((B, H, L, D_STATE), **f32)
    dg = torch.empty((B, H, L), **f32)
    dlam = torch.empty((H,), **f32)
    ws = _bytes(lib.sisa_attn_bwd_workspace(B, H, L), dev)
    st = backends.status_word(dev)
    vs = [_lib.view4(t) for t in (q, k, v, c, b, o, do, dq, dk, dv, dc, db)]
    r = [_lib.vref(x) for x in vs]
    rc = lib.sisa_attn_bwd(r[0], r[1], r[2], r[3], r[4], pos.data_ptr(), lam.data_ptr(), r[5], r[6],
                           lse.data_ptr(), _lib.ptr(_none_if_empty(o32)), B, H, L, _lib.dtype_code(q.dtype),
                           r[7], r[8], r[9], r[10], r[11], dg.data_ptr(), _lib.ptr(dF), dlam.data_ptr(),
                           ws.data_ptr(), st.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(rc, "sisa_attn_bwd")
    return dc, db, dg, dlam


@torch.library.custom_op("sisa_b200::attn_bwd", mutates_args=())
def attn_bwd(q: Tensor, k: Tensor, v: Tensor, c: Tensor, b: Tensor, pos: Tensor, lam: Tensor, o: Tensor,
             do: Tensor, lse: Tensor, o32: Tensor, has_f: bool) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor,
                                                                         Tensor, Tensor, Tensor]:
    """``sisa_attn_bwd`` of the unfused attention: dq, dk, dv (q.dtype), dc, db (fp32), dg, dlam and, with
    ``has_f``, dF (else empty)."""
    B, H, L, _ = q.shape
    dq, dk, dv = (torch.empty((B, H, L, D_HEAD), device=q.device, dtype=q.dtype) for _ in range(3))
    dF = torch.empty((B, H, L), device=q.device, dtype=torch.float32) if has_f else None
    dc, db, dg, dlam = _attn_bwd_into(q, k, v, c, b, pos, lam, o, do, lse, o32, dq, dk, dv, dF)
    backends.after_call(q.device)
    return dq, dk, dv, dc, db, dg, dlam, dF if dF is not None else dg.new_empty(0)


@attn_bwd.register_fake
def _(q, k, v, c, b, pos, lam, o, do, lse, o32, has_f):
    B, H, L, _ = q.shape
    f32 = dict(dtype=torch.float32)
    return (torch.empty_like(q), torch.empty_like(q), torch.empty_like(q), q.new_empty((B, H, L, D_STATE), **f32),
            q.new_empty((B, H, L, D_STATE), **f32), q.new_empty((B, H, L), **f32), q.new_empty((H,), **f32),
            q.new_empty((B, H, L) if has_f else (0,), **f32))


# ------------------------------------------------------------------------------------------------ fused layer
@torch.library.custom_op("sisa_b200::fused_bwd", mutates_args=())
def fused_bwd(proj: Tensor, z: Tensor | None, lam: Tensor, c_rot: Tensor, b_rot: Tensor, pos: Tensor, tot: Tensor,
              o: Tensor, lse: Tensor, o32: Tensor, dy: Tensor, n_head: int) -> tuple[Tensor, Tensor, Tensor]:
    """The fused layer's backward: ``sisa_attn_bwd`` writing dq, dk, dv into the Q/K/V columns of d_proj,
    then ``sisa_prep_bwd`` filling its B, C, theta, alpha and padding columns and dz. Returns d_proj
    (B, L, NPAD) in proj.dtype, dz (B, L, H) fp32 (empty without z) and dlam (H,) fp32."""
    lib = _lib.load()
    H = int(n_head)
    B, L, _ = proj.shape
    dev = proj.device
    off = fused_layout(H)
    dy = dy.contiguous()
    if dy.dtype != proj.dtype:
        dy = dy.to(proj.dtype)
    do = dy.view(B, L, H, D_HEAD).transpose(1, 2)
    dproj = torch.empty_like(proj)
    q, k, v = heads(proj, off["Q"], H, 64), heads(proj, off["K"], H, 64), heads(proj, off["V"], H, 64)
    dq, dk, dv = heads(dproj, off["Q"], H, 64), heads(dproj, off["K"], H, 64), heads(dproj, off["V"], H, 64)
    dF = torch.empty((B, H, L), device=dev, dtype=torch.float32) if z is not None else None
    dc, db, dg, dlam = _attn_bwd_into(q, k, v, c_rot, b_rot, pos, lam, o, do, lse, o32, dq, dk, dv, dF)
    dz = torch.empty((B, L, H), device=dev, dtype=torch.float32) if z is not None else \
        torch.empty(0, device=dev, dtype=torch.float32)
    bt = _bytes(lib.sisa_prep_bwd_workspace(B, H, L), dev)
    st = backends.status_word(dev)
    rc = lib.sisa_prep_bwd(proj.data_ptr(), B, L, H, proj.stride(0), proj.stride(1), _lib.dtype_code(proj.dtype),
                           _lib.ptr(z), z.stride(0) if z is not None else 0, z.stride(1) if z is not None else 0,
                           tot.data_ptr(), dc.data_ptr(), db.data_ptr(), dg.data_ptr(), _lib.ptr(dF),
                           dproj.data_ptr(), dproj.stride(0), dproj.stride(1), _lib.ptr(_none_if_empty(dz)),
                           bt.data_ptr(), st.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(rc, "sisa_prep_bwd")
    backends.after_call(dev)
    return dproj, dz, dlam


@fused_bwd.register_fake
def _(proj, z, lam, c_rot, b_rot, pos, tot, o, lse, o32, dy, n_head):
    B, L, _ = proj.shape
    H = int(n_head)
    return (torch.empty_like(proj), proj.new_empty((B, L, H) if z is not None else (0,), dtype=torch.float32),
            proj.new_empty((H,), dtype=torch.float32))
