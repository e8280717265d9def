"""Incremental-decode attention on the sm_100a kernel (mirrors the decode step of src/sisa/modeling.py:224-238).

``decode_attention(q, c, g, fgate, state, lam) -> y``: one new query row per (batch, head) against the
layer's cache (:class:`sisa_b200.generation.LayerState`, which already holds the new position). fp32
scores and softmax over the bf16/fp16 cache, split-K over the key axis.

When the state carries a device position counter (``state.pos_dev``, set by
:class:`sisa_b200.generation.DecodeGraph`), both calls take the position from that int32 on the device
(``sisa_decode_prep_dpos`` / ``sisa_decode_attn_dpos``), so that one captured CUDA graph of the step serves
every position; the host-side ``state.length`` is still advanced for bookkeeping.
"""
from __future__ import annotations

import torch

from .. import _lib, backends

__all__ = ["decode_attention", "decode_prep"]


def decode_attention(q: torch.Tensor, c: torch.Tensor, g: torch.Tensor, fgate: torch.Tensor | None, state,
                     lam: torch.Tensor) -> torch.Tensor:
    """q: (B, H, 1, 64), c: (B, H, 1, 32) compute dtype; g, fgate: (B, H, 1) fp32; lam: (H,) fp32.
    Returns y (B, H, 1, 64) in q.dtype."""
    lib = _lib.load()
    B, H, M, D = q.shape
    if M != 1 or D != 64 or c.shape[-1] != 32:
        raise ValueError(f"decode_attention takes one query row with d_head 64 and d_state 32, got {tuple(q.shape)}")
    dev = q.device
    pos_dev = getattr(state, "pos_dev", None)
    N = state.capacity if pos_dev is not None else state.length
    if c.dtype != q.dtype:
        c = c.to(q.dtype)
    q, c = (t if t.stride(-1) == 1 and t.data_ptr() % 16 == 0 else t.contiguous() for t in (q, c))
    gq = g.reshape(B, H).float().contiguous()
    fq = None if fgate is None else fgate.reshape(B, H).float().contiguous()
    y = torch.empty((B, H, 1, D), device=dev, dtype=q.dtype)
    ws = torch.empty(max(lib.sisa_decode_workspace(B, H, N), 16), dtype=torch.uint8, device=dev)
    st = backends.status_word(dev)
    vs = [_lib.view4(t) for t in (q, c, state.k_buf, state.v_buf, state.b_buf, y)]
    r = [_lib.vref(x) for x in vs]
    fc = None if fq is None else state.f_buf.data_ptr()
    lam_p = lam.float().contiguous().data_ptr()
    if pos_dev is not None:
        rc = lib.sisa_decode_attn_dpos(r[0], r[1], gq.data_ptr(), _lib.ptr(fq), r[2], r[3], r[4],
                                       state.g_buf.data_ptr(), fc, state.g_buf.shape[2], lam_p, B, H,
                                       pos_dev.data_ptr(), N, _lib.dtype_code(q.dtype), r[5], ws.data_ptr(),
                                       st.data_ptr(), _lib.stream_ptr(dev))
        _lib.check(rc, "sisa_decode_attn_dpos")
    else:
        rc = lib.sisa_decode_attn(r[0], r[1], gq.data_ptr(), _lib.ptr(fq), r[2], r[3], r[4], state.g_buf.data_ptr(),
                                  fc, state.g_buf.shape[2], lam_p, B, H, N, _lib.dtype_code(q.dtype), r[5],
                                  ws.data_ptr(), st.data_ptr(), _lib.stream_ptr(dev))
        _lib.check(rc, "sisa_decode_attn")
    backends.after_call(dev)
    return y


def decode_prep(proj: torch.Tensor, z: torch.Tensor | None, state, n_head: int):
    """One decode step's layer input on the sm_100a kernel: from the new token's fused projection row
    ``proj`` (B, 1, NPAD) and forget logits ``z`` (B, 1, H) fp32, continue the g / F / Phi recurrences
    from ``state`` (generation.py:58-95), rotate c and b, and append k, v, b~, g, F to the cache.
    Returns q (a view of proj's Q columns), c~ (B, H, 1, 32), g and F (B, H, 1) fp32, as
    :func:`decode_attention` takes them; the state then holds the new position."""
    lib = _lib.load()
    B, H = proj.shape[0], n_head
    proj2 = proj.reshape(B, proj.shape[-1])
    if proj2.stride(-1) != 1 or proj2.stride(0) % 2:
        proj2 = proj2.contiguous()
    if proj2.dtype != state.k_buf.dtype:
        raise TypeError(f"decode_prep: projection dtype {proj2.dtype} differs from the cache's {state.k_buf.dtype}")
    dev = proj.device
    pos_dev = getattr(state, "pos_dev", None)
    if pos_dev is not None:
        if state.length + 1 > state.capacity:      # a reallocation would leave a captured graph's pointers stale
            raise ValueError(f"decode_prep: the cache holds {state.capacity} positions and is full")
    else:
        state.reserve(1)
    phi = state.phi_buffer()
    pos = state.length
    c = torch.empty((B, H, 1, 32), dtype=proj2.dtype, device=dev)
    g = torch.empty((B, H, 1), dtype=torch.float32, device=dev)
    f = None
    z2 = None
    if z is not None:
        z2 = z.reshape(B, H).float().contiguous()
        f = torch.empty((B, H, 1), dtype=torch.float32, device=dev)
    vk, vv, vb = (_lib.view4(t) for t in (state.k_buf, state.v_buf, state.b_buf))
    st = backends.status_word(dev)
    args = (proj2.data_ptr(), proj2.stride(0), _lib.ptr(z2), 0 if z2 is None else z2.stride(0), B, H,
            _lib.dtype_code(proj2.dtype), _lib.vref(vk), _lib.vref(vv), _lib.vref(vb),
            state.g_buf.data_ptr(), None if z2 is None else state.f_buf.data_ptr(), state.g_buf.shape[2])
    outs = (phi.data_ptr(), c.data_ptr(), g.data_ptr(), _lib.ptr(f), st.data_ptr(), _lib.stream_ptr(dev))
    if pos_dev is not None:
        rc = lib.sisa_decode_prep_dpos(*args, pos_dev.data_ptr(), state.capacity, *outs)
        _lib.check(rc, "sisa_decode_prep_dpos")
    else:
        rc = lib.sisa_decode_prep(*args, pos, *outs)
        _lib.check(rc, "sisa_decode_prep")
    backends.after_call(dev)
    state.length = pos + 1
    q = proj2[:, :H * 64].view(B, H, 64).unsqueeze(2)
    return q, c, g, f
