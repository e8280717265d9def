"""The compute-dtype copies of a model's fp32 weights, refreshed in one launch (``sisa_copy_rows``).

Under autocast the reference casts every weight to the compute dtype on every forward
(src/sisa/modeling.py:39-49,213-222). Here the fused linears keep those copies on their modules (the
projection's concatenation in kernels/fused.py, the interleaved gate/up weight in kernels/ffn.py, W_O and
w_down in kernels/linear.py), keyed on their weights' storage, version and dtype. :func:`refresh`
writes the copies of all blocks with one kernel, where the lookups would otherwise cast each weight
with its own small launches (about a dozen per block), and marks them fresh for the lookups of this
forward:

- with gradients (a training forward) it rewrites every copy: fused optimizers (torch's
  ``AdamW(fused=True)``, the reference's choice) change the weights in place without advancing their
  versions, so a version key cannot tell a stale copy there, and a lookup uses only a copy marked fresh;
- without gradients it rewrites only the copies whose keys changed, and the keys decide.

A copy that the refresh does not cover (other dtypes, weights that are not fp32 CUDA tensors) is built
by its lookup.

The copies are rewritten in place: an autograd graph recorded before an optimizer step must have run
its backward before the next forward (as in every training loop). The job table (source and
destination pointers) is kept on the device while it stays the same, so a captured CUDA graph replays
the launch; a table that changes while a capture is running is not uploaded, and the lookups then
build their copies as before.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch
from torch import Tensor

from .. import _lib, backends

__all__ = ["refresh"]

_JOB = np.dtype([("src", "<u8"), ("dst", "<u8"), ("rows", "<i8"), ("cols", "<i8"), ("src_ld", "<i8"),
                 ("dst_ld", "<i8"), ("block_rows", "<i8"), ("dst_block_stride", "<i8")])


def _fp32_rows(w: Tensor) -> bool:
    return (w.is_cuda and w.dtype == torch.float32 and w.dim() == 2 and w.is_contiguous()
            and w.shape[1] % 8 == 0 and w.data_ptr() % 16 == 0)


class _Plan:
    def __init__(self, dtype: torch.dtype):
        self.dtype = dtype
        self.jobs: list[tuple] = []
        self.updates: list[tuple] = []          # (owner, slot, key, tensor)

    def copy(self, src: Tensor | None, dst: Tensor, rows: int, cols: int, block_rows: int = 0,
             dst_block_stride: int = 0) -> None:
        self.jobs.append((0 if src is None else src.data_ptr(), dst.data_ptr(), rows, cols,
                          cols if src is None else src.stride(0), dst.stride(0), block_rows or max(rows, 1),
                          dst_block_stride))


def _dest(owner, slot: str, shape: tuple, dtype: torch.dtype, device) -> Tensor:
    """The copy kept under ``slot`` when its shape, dtype and device still fit (rewritten in place), else
    a new tensor."""
    hit = owner.__dict__.get(slot)
    if hit is not None:
        t = hit[1]
        if tuple(t.shape) == tuple(shape) and t.dtype == dtype and t.device == device and t.is_contiguous():
            return t
    return torch.empty(shape, dtype=dtype, device=device)


def _stale(owner, slot: str, key: tuple) -> bool:
    hit = owner.__dict__.get(slot)
    return torch.is_grad_enabled() or hit is None or hit[0] != key


def _plan_block(plan: _Plan, attn, ffn) -> None:
    from .ffn import BLOCK, gate_up_key
    from .fused import fused_layout, wcat_key
    from .linear import weight_key

    dt = plan.dtype
    # the projection's concatenation (zero rows up to NPAD)
    ws = attn.projection_weights()
    if all(_fp32_rows(w) for w in ws):
        key = wcat_key(ws, dt)
        if _stale(attn, "_wcat_train", key):
            off = fused_layout(ws[-1].shape[0])
            d = ws[0].shape[1]
            dst = _dest(attn, "_wcat_train", (off["NPAD"], d), dt, ws[0].device)
            row = 0
            for w in ws:
                plan.copy(w, dst[row:row + w.shape[0]], w.shape[0], d)
                row += w.shape[0]
            if row < off["NPAD"]:
                # every time, so that the table stays the same from step to step
                plan.copy(None, dst[row:], off["NPAD"] - row, d)
            plan.updates.append((attn, "_wcat_train", key, dst))
    # W_O and w_down
    for owner, name, w in ((attn, "W_O", attn.W_O.weight), (ffn, "w_down", ffn.w_down.weight)):
        if _fp32_rows(w):
            key = weight_key(w, dt)
            if _stale(owner, "_lp_" + name, key):
                dst = _dest(owner, "_lp_" + name, tuple(w.shape), dt, w.device)
                plan.copy(w, dst, w.shape[0], w.shape[1])
                plan.updates.append((owner, "_lp_" + name, key, dst))
    # the gate and up weights interleaved in blocks of BLOCK rows
    wg, wu = ffn.w_gate.weight, ffn.w_up.weight
    if _fp32_rows(wg) and _fp32_rows(wu) and wg.shape == wu.shape and wg.shape[0] % BLOCK == 0:
        key = gate_up_key(wg, wu, dt)
        if _stale(ffn, "_gate_up_il", key):
            d_ff, d = wg.shape
            dst = _dest(ffn, "_gate_up_il", (2 * d_ff, d), dt, wg.device)
            plan.copy(wg, dst, d_ff, d, BLOCK, 2 * BLOCK)
            plan.copy(wu, dst[BLOCK:], d_ff, d, BLOCK, 2 * BLOCK)
            plan.updates.append((ffn, "_gate_up_il", key, dst))


def refresh(model, dtype: torch.dtype) -> int:
    """Write the compute-dtype weight copies of ``model``'s blocks in one launch (all of them when
    gradients are enabled, else the stale ones), record their keys and mark them fresh. Returns the
    number of row-block copies launched (0 when nothing was due or the table could not be used)."""
    if dtype not in (torch.bfloat16, torch.float16) or not len(model.layers):
        return 0
    plan = _Plan(dtype)
    for layer in model.layers:
        _plan_block(plan, layer.attn, layer.ffn)
    if not plan.jobs:
        return 0
    dev = model.layers[0].attn.W_O.weight.device
    lib = _lib.load()
    host = np.array(plan.jobs, dtype=_JOB)
    raw = host.tobytes()
    kept = model.__dict__.get("_weight_copy_table")
    if kept is None or kept[0] != raw:
        if torch.cuda.is_current_stream_capturing():
            return 0
        for i in range(len(host)):
            job = _lib.RowCopy.from_buffer_copy(host[i].tobytes())
            _lib.check(lib.sisa_row_copy_check(ctypes.byref(job)), "sisa_row_copy_check")
        table = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(dev)
        kept = (raw, table)
        model.__dict__["_weight_copy_table"] = kept
    max_vec = int((host["rows"] * host["cols"]).max()) // 8
    _lib.check(lib.sisa_copy_rows(kept[1].data_ptr(), len(host), max_vec, _lib.dtype_code(dtype),
                                  backends.status_word(dev).data_ptr(), _lib.stream_ptr(dev)), "sisa_copy_rows")
    for owner, slot, key, t in plan.updates:
        owner.__dict__[slot] = (key, t, True)
    return len(host)
