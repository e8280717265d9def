"""AdamW with global-norm gradient clipping over flat fp32 buffers (``sisa_adamw_flat``).

The training step's ``clip_grad_norm_`` + ``torch.optim.AdamW`` (the reference's
examples/train_minimal.py:253-301) as two kernels over one contiguous layout of every parameter, its
gradient and its two moments, instead of per-tensor launches. The layout is the one of
:class:`sisa_b200.dp.GradBuckets` (each parameter at a 4-element-aligned offset); the parameters
themselves become views of the flat buffer. The step counter lives on the device, so the update can be
captured in a CUDA graph; learning rates and weight decays come from the parameter groups and are
copied to the device when they change.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _lib, backends

__all__ = ["FlatAdamW", "TensorAdamW"]

_SEG = np.dtype([("start", "<i8"), ("end", "<i8"), ("lr", "<f4"), ("weight_decay", "<f4")])
NPART = 592      # fixed grid of the norm pass, 4 blocks per SM (fixed-order partial sums: a deterministic norm)


class FlatAdamW:
    """AdamW over parameters laid out by ``layout`` (a :class:`~sisa_b200.dp.GradBuckets`), with
    ``param_groups`` in the reference's form (``{"params", "lr", "weight_decay"}``). ``step()`` clips
    the gradients to a global norm of ``max_norm`` (0 disables it) and applies one AdamW step."""

    def __init__(self, param_groups, layout, *, betas=(0.9, 0.95), eps: float = 1e-8, max_norm: float = 1.0):
        self.layout = layout
        self.param_groups = [dict(g) for g in param_groups]
        for g in self.param_groups:
            g["params"] = list(g["params"])
            g.setdefault("betas", betas)
            g.setdefault("eps", eps)
        self.betas = (float(betas[0]), float(betas[1]))
        self.eps = float(eps)
        self.max_norm = float(max_norm)
        dev = layout.buffer.device
        n = layout.buffer.numel()
        # the parameters become views of one fp32 buffer with the gradients' layout
        self.params = torch.zeros(n, dtype=torch.float32, device=dev)
        with torch.no_grad():
            for p in layout.order:
                off, cnt = layout.offset[id(p)]
                self.params[off:off + cnt].copy_(p.data.reshape(-1))
                p.data = self.params[off:off + cnt].view_as(p)
        self.m = torch.zeros(n, dtype=torch.float32, device=dev)
        self.v = torch.zeros(n, dtype=torch.float32, device=dev)
        self.step_count = torch.zeros(1, dtype=torch.float32, device=dev)
        self.partials = torch.empty(NPART, dtype=torch.float64, device=dev)
        self._group_of = {id(p): gi for gi, g in enumerate(self.param_groups) for p in g["params"]}
        missing = [p for p in layout.order if id(p) not in self._group_of]
        if missing:
            raise ValueError(f"{len(missing)} parameters of the layout belong to no parameter group")
        self._segs = None
        self._seg_key = None

    def _segments(self) -> torch.Tensor:
        key = tuple((float(g["lr"]), float(g["weight_decay"])) for g in self.param_groups)
        if key != self._seg_key:
            rows = []
            for p in self.layout.order:
                off, cnt = self.layout.offset[id(p)]
                lr, wd = key[self._group_of[id(p)]]
                end = off + -(-cnt // 4) * 4
                if rows and rows[-1][1] == off and rows[-1][2] == lr and rows[-1][3] == wd:
                    rows[-1] = (rows[-1][0], end, lr, wd)
                else:
                    rows.append((off, end, lr, wd))
            arr = np.array(rows, dtype=_SEG)
            host = torch.from_numpy(arr.view(np.uint8).copy())
            if self._segs is None or self._segs.numel() != host.numel():
                self._segs = torch.empty(host.numel(), dtype=torch.uint8, device=self.params.device)
            self._segs.copy_(host, non_blocking=False)
            self._nseg = len(rows)
            self._seg_key = key
        return self._segs

    def zero_grad(self, set_to_none: bool = False) -> None:
        self.layout.buffer.zero_()

    @torch.no_grad()
    def step(self) -> None:
        dev = self.params.device
        segs = self._segments()
        b1, b2 = self.betas
        _lib.check(_lib.load().sisa_adamw_flat(self.params.data_ptr(), self.layout.buffer.data_ptr(),
                                               self.m.data_ptr(), self.v.data_ptr(), self.params.numel(),
                                               segs.data_ptr(), self._nseg, self.step_count.data_ptr(),
                                               self.partials.data_ptr(), NPART, b1, b2, self.eps, self.max_norm,
                                               backends.status_word(dev).data_ptr(), _lib.stream_ptr(dev)),
                   "sisa_adamw_flat")
        backends.after_call(dev)
        # the kernel wrote the parameters behind autograd's back: mark them modified, so that the
        # weight copies kept per version (projection, MLP, W_O / w_down) are rebuilt
        for p in self.layout.order:
            torch.autograd.graph.increment_version(p)


class TensorAdamW:
    """The same clipping and AdamW (``sisa_adamw_tensors``) over the parameters as they are: gradients
    stay the tensors autograd hands over, and only the moments live in flat buffers (each parameter at a
    4-element-aligned offset). Parameters without a gradient are left alone and out of the norm, as in
    ``clip_grad_norm_`` + ``torch.optim.AdamW``. The learning rates and weight decays are read from
    ``param_groups`` at every step; a captured CUDA graph replays the values of its capture.

    One step counter serves all parameters (torch keeps one per parameter; they differ only for
    parameters that miss steps)."""

    MAX_TENSORS = 384

    def __init__(self, param_groups, *, betas=(0.9, 0.95), eps: float = 1e-8, max_norm: float = 1.0):
        self.param_groups = [dict(g) for g in param_groups]
        for g in self.param_groups:
            g["params"] = list(g["params"])
            g.setdefault("betas", betas)
            g.setdefault("eps", eps)
        self.params = [p for g in self.param_groups for p in g["params"]]
        if len(self.params) > self.MAX_TENSORS:
            raise ValueError(f"TensorAdamW takes at most {self.MAX_TENSORS} parameter tensors, got {len(self.params)}")
        if not self.params or any(not p.is_cuda or p.dtype != torch.float32 for p in self.params):
            raise ValueError("TensorAdamW needs fp32 CUDA parameters")
        self.betas = (float(betas[0]), float(betas[1]))
        self.eps = float(eps)
        self.max_norm = float(max_norm)
        dev = self.params[0].device
        self.offset, off = [], 0
        for p in self.params:
            self.offset.append(off)
            off += -(-p.numel() // 4) * 4
        if len({id(p) for p in self.params}) != len(self.params):
            raise ValueError("a parameter appears in more than one group")
        self._index = {id(p): k for k, p in enumerate(self.params)}
        self.m = torch.zeros(off, dtype=torch.float32, device=dev)
        self.v = torch.zeros(off, dtype=torch.float32, device=dev)
        self.step_count = torch.zeros(1, dtype=torch.float32, device=dev)
        self.partials = torch.empty(NPART, dtype=torch.float64, device=dev)
        self._table = (_lib.AdamTensor * len(self.params))()

    def zero_grad(self, set_to_none: bool = True) -> None:
        for p in self.params:
            if set_to_none:
                p.grad = None
            elif p.grad is not None:
                p.grad.zero_()

    @torch.no_grad()
    def step(self) -> None:
        n = 0
        for g in self.param_groups:
            lr, wd = float(g["lr"]), float(g["weight_decay"])
            for p in g["params"]:
                if p.grad is None:
                    continue
                if p.grad.dtype != torch.float32 or not p.grad.is_contiguous():
                    raise ValueError("TensorAdamW needs contiguous fp32 gradients")
                k = self._index[id(p)]
                e = self._table[n]
                e.param, e.grad = p.data_ptr(), p.grad.data_ptr()
                e.offset, e.n, e.lr, e.weight_decay = self.offset[k], p.numel(), lr, wd
                n += 1
        if n == 0:
            return
        dev = self.m.device
        b1, b2 = self.betas
        _lib.check(_lib.load().sisa_adamw_tensors(self._table, n, self.m.data_ptr(), self.v.data_ptr(),
                                                  self.m.numel(), self.step_count.data_ptr(),
                                                  self.partials.data_ptr(), NPART, b1, b2, self.eps, self.max_norm,
                                                  backends.status_word(dev).data_ptr(), _lib.stream_ptr(dev)),
                   "sisa_adamw_tensors")
        backends.after_call(dev)
        torch.autograd.graph.increment_version([p for p in self.params if p.grad is not None])
