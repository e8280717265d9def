"""Implementation selection, device checks and the run-time check mode (mirrors src/sisa/backends.py).

Two implementations of SISA attention exist in this package:

* ``"torch"``: exact blocked attention in plain PyTorch (any device and dtype).
* ``"cuda"``: the hand-written sm_100a kernels of ``libsisa_b200.so`` (fused preparation, tcgen05
  attention forward/backward). At the layer level it is the fused path (one projection GEMM, then
  the preparation and attention kernels); ``"triton"`` and ``"triton_fused"`` are aliases.

``"auto"`` picks ``"cuda"`` for CUDA inputs on an sm_100 GPU with d_head 64, d_state 32 and a
bf16/fp16 compute dtype, else ``"torch"`` (with a one-time warning on CUDA). Forcing ``"cuda"`` on an
input it cannot take raises ``ValueError``; the CUDA path never falls back to anything.

Check mode (src/sisa/backends.py:65-94): the kernels OR condition bits into a device status word
instead of asserting. ``"sync"`` reads the word after each call and raises right away
(``ValueError`` for a non-monotone decay, ``FloatingPointError`` for non-finite values,
``RuntimeError`` for a device wait that timed out). ``"async"`` (default) never synchronises;
:func:`check_status` reads and clears the word and raises the same exceptions. ``"off"`` skips the
host-side reads.
"""
from __future__ import annotations

import threading
import warnings
from typing import TYPE_CHECKING

import torch

from . import _lib
from .config import CUDA_ALIASES, CUDA_D_HEAD, CUDA_D_STATE

if TYPE_CHECKING:  # pragma: no cover
    from .config import SISAConfig

__all__ = ["IMPLS", "cuda_status", "fused_eligible", "set_check_mode", "get_check_mode", "check_status",
           "status_word", "describe", "select_impl", "device_info"]

IMPLS = ("auto", "torch", "cuda", "triton", "triton_fused")
_CHECK_MODES = ("async", "sync", "off")
_STATE = {"check": "async"}
_LOCK = threading.Lock()
_STATUS: dict[int, torch.Tensor] = {}
_CUDA_STATUS: dict[int, tuple[bool, str]] = {}
_WARNED: set = set()

_GUARD_MSG = ("SISA cuda kernels: non-finite input (NaN/inf in q/k/c/b/lambda/g/F, i.e. in a parameter such as "
              "alpha_proj, theta_proj, forget_proj, W_Q or lambda_raw)")


def set_check_mode(mode: str) -> None:
    """``"async"`` (default), ``"sync"`` or ``"off"``; see the module docstring."""
    if mode not in _CHECK_MODES:
        raise ValueError(f"check mode must be one of {_CHECK_MODES}, got {mode!r}")
    _STATE["check"] = mode


def get_check_mode() -> str:
    return _STATE["check"]


def status_word(device: torch.device) -> torch.Tensor:
    """The per-device int32 status word the kernels OR their condition bits into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _STATUS.get(idx)
    if t is None:
        with _LOCK:
            t = _STATUS.get(idx)
            if t is None:
                t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
                _STATUS[idx] = t
    return t


def _raise_for(bits: int) -> None:
    if bits & _lib.ST_TIMEOUT:
        raise RuntimeError("SISA cuda kernels: a bounded device wait timed out; results are invalid")
    if bits & _lib.ST_NONMONOTONE:
        raise ValueError("g must be non-increasing along the sequence (max increase > 1e-3)")
    if bits & _lib.ST_NONFINITE:
        raise FloatingPointError(_GUARD_MSG)
    if bits & _lib.ST_BAD_SEED:
        raise RuntimeError("linear_cross_entropy: backward seed differs from the promised grad_scale")
    if bits & _lib.ST_BAD_POS:
        raise ValueError("decode: the device position lay outside the cache; the step wrote nothing")


def check_status(device: torch.device | int | None = None) -> None:
    """Read and clear the status word of ``device`` (synchronises) and raise for any bit set."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else torch.device(device).index or 0))
    st = status_word(dev)
    bits = int(st.item())
    if bits:
        st.zero_()
        _raise_for(bits)


def after_call(device: torch.device) -> None:
    """Called after each kernel entry point: raises right away in ``"sync"`` mode."""
    if _STATE["check"] == "sync":
        check_status(device)


def device_info(device=None) -> dict:
    idx = device if isinstance(device, int) else (torch.cuda.current_device() if device is None
                                                  else (torch.device(device).index or 0))
    p = torch.cuda.get_device_properties(idx)
    return dict(index=idx, name=p.name, capability=(p.major, p.minor), sm_count=int(p.multi_processor_count),
                total_memory=int(p.total_memory))


def cuda_status(device=None) -> tuple[bool, str]:
    """Whether the sm_100a kernels can run on ``device``: ``(True, summary)`` or ``(False, why_not)``."""
    if not torch.cuda.is_available():
        return False, "CUDA is not available"
    idx = device if isinstance(device, int) else (torch.cuda.current_device() if device is None
                                                  else (torch.device(device).index or 0))
    hit = _CUDA_STATUS.get(idx)
    if hit is not None:
        return hit
    try:
        lib = _lib.load()
    except (RuntimeError, OSError) as e:
        res = (False, str(e))
    else:
        rc = lib.sisa_device_check(idx)
        res = (True, f"{lib.sisa_version().decode()} on {torch.cuda.get_device_name(idx)}") if rc == 0 else \
              (False, _lib.last_error())
    _CUDA_STATUS[idx] = res
    return res


def _compute_dtype(x: torch.Tensor) -> torch.dtype:
    dt = x.device.type
    try:
        if torch.is_autocast_enabled(dt):
            return torch.get_autocast_dtype(dt)
    except (TypeError, RuntimeError):
        pass
    return x.dtype


def fused_eligible(x: torch.Tensor) -> bool:
    if not isinstance(x, torch.Tensor) or x.device.type != "cuda":
        return False
    if _compute_dtype(x) not in (torch.bfloat16, torch.float16):
        return False
    return cuda_status(x.device)[0]


def _shape_problem(cfg) -> str | None:
    if cfg is None:
        return None
    d_head = cfg.d_model // cfg.n_head
    if d_head != CUDA_D_HEAD or cfg.d_state != CUDA_D_STATE:
        return (f"the cuda kernels need d_head == {CUDA_D_HEAD} and d_state == {CUDA_D_STATE} "
                f"(got d_head={d_head}, d_state={cfg.d_state})")
    return None


def select_impl(requested: str, x: torch.Tensor, cfg: "SISAConfig | None") -> str:
    """Resolve ``requested`` to ``"torch"`` or ``"cuda"`` for layer input ``x`` (src/sisa/backends.py:284-336)."""
    if requested not in IMPLS:
        raise ValueError(f"attn_impl must be one of {IMPLS}, got {requested!r}")
    if requested == "torch":
        return "torch"
    on_cuda = isinstance(x, torch.Tensor) and x.device.type == "cuda"
    if on_cuda:
        ok, why = cuda_status(x.device)
    else:
        ok, why = False, f"input is on {x.device.type if isinstance(x, torch.Tensor) else type(x).__name__}, not CUDA"
    shape = _shape_problem(cfg)
    cdt = _compute_dtype(x) if isinstance(x, torch.Tensor) else None
    dtype_ok = cdt in (torch.bfloat16, torch.float16)
    if requested in CUDA_ALIASES:
        if not ok:
            raise ValueError(f"attn_impl={requested!r} is not available: {why}")
        if shape:
            raise ValueError(f"attn_impl={requested!r} is not available: {shape}")
        if not dtype_ok:
            raise ValueError(f"attn_impl={requested!r} needs a bf16/fp16 compute dtype (enable autocast or use "
                             f"low-precision parameters); got {cdt}")
        return "cuda"
    if ok and not shape and dtype_ok:
        return "cuda"
    if on_cuda:
        reason = why if not ok else (shape or f"compute dtype {cdt}")
        key = (x.device.index, reason)
        if key not in _WARNED:
            _WARNED.add(key)
            warnings.warn(f"SISA: using the torch attention implementation on CUDA because {reason}", stacklevel=2)
    return "torch"


def describe() -> str:
    lines = [f"torch {torch.__version__} (CUDA {torch.version.cuda})", f"check mode: {get_check_mode()}"]
    if not torch.cuda.is_available():
        lines.append("CUDA: not available -> attn_impl='auto' uses 'torch'")
        return "\n".join(lines)
    for idx in range(torch.cuda.device_count()):
        ok, why = cuda_status(idx)
        lines.append(f"cuda:{idx} {torch.cuda.get_device_name(idx)}: cuda kernels "
                     f"{'available' if ok else 'unavailable'} - {why}")
    return "\n".join(lines)
