"""sisa_b200: B200-native (sm_100a) implementation of SISA's training and inference hot path.

SISA (SSM-Informed Softmax Attention, tlstngud/sisa) scores query i against key j <= i with
``s_ij = q_i.k_j/sqrt(d) + lam_h exp(g_i - g_j)(C~_i.B~_j) + (F_i - F_j)``. This package keeps the
reference's public API (``SISAConfig``, ``SISAAttention``, ``SISABlock``, ``SISAForCausalLM``,
``sisa_attention``, ``backends``, ``generate``) and adds the ``"cuda"`` implementation: hand-written
sm_100a kernels (fused preparation scans, tcgen05 attention forward/backward, fused linear +
cross-entropy, incremental decode) behind the C ABI of ``libsisa_b200.so``.
"""
from __future__ import annotations

import importlib
from typing import Any

from .config import PRESETS, SISAConfig

__version__ = "0.1.0"

__all__ = ["SISAConfig", "PRESETS", "SISAAttention", "SISABlock", "SISAModel", "SISAForCausalLM", "SISAOutput",
           "sisa_attention", "load_paper_checkpoint", "convert_state_dict", "set_check_mode", "__version__"]

_LAZY_ATTRS = {
    "SISAAttention": "modeling", "SISABlock": "modeling", "SISAModel": "modeling",
    "SISAForCausalLM": "modeling", "SISAOutput": "modeling", "sisa_attention": "functional",
    "load_paper_checkpoint": "checkpoint", "convert_state_dict": "checkpoint",
}
_LAZY_SUBMODULES = ("backends", "kernels", "generation", "functional", "modeling", "checkpoint")


def set_check_mode(mode: str) -> None:
    """``"async"`` (default), ``"sync"`` or ``"off"``; see :func:`sisa_b200.backends.set_check_mode`."""
    from .backends import set_check_mode as _set

    _set(mode)


def __getattr__(name: str) -> Any:
    if name in _LAZY_ATTRS:
        value = getattr(importlib.import_module(f".{_LAZY_ATTRS[name]}", __name__), name)
        globals()[name] = value
        return value
    if name in _LAZY_SUBMODULES:
        return importlib.import_module(f".{name}", __name__)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
