"""sm_100a kernels of SISA behind the C ABI of ``libsisa_b200.so`` (mirrors src/sisa/kernels/__init__.py).

``sisa_attention_cuda(q, k, v, c, b, g, lam, fgate=None) -> o``   (:mod:`.attention`)
``sisa_fused(proj, z, lam, n_head) -> y``, ``fused_layout``, ``concat_fused_weights``   (:mod:`.fused`)
``linear_cross_entropy(hidden, weight, labels, ignore_index=-100)``   (:mod:`.linear_ce`)
``decode_attention(...)``   (:mod:`.decode`)

Submodules load on first attribute access.
"""
from __future__ import annotations

import importlib

__all__ = ["sisa_attention_cuda", "sisa_fused", "fused_layout", "concat_fused_weights", "linear_cross_entropy",
           "decode_attention"]

_LAZY = {
    "sisa_attention_cuda": "attention",
    "sisa_fused": "fused",
    "fused_layout": "fused",
    "concat_fused_weights": "fused",
    "linear_cross_entropy": "linear_ce",
    "decode_attention": "decode",
}


def __getattr__(name):
    mod = _LAZY.get(name)
    if mod is None:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    value = getattr(importlib.import_module(f"{__name__}.{mod}"), name)
    globals()[name] = value
    return value


def __dir__():
    return sorted(list(globals()) + list(_LAZY))
