"""The token embedding with its weight gradient on ``sisa_embedding_bwd``.

The reference's model looks tokens up with ``nn.Embedding`` (src/sisa/modeling.py), whose backward torch
computes by sorting the ids and summing segments over several launches. Here the forward is the same
lookup and the backward is one deterministic launch that writes the whole (V, D) weight gradient: each
block of the kernel owns a range of vocabulary rows and adds the matching gradient rows in position
order. The kernel scans every id once per block, so batches above ``EMBED_MAX_IDS`` tokens keep torch's
backward.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import Tensor

from .. import _lib

__all__ = ["embedding", "EMBED_MAX_IDS"]

EMBED_MAX_IDS = 262144      # SISA_EMBED_MAX_IDS of the C ABI


class _EmbeddingFn(torch.autograd.Function):
    """``F.embedding(ids, weight)``; the weight gradient from ``sisa_embedding_bwd``."""

    @staticmethod
    def forward(ctx, ids, weight):
        ctx.save_for_backward(ids)
        ctx.shape = weight.shape
        return F.embedding(ids, weight)

    @staticmethod
    def backward(ctx, g):
        (ids,) = ctx.saved_tensors
        V, D = ctx.shape
        g2 = g.reshape(-1, D)
        if g2.dtype != torch.float32:
            g2 = g2.float()
        if g2.stride(-1) != 1 or g2.stride(0) % 4 or g2.data_ptr() % 16:
            g2 = g2.contiguous()
        ids1 = ids.reshape(-1).contiguous()
        dw = torch.empty((V, D), dtype=torch.float32, device=g.device)
        _lib.check(_lib.load().sisa_embedding_bwd(ids1.data_ptr(), ids1.numel(), g2.data_ptr(), g2.stride(0),
                                                  dw.data_ptr(), V, D, _lib.stream_ptr(g.device)),
                   "sisa_embedding_bwd")
        return None, dw


def embedding(ids: Tensor, weight: Tensor) -> Tensor:
    """``F.embedding(ids, weight)``, with the weight gradient on ``sisa_embedding_bwd`` for an fp32 CUDA
    weight that needs one (D a multiple of 4, int64 ids, at most ``EMBED_MAX_IDS`` of them)."""
    if (weight.is_cuda and weight.dtype == torch.float32 and weight.requires_grad and torch.is_grad_enabled()
            and ids.dtype == torch.int64 and ids.numel() <= EMBED_MAX_IDS and weight.shape[1] % 4 == 0):
        return _EmbeddingFn.apply(ids, weight)
    return F.embedding(ids, weight)
