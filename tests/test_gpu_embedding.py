"""The token embedding's weight gradient (``sisa_embedding_bwd``, ``kernels.embedding``) against an fp64
scatter-add of the same gradient rows: repeated ids, one id repeated past the kernel's 2048-entry list
(the list is added and refilled), ids outside the vocabulary, widths that leave threads idle, and the
same bits on a second run."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _fp64_scatter(ids, g, V):
    want = torch.zeros((V, g.shape[1]), dtype=torch.float64)
    keep = (ids >= 0) & (ids < V)
    want.index_add_(0, ids[keep], g[keep].double())
    return want


@pytest.mark.parametrize("n,V,D,hot", [(16384, 50277, 768, 0), (5000, 1000, 12, 4000), (1, 7, 4, 0),
                                       (3000, 600, 1028, 2500)])
def test_embedding_grad_matches_fp64_scatter(cuda_dev, n, V, D, hot):
    from sisa_b200 import _lib

    gen = torch.Generator().manual_seed(n + V)
    ids = torch.randint(0, V, (n,), generator=gen)
    if hot:
        ids[torch.randperm(n, generator=gen)[:hot]] = V // 3          # one id far past the list size
    ids[::97] = -1                                                   # outside the vocabulary: no row
    ids[5::101] = V + 3
    g = torch.randn((n, D), generator=gen)
    dw = torch.full((V, D), float("nan"), device=cuda_dev)           # every row must be written
    gd, idd = g.to(cuda_dev), ids.to(cuda_dev)
    for run in range(2):
        _lib.check(_lib.load().sisa_embedding_bwd(idd.data_ptr(), n, gd.data_ptr(), D, dw.data_ptr(), V, D,
                                                  _lib.stream_ptr(cuda_dev)), "sisa_embedding_bwd")
        torch.cuda.synchronize()
        if run == 0:
            first = dw.clone()
    assert torch.equal(dw, first)
    want = _fp64_scatter(ids, g, V)
    mag = torch.zeros((V, D), dtype=torch.float64).index_add_(0, ids.clamp(0, V - 1), g.double().abs())
    err = (dw.cpu().double() - want).abs()
    assert bool((err <= 1e-6 * mag + 1e-30).all()), float(err.max())


def test_model_embedding_grad_equals_torch(cuda_dev):
    """kernels.embedding: the forward is F.embedding's lookup bit for bit, and the weight gradient
    equals torch's embedding backward to fp32 summation order."""
    from sisa_b200.kernels.embedding import embedding

    gen = torch.Generator().manual_seed(3)
    w = torch.randn((5000, 64), generator=gen).to(cuda_dev).requires_grad_()
    w2 = w.detach().clone().requires_grad_()
    ids = torch.randint(0, 5000, (4, 1024), generator=gen).to(cuda_dev)
    up = torch.randn((4, 1024, 64), generator=gen).to(cuda_dev)
    y = embedding(ids, w)
    y2 = torch.nn.functional.embedding(ids, w2)
    assert torch.equal(y, y2)
    (y * up).sum().backward()
    (y2 * up).sum().backward()
    assert torch.allclose(w.grad, w2.grad, rtol=0, atol=1e-5)
