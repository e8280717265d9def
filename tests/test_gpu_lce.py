"""Chunked linear + cross-entropy (tcgen05 logits kernel + gradient kernel) against fp64 and the eager
autocast formula, through the C ABI."""
from __future__ import annotations

import pytest
import torch

from oracle import sisa_oracle as O
from tests.helpers import GRAD_REL, rel_err

pytestmark = pytest.mark.gpu


def make_case(N, D, V, seed, n_ignore=5):
    gen = torch.Generator().manual_seed(seed)
    h = torch.randn(N, D, generator=gen).to(torch.bfloat16)
    w = torch.randn(V, D, generator=gen) * 0.02
    labels = torch.randint(0, V, (N,), generator=gen)
    if n_ignore:
        labels[torch.randperm(N, generator=gen)[:n_ignore]] = -100
    return h, w, labels


def run(h, w, labels, dev, **kw):
    from sisa_b200.kernels.linear_ce import linear_cross_entropy

    H = h.to(dev).requires_grad_(True)
    W = w.to(dev).requires_grad_(True)
    loss = linear_cross_entropy(H, W, labels.to(dev), **kw)
    loss.backward()
    torch.cuda.synchronize()
    return loss.detach().cpu(), H.grad.cpu(), W.grad.cpu()


@pytest.mark.parametrize("N,D,V", [(300, 128, 1003), (777, 768, 50277), (4096, 1024, 50277)])
def test_lce_matches_fp64(cuda_dev, N, D, V):
    h, w, labels = make_case(N, D, V, seed=N)
    loss, dh, dw = run(h, w, labels, cuda_dev)
    # truth: fp64 on the bf16-rounded operands (the kernel and autocast compute on bf16 h and W)
    l64, dh64, dw64 = O.linear_cross_entropy(h.double(), w.to(torch.bfloat16).double(), labels)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        from sisa_b200.kernels.linear_ce import reference_linear_cross_entropy
        eager = reference_linear_cross_entropy(h.to(cuda_dev), w.to(cuda_dev), labels.to(cuda_dev)).float().cpu()
    e_eager = abs(float(eager) - float(l64))
    assert abs(float(loss) - float(l64)) <= 2 * e_eager + 1e-5
    assert rel_err(dh, dh64) <= GRAD_REL
    assert rel_err(dw, dw64) <= GRAD_REL
    ignored = labels == -100
    assert bool((dh[ignored] == 0).all())


def test_lce_chunking_invariant(cuda_dev):
    h, w, labels = make_case(1000, 256, 3000, seed=3)
    l1, dh1, dw1 = run(h, w, labels, cuda_dev)
    l2, dh2, dw2 = run(h, w, labels, cuda_dev, chunk_tokens=128)
    assert torch.equal(dh1, dh2)                       # rows are independent of the chunking
    assert float((l1 - l2).abs()) <= 1e-6 * abs(float(l1))
    assert rel_err(dw2, dw1) <= 1e-5                   # fp32 accumulation order across chunks


def test_lce_grad_scale_promise(cuda_dev):
    from sisa_b200 import backends
    from sisa_b200.kernels.linear_ce import linear_cross_entropy

    h, w, labels = make_case(200, 128, 500, seed=4)
    l_ref, dh_ref, dw_ref = run(h, w, labels, cuda_dev)
    H = h.to(cuda_dev).requires_grad_(True)
    W = w.to(cuda_dev).requires_grad_(True)
    loss = linear_cross_entropy(H, W, labels.to(cuda_dev), grad_scale=0.25)
    (loss * 0.25).backward()
    backends.check_status(0)
    assert rel_err(H.grad.cpu(), dh_ref * 0.25) <= 1e-2
    # a broken promise is reported through the status word, not a device assert
    H2 = h.to(cuda_dev).requires_grad_(True)
    loss = linear_cross_entropy(H2, w.to(cuda_dev), labels.to(cuda_dev), grad_scale=0.25)
    (loss * 0.5).backward()
    with pytest.raises(RuntimeError, match="grad_scale"):
        backends.check_status(0)


def test_lce_nan_propagates(cuda_dev):
    from sisa_b200 import backends

    h, w, labels = make_case(64, 128, 300, seed=5, n_ignore=0)
    h[7, 3] = float("nan")
    loss, _, _ = run(h, w, labels, cuda_dev)
    assert torch.isnan(loss)
    with pytest.raises(FloatingPointError):
        backends.check_status(0)


def test_lce_backward_seed_and_dtypes(cuda_dev):
    """The backward multiplies the stored gradients by its seed on the device (nothing to do for 1), in
    the dtypes of hidden and weight; a second backward through one graph is refused."""
    from sisa_b200.kernels.linear_ce import linear_cross_entropy

    h, w, labels = make_case(300, 128, 1003, seed=6)
    lab = labels.to(cuda_dev)
    grads = {}
    for seed in (1.0, 3.0):
        H = h.to(cuda_dev).requires_grad_(True)
        W = w.to(cuda_dev).requires_grad_(True)
        (linear_cross_entropy(H, W, lab) * seed).backward()
        grads[seed] = (H.grad, W.grad)
    assert grads[3.0][0].dtype == torch.bfloat16 and grads[3.0][1].dtype == torch.float32
    assert torch.equal(grads[3.0][1], grads[1.0][1] * 3.0)          # fp32 dW: the same product
    assert rel_err(grads[3.0][0].float(), grads[1.0][0].float() * 3.0) <= 1e-2
    # fp32 hidden under autocast: dh comes back fp32
    H = h.float().to(cuda_dev).requires_grad_(True)
    W = w.to(cuda_dev).requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        loss = linear_cross_entropy(H, W, lab)
    (loss * 2.0).backward(retain_graph=True)
    assert H.grad.dtype == torch.float32
    assert rel_err(H.grad, grads[1.0][0].float() * 2.0) <= 1e-2
    with pytest.raises(RuntimeError, match="retain_graph"):
        loss.backward()


@pytest.mark.parametrize("V", [50277, 3000])
def test_lce_records_outside_dx(cuda_dev, V):
    """Without a dX gradient the per-row records take a buffer of their own instead of the chunk's dX
    rows: the loss and dW equal those of the call that also computes dX, bit for bit."""
    from sisa_b200.kernels.linear_ce import linear_cross_entropy

    h, w, labels = make_case(700, 256, V, seed=V)
    l_both, _, dw_both = run(h, w, labels, cuda_dev, chunk_tokens=256)
    W = w.to(cuda_dev).requires_grad_(True)
    loss = linear_cross_entropy(h.to(cuda_dev), W, labels.to(cuda_dev), chunk_tokens=256)
    loss.backward()
    torch.cuda.synchronize()
    assert torch.equal(loss.detach().cpu(), l_both)
    assert torch.equal(W.grad.cpu(), dw_both)
