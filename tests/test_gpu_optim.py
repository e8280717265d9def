"""The AdamW kernels (``sisa_adamw_flat``, ``sisa_adamw_tensors``, sisa_b200/optim.py) against an fp64
restatement of ``clip_grad_norm_`` + ``torch.optim.AdamW``, against each other and against torch's own
optimizer inside the Trainer."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.helpers import rel_err

pytestmark = pytest.mark.gpu


def _adamw64(p, g, m, v, t, lr, wd, b1, b2, eps, clip):
    g = g * clip
    p = p * (1 - lr * wd)
    m = b1 * m + (1 - b1) * g
    v = b2 * v + (1 - b2) * g * g
    denom = np.sqrt(v) / np.sqrt(1 - b2 ** t) + eps
    return p - lr / (1 - b1 ** t) * m / denom, m, v


def test_flat_adamw_kernel_matches_fp64(cuda_dev):
    from sisa_b200 import _lib, backends
    from sisa_b200.optim import _SEG, NPART

    rng = np.random.default_rng(0)
    n = 40000
    p = rng.standard_normal(n).astype(np.float32)
    g = (rng.standard_normal(n) * 3).astype(np.float32)
    segs = np.array([(0, 12000, 1e-3, 0.1), (12000, 12004, 1e-3, 0.0), (12008, 40000, 5e-4, 0.1)], dtype=_SEG)
    P, G = torch.tensor(p, device=cuda_dev), torch.tensor(g, device=cuda_dev)
    M, V = torch.zeros(n, device=cuda_dev), torch.zeros(n, device=cuda_dev)
    S = torch.from_numpy(segs.view(np.uint8).copy()).to(cuda_dev)
    step = torch.zeros(1, device=cuda_dev)
    part = torch.empty(NPART, dtype=torch.float64, device=cuda_dev)
    lib = _lib.load()
    p64, m64, v64 = p.astype(np.float64), np.zeros(n), np.zeros(n)
    b1, b2, eps, max_norm = 0.9, 0.95, 1e-8, 1.0
    for t in (1, 2, 3):
        _lib.check(lib.sisa_adamw_flat(P.data_ptr(), G.data_ptr(), M.data_ptr(), V.data_ptr(), n, S.data_ptr(), 3,
                                       step.data_ptr(), part.data_ptr(), NPART, b1, b2, eps, max_norm,
                                       backends.status_word(cuda_dev).data_ptr(), _lib.stream_ptr(cuda_dev)),
                   "sisa_adamw_flat")
        norm = np.sqrt((g.astype(np.float64) ** 2).sum())
        clip = min(1.0, max_norm / (norm + 1e-6))
        new = p64.copy()
        for s0, s1, lr, wd in segs:
            new[s0:s1], m64[s0:s1], v64[s0:s1] = _adamw64(p64[s0:s1], g[s0:s1].astype(np.float64), m64[s0:s1],
                                                          v64[s0:s1], t, float(lr), float(wd), b1, b2, eps, clip)
        p64 = new
    torch.cuda.synchronize()
    assert float(step.item()) == 3.0
    got = P.cpu().double().numpy()
    assert np.abs(got - p64).max() <= 1e-6 * (1 + np.abs(p64).max())
    # elements in no segment (12004 .. 12007) are left alone
    assert np.array_equal(got[12004:12008], p[12004:12008].astype(np.float64))
    assert int(backends.status_word(cuda_dev).item()) == 0


def _packed(arrays, dev):
    """Views into one buffer, back to back: every tensor after an odd-sized one starts off 16 bytes (as
    gradients do inside a DDP bucket)."""
    buf = torch.tensor(np.concatenate(arrays), device=dev)
    out, o = [], 0
    for a in arrays:
        out.append(buf[o:o + a.size])
        o += a.size
    return out


@pytest.mark.parametrize("packed", [False, True])
def test_tensor_adamw_matches_fp64(cuda_dev, packed):
    """TensorAdamW (``sisa_adamw_tensors``) over tensors of awkward sizes, two groups, two parameters
    without a gradient: three steps against the fp64 restatement of clip_grad_norm_ + AdamW. ``packed``
    makes parameters and gradients views into one buffer, most of them not 16-byte aligned."""
    from sisa_b200 import backends
    from sisa_b200.optim import TensorAdamW

    rng = np.random.default_rng(1)
    sizes = [12, 5, 1003, 40000, 7, 4096]
    init = [rng.standard_normal(n).astype(np.float32) for n in sizes]
    ps = (_packed(init, cuda_dev) if packed else [torch.tensor(a, device=cuda_dev) for a in init])
    if packed:
        assert any(p.data_ptr() % 16 for p in ps)
    groups = [{"params": ps[:3], "lr": 1e-3, "weight_decay": 0.1}, {"params": ps[3:], "lr": 5e-4, "weight_decay": 0.0}]
    opt = TensorAdamW(groups, betas=(0.9, 0.95), eps=1e-8, max_norm=1.0)
    p64 = [p.double().cpu().numpy() for p in ps]
    m64 = [np.zeros(n) for n in sizes]
    v64 = [np.zeros(n) for n in sizes]
    untouched = {k: ps[k].clone() for k in (0, 4)}          # no gradient: the first table entry starts past 0
    for t in (1, 2, 3):
        grads = [None if k in untouched else (rng.standard_normal(n) * 3).astype(np.float32)
                 for k, n in enumerate(sizes)]
        if packed:
            views = iter(_packed([np.zeros(n, np.float32) if g is None else g for n, g in zip(sizes, grads)],
                                 cuda_dev))
            for p, g in zip(ps, grads):
                view = next(views)
                p.grad = None if g is None else view
        else:
            for p, g in zip(ps, grads):
                p.grad = None if g is None else torch.tensor(g, device=cuda_dev)
        opt.step()
        norm = np.sqrt(sum((g.astype(np.float64) ** 2).sum() for g in grads if g is not None))
        clip = min(1.0, 1.0 / (norm + 1e-6))
        for k, g in enumerate(grads):
            if g is None:
                continue
            lr, wd = (1e-3, 0.1) if k < 3 else (5e-4, 0.0)
            p64[k], m64[k], v64[k] = _adamw64(p64[k], g.astype(np.float64), m64[k], v64[k], t, lr, wd, 0.9, 0.95,
                                              1e-8, clip)
    torch.cuda.synchronize()
    assert float(opt.step_count.item()) == 3.0
    for k, p in enumerate(ps):
        if k in untouched:
            assert torch.equal(p, untouched[k])
            continue
        got = p.double().cpu().numpy()
        assert np.abs(got - p64[k]).max() <= 1e-6 * (1 + np.abs(p64[k]).max()), k
    assert int(backends.status_word(cuda_dev).item()) == 0


def test_tensor_adamw_equals_flat_adamw(cuda_dev):
    """The tensor-list kernels and the flat kernels compute the same update, bit for bit."""
    from sisa_b200 import _lib, backends
    from sisa_b200.optim import _SEG, NPART, TensorAdamW

    rng = np.random.default_rng(4)
    sizes = [64, 1024, 36]
    ps = [torch.tensor(rng.standard_normal(n).astype(np.float32), device=cuda_dev) for n in sizes]
    flat = torch.cat([p.clone() for p in ps])
    gs = [torch.tensor((rng.standard_normal(n) * 2).astype(np.float32), device=cuda_dev) for n in sizes]
    gflat = torch.cat(gs)
    opt = TensorAdamW([{"params": ps, "lr": 1e-3, "weight_decay": 0.1}], max_norm=1.0)
    n = flat.numel()
    M, V = torch.zeros(n, device=cuda_dev), torch.zeros(n, device=cuda_dev)
    S = torch.from_numpy(np.array([(0, n, 1e-3, 0.1)], dtype=_SEG).view(np.uint8).copy()).to(cuda_dev)
    step = torch.zeros(1, device=cuda_dev)
    part = torch.empty(NPART, dtype=torch.float64, device=cuda_dev)
    for _ in range(2):
        for p, g in zip(ps, gs):
            p.grad = g
        opt.step()
        _lib.check(_lib.load().sisa_adamw_flat(flat.data_ptr(), gflat.data_ptr(), M.data_ptr(), V.data_ptr(), n,
                                               S.data_ptr(), 1, step.data_ptr(), part.data_ptr(), NPART, 0.9, 0.95,
                                               1e-8, 1.0, backends.status_word(cuda_dev).data_ptr(),
                                               _lib.stream_ptr(cuda_dev)), "sisa_adamw_flat")
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(ps), flat)


def test_trainer_flat_adamw_matches_torch_adamw(cuda_dev):
    """Trainer steps of a small model: the flat kernels against torch.optim.AdamW(fused) with
    clip_grad_norm_ on the same data and initial weights, and the graphed flat step against the eager
    one. Adam's first step moves every weight by lr * sign(g): after it the weights agree except where a
    gradient is so close to 0 that its sign differs with the last bits of the two computations; the
    losses of later steps agree closely."""
    import sisa_b200 as sisa
    from sisa_b200 import dp

    lr = 6e-4
    cfg = sisa.SISAConfig(d_model=256, n_head=4, d_ff=512, n_layer=2, vocab_size=512, attn_impl="cuda")
    gen = torch.Generator(device=cuda_dev).manual_seed(3)
    batches = [torch.randint(0, 512, (2, 256), generator=gen, device=cuda_dev) for _ in range(5)]
    one_step, losses = {}, {}
    for name, kw in (("flat", dict(flat_optimizer=True)), ("torch", dict(tensor_optimizer=False)),
                     ("tensor", dict()), ("graph", dict(flat_optimizer=True, cuda_graph=True)),
                     ("tensor_graph", dict(cuda_graph=True))):
        for n_steps in (1, 5):
            model = dp.build_model(cfg, cuda_dev, seed=0)
            tr = dp.Trainer(model, **kw)
            assert tr.flat_opt == (name in ("flat", "graph"))
            assert tr.list_opt == (name in ("tensor", "tensor_graph"))
            ls = [float(tr.step(b)) for b in batches[:n_steps]]
            torch.cuda.synchronize()
            if n_steps == 1:
                one_step[name] = {k: v.detach().clone() for k, v in model.state_dict().items()}
            else:
                losses[name] = ls
            tr.close()
    for other in ("torch", "graph", "tensor", "tensor_graph"):
        diff = torch.cat([(one_step["flat"][k].float() - one_step[other][k].float()).abs().reshape(-1)
                          for k in one_step["flat"]])
        assert float(diff.max()) <= 2.05 * lr
        assert float((diff > 1e-6).float().mean()) <= 1e-3, other
    for other in ("torch", "graph", "tensor", "tensor_graph"):
        for a, b in zip(losses["flat"], losses[other]):
            assert abs(a - b) <= 2e-3 * abs(b), (other, losses)
