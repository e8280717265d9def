"""Model-level: the cuda implementation (fused layer core, linear-CE) against the torch implementation and
fp64, under bf16 autocast (the reference's tests/test_model_cuda.py gates)."""
from __future__ import annotations

import types

import pytest
import torch

import sisa_b200 as sisa
from tests.helpers import max_abs, rel_err

pytestmark = pytest.mark.gpu

GROUPS = {"attn": ("attn.W_", "attn.alpha", "attn.theta", "attn.forget", "attn.lambda"),
          "ffn": ("ffn.",), "embed": ("embed.",), "norm": ("norm.",)}


def tiny(seed=0):
    torch.manual_seed(seed)
    cfg = sisa.SISAConfig(vocab_size=97, d_model=128, n_layer=2, n_head=2, d_ff=96, zero_init_c=False,
                          attn_impl="torch")
    m = sisa.SISAForCausalLM(cfg)
    gen = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        for layer in m.layers:
            a = layer.attn
            a.theta_proj.weight.copy_(torch.randn(a.theta_proj.weight.shape, generator=gen) * 0.2)
            a.alpha_proj.bias.copy_(torch.rand(2, generator=gen) * 3.0 - 4.0)
            a.forget_proj.bias.copy_(torch.rand(2, generator=gen) * 3.0)
            a.lambda_raw.copy_(torch.rand(2, generator=gen) * 2.0 - 0.5)
    return m


def run(model, ids, dev, impl, fused_ce=False):
    m = model.to(dev)
    m.set_attn_impl(impl)
    m.zero_grad(set_to_none=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = m(ids.to(dev), labels=ids.to(dev), fused_ce=fused_ce)
    out.loss.backward()
    torch.cuda.synchronize()
    grads = {n: p.grad.detach().float().cpu() for n, p in m.named_parameters()}
    return out.loss.detach().float().cpu(), (None if out.logits is None else out.logits.detach().float().cpu()), grads


def group_err(grads, ref):
    out = {}
    for gname, keys in GROUPS.items():
        names = [n for n in ref if any(k in n for k in keys)]
        a = torch.cat([grads[n].flatten().double() for n in names])
        b = torch.cat([ref[n].flatten().double() for n in names])
        out[gname] = rel_err(a, b)
    return out


def test_cuda_model_matches_torch_and_fp64(cuda_dev):
    model = tiny()
    ids = torch.randint(0, 97, (2, 300), generator=torch.Generator().manual_seed(3))
    m64 = tiny().double()
    o64 = m64(ids, labels=ids)
    o64.loss.backward()
    g64 = {n: p.grad.detach() for n, p in m64.named_parameters()}
    lt, logt, gt = run(model, ids, cuda_dev, "torch")
    lc, logc, gc = run(model, ids, cuda_dev, "cuda")
    d_torch = abs(float(lt) - float(o64.loss))
    assert abs(float(lc) - float(o64.loss)) <= max(2 * d_torch, 2e-3)
    e_torch = max_abs(logt, o64.logits)
    assert max_abs(logc, o64.logits) <= 2 * e_torch + 1e-3
    et, ec = group_err(gt, g64), group_err(gc, g64)
    for gname in GROUPS:
        assert ec[gname] <= 3 * et[gname] + 2e-3, (gname, ec, et)


def test_fused_ce_loss_and_grads(cuda_dev):
    model = tiny(1)
    ids = torch.randint(0, 97, (2, 257), generator=torch.Generator().manual_seed(4))
    l1, _, g1 = run(model, ids, cuda_dev, "cuda", fused_ce=False)
    l2, logits2, g2 = run(model, ids, cuda_dev, "cuda", fused_ce=True)
    assert logits2 is None
    assert abs(float(l1) - float(l2)) <= 1e-2
    e = group_err(g2, g1)
    assert all(v <= 5e-2 for v in e.values()), e


def test_cuda_model_deterministic(cuda_dev):
    model = tiny(2)
    ids = torch.randint(0, 97, (2, 200), generator=torch.Generator().manual_seed(5))
    l1, _, g1 = run(model, ids, cuda_dev, "cuda")
    l2, _, g2 = run(model, ids, cuda_dev, "cuda")
    assert torch.equal(l1, l2)
    for n in g1:
        assert torch.equal(g1[n], g2[n]), n


def test_trainer_cuda_graph_matches_eager(cuda_dev):
    """The captured whole-step graph (forward, backward, clipping, AdamW) trains like the eager step."""
    from sisa_b200 import dp

    cfg = sisa.SISAConfig(vocab_size=97, d_model=128, n_layer=2, n_head=2, d_ff=96, attn_impl="cuda")
    ids = [torch.randint(0, 97, (2, 256), generator=torch.Generator().manual_seed(7 + i)).to(cuda_dev)
           for i in range(4)]
    losses = {}
    params = {}
    for mode in (False, True):
        model = dp.build_model(cfg, cuda_dev, seed=3)
        tr = dp.Trainer(model, cuda_graph=mode)
        losses[mode] = [float(tr.step(ids[i % 4])) for i in range(6)]
        torch.cuda.synchronize()
        params[mode] = {n: p.detach().clone() for n, p in model.named_parameters()}
    assert losses[True][0] == losses[False][0]
    for a, b in zip(losses[True], losses[False]):
        assert abs(a - b) <= 1e-4 * max(1.0, abs(b)), (losses[True], losses[False])
    for n in params[False]:
        assert torch.allclose(params[True][n], params[False][n], rtol=1e-4, atol=1e-5), n


def test_fused_projection_matches_autocast_linear(cuda_dev):
    """fused_projection = F.linear(x, W_cat, b_cat) under bf16 autocast: identical output and input
    gradient; the weight gradients are the same product kept in fp32 (autocast rounds it to bf16
    first); the bias gradient from the alpha columns only."""
    from sisa_b200.kernels.fused import concat_fused_weights, fused_projection, fused_layout

    H, d = 4, 256
    gen = torch.Generator(device=cuda_dev).manual_seed(5)
    rnd = lambda *s: torch.randn(s, generator=gen, device=cuda_dev) * 0.05  # noqa: E731
    ws = [rnd(H * 64, d), rnd(H * 64, d), rnd(H * 64, d), rnd(H * 32, d), rnd(H * 32, d), rnd(H * 16, d), rnd(H, d)]
    ba = rnd(H)
    x = torch.randn((2, 96, d), generator=gen, device=cuda_dev).to(torch.bfloat16)
    ref = [t.detach().clone().requires_grad_(True) for t in ws + [ba]]
    ker = [t.detach().clone().requires_grad_(True) for t in ws + [ba]]
    xr, xk = x.detach().clone().requires_grad_(True), x.detach().clone().requires_grad_(True)
    go = torch.randn((2, 96, fused_layout(H)["NPAD"]), generator=gen, device=cuda_dev).to(torch.bfloat16)
    owner = types.SimpleNamespace()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        W, b = concat_fused_weights(*ref)
        yr = torch.nn.functional.linear(xr, W, b)
        yk = fused_projection(xk, ker[:-1], ker[-1], torch.bfloat16, owner)
    assert yk.dtype == yr.dtype and torch.equal(yk, yr)
    yr.backward(go)
    yk.backward(go)
    assert torch.equal(xk.grad, xr.grad)
    dw32 = torch.mm(go.reshape(-1, go.shape[-1]).t(), x.reshape(-1, d), out_dtype=torch.float32)
    row = 0
    for a, r in zip(ker[:-1], ref[:-1]):
        n = a.shape[0]
        assert a.grad.dtype == torch.float32 and torch.equal(a.grad, dw32[row:row + n])
        assert torch.allclose(a.grad.to(torch.bfloat16).float(), r.grad, rtol=2 ** -7, atol=0)
        row += n
    assert torch.allclose(ker[-1].grad, ref[-1].grad, rtol=1e-2, atol=1e-3)
    # without gradients the compute-dtype concatenation is kept while the weights are unchanged and
    # rebuilt after an update
    cached = owner.__dict__["_wcat_train"][1]
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        fused_projection(xk, ker[:-1], ker[-1], torch.bfloat16, owner)
    assert owner.__dict__["_wcat_train"][1] is cached
    with torch.no_grad():
        ker[0].add_(1.0)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        y2 = fused_projection(xk, ker[:-1], ker[-1], torch.bfloat16, owner)
        W2, b2 = concat_fused_weights(*[t.detach() for t in ker])
        y2r = torch.nn.functional.linear(xk.detach(), W2, b2)
    assert owner.__dict__["_wcat_train"][1] is not cached
    assert torch.equal(y2, y2r)
    # with gradients it is rebuilt on every call, so an update that leaves the versions alone (a fused
    # optimizer's) is seen as well
    ker[1].data.add_(1.0)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y3 = fused_projection(xk, ker[:-1], ker[-1], torch.bfloat16, owner)
        W3, b3 = concat_fused_weights(*[t.detach() for t in ker])
        y3r = torch.nn.functional.linear(xk.detach(), W3, b3)
    assert torch.equal(y3.detach(), y3r)
