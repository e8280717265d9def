"""Incremental-decode kernel (sisa_decode_attn) against the fp64 oracle, and cached generation on CUDA."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import sisa_oracle as O
from tests.helpers import max_abs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N", [1, 2, 255, 256, 257, 1000, 5000])
def test_decode_matches_oracle(cuda_dev, N):
    from sisa_b200.generation import LayerState
    from sisa_b200.kernels.decode import decode_attention

    B, H = 2, 3
    proj, z, lam = O.make_proj_inputs(B, N, H, seed=N, a_mean=-3.0, z_mean=2.0)
    pr = O.prep(proj.to(torch.bfloat16).double(), z.double(), H)
    bf = torch.bfloat16
    k, v, b = pr["k"].to(bf), pr["v"].to(bf), pr["b"].to(bf)
    g, Fg = pr["g"].float(), pr["F"].float()
    q, c = pr["q"][:, :, -1:].to(bf), pr["c"][:, :, -1:].to(bf)
    lam = lam * torch.linspace(0.5, 2.0, H)
    dev = cuda_dev
    state = LayerState(k.to(dev), v.to(dev), b.to(dev), g.to(dev), Fg.to(dev), torch.zeros(B, H, 16, device=dev),
                       capacity=N + 37)
    y = decode_attention(q.to(dev), c.to(dev), g[:, :, -1:].to(dev), Fg[:, :, -1:].to(dev), state, lam.to(dev))
    torch.cuda.synchronize()
    ref = O.decode_rows(q.double(), c.double(), g[:, :, -1:].double(), Fg[:, :, -1:].double(), k.double(),
                        v.double(), b.double(), g.double(), Fg.double(), lam.double(), N - 1)
    assert max_abs(y.cpu(), ref) <= 1e-2


def _tiny(dev, impl):
    import sisa_b200 as sisa

    torch.manual_seed(0)
    cfg = sisa.SISAConfig(vocab_size=97, d_model=128, n_layer=2, n_head=2, d_ff=96, attn_impl=impl, zero_init_c=False)
    model = sisa.SISAForCausalLM(cfg)
    with torch.no_grad():
        for layer in model.layers:
            layer.attn.theta_proj.weight.mul_(20)
            layer.attn.alpha_proj.bias.fill_(-2.0)
            layer.attn.forget_proj.bias.fill_(1.0)
    return model


def test_cached_decode_logits_match_fp64(cuda_dev):
    """Prefill through the tcgen05 attention and 6 decode steps through the decode kernel, bf16 weights,
    against the same model in fp64 on CPU (the reference's bf16 decode gate is 5e-2)."""
    from sisa_b200.generation import SISACache

    model = _tiny(cuda_dev, "cuda")
    ref = _tiny(cuda_dev, "torch").double()
    gen = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 97, (3, 150), generator=gen)
    m = model.to(cuda_dev).to(torch.bfloat16)
    cache, cache64 = SISACache(), SISACache()
    with torch.no_grad():
        got = [m(ids[:, :144].to(cuda_dev), cache=cache, logits_to_keep=1).logits[:, -1].float().cpu()]
        want = [ref(ids[:, :144], cache=cache64, logits_to_keep=1).logits[:, -1]]
        for t in range(144, 150):
            got.append(m(ids[:, t:t + 1].to(cuda_dev), cache=cache, logits_to_keep=1).logits[:, -1].float().cpu())
            want.append(ref(ids[:, t:t + 1], cache=cache64, logits_to_keep=1).logits[:, -1])
    for a, b in zip(got, want):
        assert max_abs(a, b) <= 5e-2


def test_generate_cuda_runs_and_is_deterministic(cuda_dev):
    model = _tiny(cuda_dev, "cuda").to(cuda_dev).to(torch.bfloat16)
    ids = torch.randint(0, 97, (4, 65), generator=torch.Generator().manual_seed(2)).to(cuda_dev)
    a = model.generate(ids, max_new_tokens=12)
    b = model.generate(ids, max_new_tokens=12)
    assert a.shape == (4, 77) and torch.equal(a, b)


def test_fused_decode_step_matches_unfused_glue(cuda_dev, monkeypatch):
    """The fused decode step (one projection GEMM + sisa_decode_prep) against the unfused glue of the same
    step (separate projections, torch recurrences and rotation, cache append), logits and caches; the
    cache starts with one free slot, so the fused step also grows it."""
    from sisa_b200 import modeling
    from sisa_b200.generation import SISACache

    model = _tiny(cuda_dev, "cuda").to(cuda_dev).to(torch.bfloat16)
    ids = torch.randint(0, 97, (3, 40), generator=torch.Generator().manual_seed(3)).to(cuda_dev)

    def run(fused):
        if not fused:
            monkeypatch.setattr(modeling.SISAAttention, "_use_fused_decode", lambda self, x, state, requested: False)
        cache = SISACache(capacity=34)
        out = []
        with torch.no_grad():
            out.append(model(ids[:, :33], cache=cache, logits_to_keep=1).logits[:, -1].float())
            for t in range(33, 40):
                out.append(model(ids[:, t:t + 1], cache=cache, logits_to_keep=1).logits[:, -1].float())
        monkeypatch.undo()
        return out, cache

    got, cg = run(True)
    want, cw = run(False)
    for a, b in zip(got, want):
        assert max_abs(a.cpu(), b.cpu()) <= 2e-2
    for i in range(2):
        sg, sw = cg.get(i), cw.get(i)
        assert sg.length == sw.length == 40
        for name in ("k", "v", "b"):
            assert max_abs(getattr(sg, name).float().cpu(), getattr(sw, name).float().cpu()) <= 2e-2, name
        for name in ("g", "fgate"):
            assert max_abs(getattr(sg, name).cpu(), getattr(sw, name).cpu()) <= 1e-3, name
        assert max_abs(sg.phi.reshape(sw.phi.shape).cpu(), sw.phi.float().cpu()) <= 1e-3
