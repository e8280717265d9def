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


def test_fused_prefill_matches_unfused_glue(cuda_dev, monkeypatch):
    """The prompt pass through the fused layer core (one projection GEMM, sisa_prep_fwd, sisa_attn_fwd, the
    cache filled from their outputs, block norms on the norm kernels) against the unfused glue of the
    reference's prefill (separate projections, torch recurrences and rotations, the unfused attention):
    the last position's logits, every cache entry, and three decode steps from each cache."""
    from sisa_b200 import modeling
    from sisa_b200.generation import SISACache

    model = _tiny(cuda_dev, "cuda").to(cuda_dev).to(torch.bfloat16)
    ids = torch.randint(0, 97, (3, 203), generator=torch.Generator().manual_seed(5)).to(cuda_dev)

    def run(fused):
        if not fused:
            monkeypatch.setattr(modeling.SISAAttention, "_use_fused_prefill", lambda self, x, state, requested: False)
        cache = SISACache(capacity=210)
        out = []
        with torch.no_grad():
            out.append(model(ids[:, :200], cache=cache, logits_to_keep=1).logits[:, -1].float())
            for t in range(200, 203):
                out.append(model(ids[:, t:t + 1], cache=cache, logits_to_keep=1).logits[:, -1].float())
        monkeypatch.undo()
        return out, cache

    got, cg = run(True)
    want, cw = run(False)
    for a, b in zip(got, want):
        assert max_abs(a.cpu(), b.cpu()) <= 2e-2
    for i in range(2):
        sg, sw = cg.get(i), cw.get(i)
        assert sg.length == sw.length == 203
        for name in ("k", "v", "b"):
            assert max_abs(getattr(sg, name).float().cpu(), getattr(sw, name).float().cpu()) <= 2e-2, name
        for name in ("g", "fgate"):
            # cumulative sums over 200 positions of gate values that the two paths round through different
            # GEMMs: compare relative to the sums' size
            a, b = getattr(sg, name).cpu(), getattr(sw, name).cpu()
            assert max_abs(a, b) <= 1e-4 * float(b.abs().max()) + 1e-3, name
        # Phi at the last position sums theta (|theta| up to ~4 in this model) over the prompt; one element
        # rounded one bf16 step apart by the two GEMMs moves it by 2^-5, a missing token by ~|theta|
        assert max_abs(sg.phi.reshape(sw.phi.shape).float().cpu(), sw.phi.float().cpu()) <= 0.1


def _prefilled(model, ids, n_prompt, capacity):
    from sisa_b200.generation import SISACache

    cache = SISACache(capacity=capacity)
    with torch.no_grad():
        logits = model(ids[:, :n_prompt], cache=cache, logits_to_keep=1).logits[:, -1]
    return cache, logits


def test_decode_graph_matches_eager_steps(cuda_dev):
    """A DecodeGraph replay (device position counter, capacity-sized split-K) against eager decode steps of
    the same model from the same prefill: logits of every step and the caches afterwards."""
    from sisa_b200.generation import DecodeGraph

    model = _tiny(cuda_dev, "cuda").to(cuda_dev).to(torch.bfloat16).eval()
    ids = torch.randint(0, 97, (3, 60), generator=torch.Generator().manual_seed(4)).to(cuda_dev)
    ce, _ = _prefilled(model, ids, 41, 300)
    cg, _ = _prefilled(model, ids, 41, 300)
    with torch.no_grad():
        want = [model(ids[:, t:t + 1], cache=ce, logits_to_keep=1).logits[:, -1].float() for t in range(41, 60)]
        got = [model(ids[:, 41:42], cache=cg, logits_to_keep=1).logits[:, -1].float()]
        assert DecodeGraph.supported(model, cg)
        graph = DecodeGraph(model, cg, 3)
        assert all(cg.get(i).length == 42 for i in range(2))
        for t in range(42, 60):
            got.append(graph.step(ids[:, t]).float().clone())
        assert int(graph.pos_dev.item()) == 60 and graph.room() == cg.get(0).capacity - 60
        graph.close()
    assert all(cg.get(i).pos_dev is None for i in range(2))
    for a, b in zip(got, want):
        assert max_abs(a.cpu(), b.cpu()) <= 2e-2
    for i in range(2):
        sg, se = cg.get(i), ce.get(i)
        assert sg.length == se.length == 60
        for name in ("k", "v", "b"):
            assert max_abs(getattr(sg, name).float().cpu(), getattr(se, name).float().cpu()) <= 2e-2, name
        for name in ("g", "fgate"):
            assert max_abs(getattr(sg, name).cpu(), getattr(se, name).cpu()) <= 1e-3, name
    # the cache stays usable eagerly after the graph is closed
    with torch.no_grad():
        more = model(ids[:, 59:60], cache=cg, logits_to_keep=1).logits[:, -1]
    assert torch.isfinite(more.float()).all() and cg.get(0).length == 61


def test_generate_graph_equals_eager(cuda_dev):
    model = _tiny(cuda_dev, "cuda").to(cuda_dev).to(torch.bfloat16)
    ids = torch.randint(0, 97, (4, 70), generator=torch.Generator().manual_seed(5)).to(cuda_dev)
    a = model.generate(ids, max_new_tokens=20, cuda_graph=True)
    b = model.generate(ids, max_new_tokens=20, cuda_graph=False)
    assert a.shape == (4, 90) and torch.equal(a, b)
    c = model.generate(ids, max_new_tokens=20, eos_token_id=int(a[0, 75]))   # early stop with the graph
    assert c.shape[1] <= 90 and torch.equal(c[:, :71], a[:, :71])


def test_device_position_out_of_range_sets_status(cuda_dev):
    """A device position outside the cache: sisa_decode_prep_dpos writes nothing and sisa_decode_attn_dpos
    attends to nothing; both set SISA_ST_BAD_POS in the status word (no device fault)."""
    from sisa_b200 import _lib, backends
    from sisa_b200.kernels.decode import decode_attention, decode_prep

    model = _tiny(cuda_dev, "cuda").to(cuda_dev).to(torch.bfloat16).eval()
    ids = torch.randint(0, 97, (2, 30), generator=torch.Generator().manual_seed(6)).to(cuda_dev)
    cache, _ = _prefilled(model, ids, 20, 64)
    st = cache.get(0)
    att = model.layers[0].attn
    x = model.layers[0].attn_norm(model.embed(ids[:, 20:21]))
    word = backends.status_word(cuda_dev)
    with torch.no_grad():
        weight, bias = att._fused_weights_static()
        proj = torch.nn.functional.linear(x, weight, bias)
        before = [t.clone() for t in (st.k_buf, st.v_buf, st.b_buf, st.g_buf, st.f_buf, st.phi_buffer())]
        torch.cuda.synchronize()
        word.zero_()
        st.pos_dev = torch.full((1,), st.capacity, dtype=torch.int32, device=cuda_dev)
        try:
            q, c, g, f = decode_prep(proj, att._forget_logits(x), st, 2)
            torch.cuda.synchronize()
            assert int(word.item()) & _lib.ST_BAD_POS
            after = (st.k_buf, st.v_buf, st.b_buf, st.g_buf, st.f_buf, st.phi)
            for a, b in zip(before, after):   # bitwise: the buffers' unused tails hold arbitrary bits
                assert torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))
            word.zero_()
            y = decode_attention(q, c, g, f, st, att.lam())
            torch.cuda.synchronize()
            assert int(word.item()) & _lib.ST_BAD_POS
            assert torch.count_nonzero(y) == 0
        finally:
            st.pos_dev = None
            word.zero_()


def test_lm_logits_padded_rows_equal_linear(cuda_dev):
    """Inference logits through row-padded storage are F.linear's values (a view of padded rows)."""
    from sisa_b200.modeling import _lm_logits

    gen = torch.Generator().manual_seed(4)
    h = torch.randn(3, 5, 768, generator=gen).to(torch.bfloat16).to(cuda_dev)
    w = (torch.randn(50277, 768, generator=gen) * 0.02).to(torch.bfloat16).to(cuda_dev)
    with torch.no_grad():
        got = _lm_logits(h, w)
        want = torch.nn.functional.linear(h, w)
    assert got.shape == want.shape and got.stride(-2) == 50280
    assert torch.allclose(got.float(), want.float(), rtol=1e-2, atol=1e-2)
    assert torch.equal(got.argmax(-1), want.argmax(-1)) or (got.float() - want.float()).abs().max() < 1e-2
