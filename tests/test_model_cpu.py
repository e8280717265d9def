"""Model-level parity with the reference on CPU: the reference's own tiny model (state dict, loss, logits,
gradients, greedy generation) from tests/golden/model_case.pt, plus config known answers."""
from __future__ import annotations

import pytest
import torch

import sisa_b200 as sisa
from sisa_b200.generation import SISACache


def load_ref_model(golden):
    case = golden("model_case")
    cfg = sisa.SISAConfig.from_dict(case["config"])
    model = sisa.SISAForCausalLM(cfg)
    model.load_state_dict(case["state_dict"], strict=True)
    return case, model


def test_param_counts_and_keys(golden):
    known = golden("known")
    for name, n in known["param_counts"].items():
        assert sisa.SISAConfig.preset(name).num_parameters() == n
    assert sisa.SISAConfig.preset("sisa-152m").num_parameters() == 151_878_576
    m = sisa.SISAForCausalLM(sisa.SISAConfig(vocab_size=97, d_model=128, n_layer=2, n_head=2, d_ff=96))
    assert sorted(m.state_dict().keys()) == known["state_dict_keys"]
    assert len(known["state_dict_keys"]) == 2 + 17 * 2


def test_forward_loss_logits_grads_match_reference(golden):
    case, model = load_ref_model(golden)
    m64 = model.double()
    out = m64(case["ids"], labels=case["ids"])
    assert torch.allclose(out.logits, case["logits"], rtol=1e-10, atol=1e-12)
    assert torch.allclose(out.loss.double(), case["loss"].double(), rtol=1e-6)
    out.loss.backward()
    params = dict(m64.named_parameters())
    for name, g in case["grads"].items():
        assert torch.allclose(params[name].grad, g, rtol=1e-5, atol=1e-9), name


def test_greedy_generate_and_cached_decode_match_reference(golden):
    case, model = load_ref_model(golden)
    m64 = model.double()
    with torch.no_grad():
        out = m64.generate(case["prompt"], max_new_tokens=8)
        assert torch.equal(out, case["generated"])
        cache = SISACache()
        pre = m64(case["prompt"], cache=cache, logits_to_keep=1).logits[:, -1]
        step = m64(case["generated"][:, 12:13], cache=cache, logits_to_keep=1).logits[:, -1]
    assert torch.allclose(pre, case["prefill_logits"], rtol=1e-10, atol=1e-12)
    assert torch.allclose(step, case["step_logits"], rtol=1e-10, atol=1e-12)


def test_cache_grows_beyond_capacity():
    torch.manual_seed(0)
    cfg = sisa.SISAConfig(vocab_size=50, d_model=128, n_layer=1, n_head=2, d_ff=64, attn_impl="torch",
                          zero_init_c=False)
    model = sisa.SISAForCausalLM(cfg).double()
    ids = torch.randint(0, 50, (1, 300))
    outs = {}
    with torch.no_grad():
        full = model(ids).logits[:, -1]
        for cap in (8, 1000):
            cache = SISACache(capacity=cap)
            model(ids[:, :290], cache=cache)
            for t in range(290, 300):
                outs[cap] = model(ids[:, t:t + 1], cache=cache, logits_to_keep=1).logits[:, -1]
            assert cache.get(0).capacity >= 300 and cache.seq_len == 300
    assert torch.equal(outs[8], outs[1000])          # growing the buffers changes nothing
    # decode continues g/F/Phi in fp32 (as the reference): fp32-level agreement with the full forward
    assert torch.allclose(outs[8], full, rtol=1e-6, atol=1e-6)


def test_eos_handling_matches_per_step_semantics():
    torch.manual_seed(1)
    cfg = sisa.SISAConfig(vocab_size=5, d_model=128, n_layer=1, n_head=2, d_ff=64, attn_impl="torch")
    model = sisa.SISAForCausalLM(cfg).double()
    ids = torch.randint(0, 5, (3, 6))
    with torch.no_grad():
        a = model.generate(ids, max_new_tokens=40, eos_token_id=[1, 2], eos_check_every=1)
        b = model.generate(ids, max_new_tokens=40, eos_token_id=[1, 2], eos_check_every=16)
    assert torch.equal(a, b)


@pytest.mark.parametrize("bad", [dict(d_model=100, n_head=3), dict(d_state=31), dict(attn_impl="tpu"),
                                 dict(attn_impl="cuda", d_model=512, n_head=4)])
def test_config_validation(bad):
    with pytest.raises(ValueError):
        sisa.SISAConfig(**bad)


def test_lambda_raw_stays_fp32_under_casts():
    m = sisa.SISAForCausalLM(sisa.SISAConfig(vocab_size=11, d_model=128, n_layer=1, n_head=2, d_ff=32))
    m = m.to(torch.bfloat16)
    assert m.layers[0].attn.lambda_raw.dtype == torch.float32
    assert m.layers[0].attn.W_Q.weight.dtype == torch.bfloat16


def test_auto_on_cpu_is_torch_and_cuda_forced_on_cpu_raises():
    from sisa_b200 import backends

    x = torch.zeros(1, 4, 128)
    assert backends.select_impl("auto", x, None) == "torch"
    with pytest.raises(ValueError):
        backends.select_impl("cuda", x, None)


def test_decode_graph_is_not_used_on_cpu(golden):
    """DecodeGraph needs the cuda attention path; on a CPU model generate() runs the eager loop whatever
    ``cuda_graph`` says, and the tokens are the reference's."""
    from sisa_b200.generation import DecodeGraph

    case, model = load_ref_model(golden)
    m64 = model.double()
    with torch.no_grad():
        cache = SISACache()
        m64(case["prompt"], cache=cache, logits_to_keep=1)
        assert not DecodeGraph.supported(m64, cache)
        a = m64.generate(case["prompt"], max_new_tokens=8)
        b = m64.generate(case["prompt"], max_new_tokens=8, cuda_graph=False)
    assert torch.equal(a, b) and torch.equal(a, case["generated"])
