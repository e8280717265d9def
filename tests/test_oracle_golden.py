"""The oracle (oracle/sisa_oracle.py) against fixtures produced by the reference implementation itself
(tests/golden/make_golden.py). CPU only."""
from __future__ import annotations

import math

import torch

from oracle import sisa_oracle as O


def test_layout_known_answers(golden):
    known = golden("known")
    for h, lay in known["layouts"].items():
        assert O.fused_layout(h) == lay
    assert {h: lay["NPAD"] for h, lay in known["layouts"].items()} == {8: 2192, 12: 3280, 16: 4368}


def test_attention_matches_reference_fp64(golden):
    case = golden("attn_case")
    x = case["inputs"]
    o, lse = O.attention(x["q"], x["k"], x["v"], x["c"], x["b"], x["g"], x["lam"], x["F"], block_q=16)
    assert torch.allclose(o, case["o"], rtol=1e-10, atol=1e-12)
    gr = O.attention_grads(x["q"], x["k"], x["v"], x["c"], x["b"], x["g"], x["lam"], x["F"], case["dout"])
    for name, ref in case["grads"].items():
        got = gr["dF" if name == "dF" else name]
        assert torch.allclose(got, ref, rtol=1e-9, atol=1e-11), name


def test_attention_lse_is_log2_normaliser(golden):
    case = golden("attn_case")
    x = case["inputs"]
    _, lse = O.attention(x["q"], x["k"], x["v"], x["c"], x["b"], x["g"], x["lam"], x["F"])
    L = x["q"].shape[2]
    s = torch.matmul(x["q"], x["k"].transpose(-1, -2)) / 8
    s = s + x["lam"].view(1, -1, 1, 1) * torch.exp((x["g"].unsqueeze(-1) - x["g"].unsqueeze(-2)).tril()) * \
        torch.matmul(x["c"], x["b"].transpose(-1, -2)) + (x["F"].unsqueeze(-1) - x["F"].unsqueeze(-2))
    s = s.masked_fill(~torch.ones(L, L, dtype=torch.bool).tril(), float("-inf"))
    assert torch.allclose(lse, torch.logsumexp(s, -1) / math.log(2), rtol=1e-12, atol=1e-12)


def test_prep_matches_reference_glue(golden):
    case = golden("prep_case")
    out = O.prep(case["proj"].double(), case["z"].double(), case["n_head"])
    ref = case["ref"]
    for name in ("q", "k", "v", "c", "b", "g", "phi"):
        assert torch.allclose(out[name], ref[name].double(), rtol=2e-5, atol=2e-5), name
    assert torch.allclose(out["F"], ref["F"].double(), rtol=2e-5, atol=2e-5)


def test_linear_ce_matches_reference(golden):
    case = golden("lce_case")
    loss, dh, dw = O.linear_cross_entropy(case["hidden"], case["weight"], case["labels"])
    # the reference casts the logits to fp32 before the CE (linear_ce.py:223): fp32-level agreement
    assert torch.allclose(loss, case["loss"].double(), rtol=1e-6)
    assert torch.allclose(dh, case["dh"], rtol=1e-5, atol=1e-8)
    assert torch.allclose(dw, case["dw"], rtol=1e-5, atol=1e-8)
    assert torch.all(dh[[3, 10, 11]] == 0)


def test_rotate_pairs_is_complex_multiply():
    gen = torch.Generator().manual_seed(0)
    z = torch.randn(3, 5, 32, generator=gen, dtype=torch.float64)
    phi = torch.randn(3, 5, 16, generator=gen, dtype=torch.float64)
    zc = torch.view_as_complex(z.view(3, 5, 16, 2).contiguous())
    ref = torch.view_as_real(zc * torch.polar(torch.ones_like(phi), phi)).flatten(-2)
    assert torch.allclose(O.rotate_pairs(z, phi), ref, atol=1e-14)


def test_decode_rows_equals_full_attention(golden):
    case = golden("attn_case")
    x = case["inputs"]
    o, _ = O.attention(x["q"], x["k"], x["v"], x["c"], x["b"], x["g"], x["lam"], x["F"])
    t = 50
    sl = slice(t, t + 1)
    got = O.decode_rows(x["q"][:, :, sl], x["c"][:, :, sl], x["g"][:, :, sl], x["F"][:, :, sl],
                        x["k"][:, :, :t + 1], x["v"][:, :, :t + 1], x["b"][:, :, :t + 1], x["g"][:, :, :t + 1],
                        x["F"][:, :, :t + 1], x["lam"], t)
    assert torch.allclose(got, o[:, :, sl], rtol=1e-12, atol=1e-12)
