"""The plain-PyTorch attention implementation (``impl="torch"``) against the fp64 oracle on CPU: forward
and every gradient of its hand-written tiled backward, for tile sizes that do and do not divide L."""
from __future__ import annotations

import pytest
import torch

from oracle import sisa_oracle as O
from sisa_b200.functional import rotate_pairs, sisa_attention_torch


def _inputs(B, H, L, dh, ds, seed, with_f=True):
    gen = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=gen, dtype=torch.float64)   # noqa: E731
    g = torch.cumsum(-torch.rand(B, H, L, generator=gen, dtype=torch.float64) * 0.3, dim=2)
    f = torch.cumsum(-torch.rand(B, H, L, generator=gen, dtype=torch.float64) * 0.2, dim=2) if with_f else None
    lam = torch.rand(H, generator=gen, dtype=torch.float64) + 0.3
    return dict(q=r(B, H, L, dh), k=r(B, H, L, dh), v=r(B, H, L, dh), c=r(B, H, L, ds), b=r(B, H, L, ds), g=g,
                lam=lam, F=f), r(B, H, L, dh)


@pytest.mark.parametrize("L,block,with_f", [(1, 4, True), (37, 8, True), (64, 16, False), (50, 256, True)])
def test_torch_attention_matches_fp64_oracle(L, block, with_f):
    x, dout = _inputs(2, 3, L, 16, 8, seed=L + block, with_f=with_f)
    names = ["q", "k", "v", "c", "b", "g", "lam"] + (["F"] if with_f else [])
    leaves = {n: x[n].clone().requires_grad_(True) for n in names}
    o = sisa_attention_torch(leaves["q"], leaves["k"], leaves["v"], leaves["c"], leaves["b"], leaves["g"],
                             leaves["lam"], leaves.get("F"), block_q=block)
    o.backward(dout)
    ref = O.attention_grads(x["q"], x["k"], x["v"], x["c"], x["b"], x["g"], x["lam"], x["F"], dout)
    assert torch.allclose(o, ref["o"], rtol=1e-10, atol=1e-12)
    for n in names:
        want = ref["dF" if n == "F" else "d" + n]
        assert torch.allclose(leaves[n].grad, want, rtol=1e-9, atol=1e-11), n


def test_torch_attention_fp32_and_bf16_inputs():
    x, dout = _inputs(1, 2, 40, 16, 8, seed=3)
    ref = O.attention_grads(x["q"], x["k"], x["v"], x["c"], x["b"], x["g"], x["lam"], x["F"], dout)
    for dt, tol in ((torch.float32, 1e-5), (torch.bfloat16, 3e-2)):
        xs = {n: (t.to(dt) if n in "qkvcb" else t.float()) for n, t in x.items()}
        o = sisa_attention_torch(xs["q"], xs["k"], xs["v"], xs["c"], xs["b"], xs["g"], xs["lam"], xs["F"],
                                 block_q=16)
        assert o.dtype == dt
        assert float((o.double() - ref["o"]).abs().max()) <= tol * 4


def test_rotate_pairs_is_complex_multiplication():
    gen = torch.Generator().manual_seed(0)
    z = torch.randn(3, 5, 8, generator=gen, dtype=torch.float64)
    phi = torch.randn(3, 5, 4, generator=gen, dtype=torch.float64)
    want = torch.view_as_real(torch.view_as_complex(z.reshape(3, 5, 4, 2)) * torch.polar(torch.ones_like(phi), phi))
    assert torch.allclose(rotate_pairs(z, phi), want.flatten(-2), atol=1e-14)
