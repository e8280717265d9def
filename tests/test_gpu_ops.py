"""The ``sisa_b200`` custom operators: schema and fake-implementation checks (``torch.library.opcheck``),
and torch.compile tracing the cuda path with no graph break (``fullgraph=True``) to the same results as
eager execution."""
from __future__ import annotations

import pytest
import torch

from oracle import sisa_oracle as O

pytestmark = pytest.mark.gpu

CHECKS = ("test_schema", "test_faketensor", "test_aot_dispatch_dynamic")


def _layer(dev, B=1, L=130, H=2, seed=3):
    proj, z, lam = O.make_proj_inputs(B, L, H, seed=seed)
    return proj.to(torch.bfloat16).to(dev), z.to(dev), lam.to(dev)


def test_opcheck_layer_ops(cuda_dev):
    from sisa_b200 import ops

    H = 2
    proj, z, lam = _layer(cuda_dev, H=H)
    torch.library.opcheck(torch.ops.sisa_b200.prep_fwd, (proj, z, H), test_utils=CHECKS)
    c_rot, b_rot, pos, tot = ops.prep_fwd(proj, z, H)
    off = ops.fused_layout(H)
    q, k, v = (ops.heads(proj, off[n], H, 64) for n in ("Q", "K", "V"))
    torch.library.opcheck(torch.ops.sisa_b200.attn_fwd, (q, k, v, c_rot, b_rot, pos, lam, True), test_utils=CHECKS)
    o, lse, o32 = ops.attn_fwd(q, k, v, c_rot, b_rot, pos, lam, True)
    dy = torch.randn(proj.shape[0], proj.shape[1], H * 64, device=cuda_dev).to(torch.bfloat16)
    torch.library.opcheck(torch.ops.sisa_b200.fused_bwd, (proj, z, lam, c_rot, b_rot, pos, tot, o, lse, o32, dy, H),
                          test_utils=CHECKS)


def test_opcheck_unfused_ops(cuda_dev):
    from sisa_b200 import ops

    gen = torch.Generator().manual_seed(4)
    B, H, L = 1, 2, 90
    bf = torch.bfloat16
    q, k, v = (torch.randn(B, H, L, 64, generator=gen).to(bf).to(cuda_dev) for _ in range(3))
    c, b = (torch.randn(B, H, L, 32, generator=gen).to(bf).to(cuda_dev) for _ in range(2))
    g = torch.cumsum(-torch.rand(B, H, L, generator=gen) * 0.1, -1).to(cuda_dev)
    f = torch.cumsum(-torch.rand(B, H, L, generator=gen) * 0.1, -1).to(cuda_dev)
    lam = torch.full((H,), 0.4, device=cuda_dev)
    torch.library.opcheck(torch.ops.sisa_b200.pack_positions, (g, f), test_utils=CHECKS)
    pos = ops.pack_positions(g, f)
    o, lse, o32 = ops.attn_fwd(q, k, v, c, b, pos, lam, True)
    do = torch.randn(B, H, L, 64, generator=gen).to(bf).to(cuda_dev)
    torch.library.opcheck(torch.ops.sisa_b200.attn_bwd, (q, k, v, c, b, pos, lam, o, do, lse, o32, True),
                          test_utils=CHECKS)


def test_compiled_fused_layer_matches_eager(cuda_dev):
    from sisa_b200.kernels.fused import sisa_fused

    H = 2
    proj, z, lam = _layer(cuda_dev, B=2, L=200, H=H, seed=9)
    dy = torch.randn(2, 200, H * 64, device=cuda_dev).to(torch.bfloat16)

    def step(p, zz, ll):
        y = sisa_fused(p, zz, ll, H)
        return y.float().mul(dy.float()).sum()

    torch._dynamo.reset()
    compiled = torch.compile(step, fullgraph=True, backend="aot_eager")
    grads = []
    for fn in (step, compiled):
        P, Z, LAM = (t.clone().requires_grad_(True) for t in (proj, z, lam))
        out = fn(P, Z, LAM)
        out.backward()
        grads.append((out.detach(), P.grad, Z.grad, LAM.grad))
    for a, b in zip(grads[0], grads[1]):
        assert torch.equal(a, b)


def test_compiled_linear_ce_matches_eager(cuda_dev):
    from sisa_b200.kernels.linear_ce import linear_cross_entropy

    gen = torch.Generator().manual_seed(2)
    N, D, V = 300, 128, 1000
    h = torch.randn(N, D, generator=gen).to(torch.bfloat16).to(cuda_dev)
    w = (torch.randn(V, D, generator=gen) * 0.05).to(cuda_dev)
    lab = torch.randint(0, V, (N,), generator=gen).to(cuda_dev)

    def f(hh, ww):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            return linear_cross_entropy(hh, ww, lab)

    torch._dynamo.reset()
    compiled = torch.compile(f, fullgraph=True, backend="aot_eager")
    res = []
    for fn in (f, compiled):
        H_, W_ = h.clone().requires_grad_(True), w.clone().requires_grad_(True)
        loss = fn(H_, W_)
        loss.backward()
        res.append((loss.detach(), H_.grad, W_.grad))
    for a, b in zip(res[0], res[1]):
        assert torch.equal(a, b)
