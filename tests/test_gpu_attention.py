"""tcgen05 attention forward/backward (unfused entry point and fused layer) against the fp64 oracle.

Tolerances (bf16 operands): output max-abs <= 2e-2, every gradient ||d - d_ref|| / ||d_ref|| <= 5e-2,
with the truth computed in fp64 from the same bf16-rounded inputs.
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import sisa_oracle as O
from tests.helpers import GRAD_REL, OUT_MAX_ABS, max_abs, rel_err

pytestmark = pytest.mark.gpu


def make_inputs(B, H, L, seed, z_mean=4.0, a_mean=-5.0, lam_raw=-1.0, dtype=torch.bfloat16):
    proj, z, _ = O.make_proj_inputs(B, L, H, seed=seed, z_mean=z_mean, a_mean=a_mean)
    pr = O.prep(proj.to(dtype).double(), z.double(), H)
    lam = F.softplus(torch.full((H,), lam_raw, dtype=torch.float64)) * torch.linspace(0.5, 1.5, H, dtype=torch.float64)
    ins = dict(q=pr["q"].to(dtype), k=pr["k"].to(dtype), v=pr["v"].to(dtype), c=pr["c"].to(dtype),
               b=pr["b"].to(dtype), g=pr["g"].float(), lam=lam.float(), F=pr["F"].float())
    gen = torch.Generator().manual_seed(seed + 1)
    dout = torch.randn(B, H, L, 64, generator=gen).to(dtype)
    return ins, dout


def run_cuda(ins, dout, dev):
    from sisa_b200.kernels.attention import sisa_attention_cuda

    xs = {n: t.to(dev).detach().requires_grad_(True) for n, t in ins.items()}
    o = sisa_attention_cuda(xs["q"], xs["k"], xs["v"], xs["c"], xs["b"], xs["g"], xs["lam"], xs["F"])
    o.backward(dout.to(dev))
    torch.cuda.synchronize()
    return o.detach().cpu(), {"d" + n: xs[n].grad.cpu() for n in xs}


def check(ins, dout, dev, out_tol=OUT_MAX_ABS, grad_tol=GRAD_REL):
    o, grads = run_cuda(ins, dout, dev)
    ref = O.attention_grads(ins["q"], ins["k"], ins["v"], ins["c"], ins["b"], ins["g"], ins["lam"], ins["F"],
                            dout.double())
    assert max_abs(o, ref["o"]) <= out_tol, f"o max abs {max_abs(o, ref['o'])}"
    errs = {n: rel_err(grads[n], ref[n]) for n in ("dq", "dk", "dv", "dc", "db", "dg", "dlam", "dF")}
    bad = {n: e for n, e in errs.items() if not e <= grad_tol}
    assert not bad, f"gradient errors {errs}"
    return errs


@pytest.mark.parametrize("L", [1, 2, 17, 63, 64, 65, 127, 128, 129, 200, 511, 1000])
def test_attention_sweep(cuda_dev, L):
    ins, dout = make_inputs(2, 2, L, seed=100 + L)
    check(ins, dout, cuda_dev)


def test_attention_long(cuda_dev):
    ins, dout = make_inputs(1, 2, 2048, seed=7)
    check(ins, dout, cuda_dev)


@pytest.mark.parametrize("regime", ["strong_forget", "fast_decay", "big_lambda"])
def test_attention_stress(cuda_dev, regime):
    kw = dict(strong_forget=dict(z_mean=-2.0), fast_decay=dict(a_mean=-0.5), big_lambda=dict(lam_raw=2.5))[regime]
    ins, dout = make_inputs(1, 3, 300, seed=9, **kw)
    check(ins, dout, cuda_dev)


def test_attention_fp16(cuda_dev):
    ins, dout = make_inputs(1, 2, 257, seed=5, dtype=torch.float16)
    check(ins, dout, cuda_dev)


def test_attention_deterministic(cuda_dev):
    ins, dout = make_inputs(2, 2, 333, seed=3)
    o1, g1 = run_cuda(ins, dout, cuda_dev)
    o2, g2 = run_cuda(ins, dout, cuda_dev)
    assert torch.equal(o1, o2)
    for n in g1:
        assert torch.equal(g1[n], g2[n]), n


def test_attention_noncontiguous_views_bitwise(cuda_dev):
    """(B, L, H, 64).transpose(1, 2) views give bit-identical results to contiguous inputs."""
    from sisa_b200.kernels.attention import sisa_attention_cuda

    ins, dout = make_inputs(2, 3, 150, seed=4)
    dev = cuda_dev
    cont = {n: t.to(dev) for n, t in ins.items()}
    view = dict(cont)
    for n in ("q", "k", "v", "c", "b"):
        view[n] = cont[n].transpose(1, 2).contiguous().transpose(1, 2)
        assert not view[n].is_contiguous()
    o1 = sisa_attention_cuda(*(cont[n] for n in ("q", "k", "v", "c", "b", "g", "lam", "F")))
    o2 = sisa_attention_cuda(*(view[n] for n in ("q", "k", "v", "c", "b", "g", "lam", "F")))
    assert torch.equal(o1, o2)


def test_attention_causal(cuda_dev):
    """Changing keys after position t leaves outputs up to t unchanged (bitwise)."""
    from sisa_b200.kernels.attention import sisa_attention_cuda

    ins, _ = make_inputs(1, 2, 200, seed=8)
    dev = cuda_dev
    a = {n: t.to(dev) for n, t in ins.items()}
    b = {n: t.clone() for n, t in a.items()}
    b["k"][:, :, 150:] = torch.randn_like(b["k"][:, :, 150:])
    b["v"][:, :, 150:] = torch.randn_like(b["v"][:, :, 150:])
    names = ("q", "k", "v", "c", "b", "g", "lam", "F")
    o1 = sisa_attention_cuda(*(a[n] for n in names))
    o2 = sisa_attention_cuda(*(b[n] for n in names))
    assert torch.equal(o1[:, :, :150], o2[:, :, :150])


@pytest.mark.parametrize("L,H", [(1, 2), (65, 2), (130, 3), (700, 2)])
def test_fused_layer_grads(cuda_dev, L, H):
    from sisa_b200.kernels.fused import sisa_fused

    proj, z, lam = O.make_proj_inputs(2, L, H, seed=L + H)
    proj = proj.to(torch.bfloat16)
    lam = lam * torch.linspace(0.5, 2.0, H)
    gen = torch.Generator().manual_seed(1)
    dy = torch.randn(2, L, H * 64, generator=gen).to(torch.bfloat16)
    P = proj.to(cuda_dev).requires_grad_(True)
    Z = z.to(cuda_dev).requires_grad_(True)
    LAM = lam.to(cuda_dev).requires_grad_(True)
    y = sisa_fused(P, Z, LAM, H)
    y.backward(dy.to(cuda_dev))
    torch.cuda.synchronize()
    # truth: fp64 with c~/b~ rounded to bf16 before the attention, as the reference's torch glue does
    y64, dproj64, dz64, dlam64 = O.fused_layer_grads(proj.double(), z.double(), lam.double(), H, dy.double(),
                                                     lowp=torch.bfloat16)
    assert max_abs(y.cpu(), y64) <= OUT_MAX_ABS
    off = O.fused_layout(H)
    dP = P.grad.cpu()
    for name, w in (("Q", 64), ("K", 64), ("V", 64), ("B", 32), ("C", 32), ("TH", 16), ("A", 1)):
        sl = slice(off[name], off[name] + H * w)
        assert rel_err(dP[..., sl], dproj64[..., sl]) <= GRAD_REL, name
    assert bool((dP[..., off["NTOT"]:] == 0).all())
    assert rel_err(Z.grad.cpu(), dz64) <= GRAD_REL
    assert rel_err(LAM.grad.cpu(), dlam64) <= GRAD_REL
