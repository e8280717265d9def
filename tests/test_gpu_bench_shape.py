"""The fused layer at the benchmarked shapes (T=4096), where the attention kernels' work order takes
both branches of its head-group mapping.

The attention kernels order their tiles in groups of 16 (batch, head) units: a launch with B*H >= 16
maps most of its grid through the full-group branch and the rest through the remainder branch. The
small-shape parity tests never reach the first. Here:

* B=1, H=18 (one full group of 16 and a remainder of 2) and B=8, H=16 (cfg1: eight full groups).
* Every head of the full-shape run must be bitwise equal to the same head run alone (B unchanged,
  H=1, whose grid has a single remainder group). The kernels are deterministic and each head's
  arithmetic does not depend on where its tiles sit in the grid, so any dropped, duplicated or
  misplaced tile shows up as a difference.
* Selected (batch, head) units are checked against the fp64 oracle with the parity tolerances of
  tests/helpers.py (output max-abs, relative L2 error of every d_proj column group, dz and dlam),
  on the benchmark's input distributions.
"""
from __future__ import annotations

import pytest
import torch

from oracle import sisa_oracle as O
from tests.helpers import GRAD_REL, OUT_MAX_ABS, max_abs, rel_err

pytestmark = pytest.mark.gpu

L_BENCH = 4096
GROUPS = (("Q", 64), ("K", 64), ("V", 64), ("B", 32), ("C", 32), ("TH", 16), ("A", 1))


def _inputs(B, H, L, seed):
    proj, z, lam = O.make_proj_inputs(B, L, H, seed=seed)
    lam = lam * torch.linspace(0.5, 1.5, H)
    gen = torch.Generator().manual_seed(seed + 1)
    dy = torch.randn(B, L, H * 64, generator=gen).to(torch.bfloat16)
    return proj.to(torch.bfloat16), z, lam, dy


def _head_slice(proj, z, lam, dy, H, h):
    """The inputs of head h alone, as a one-head fused layer (its own column layout)."""
    B, L, _ = proj.shape
    off, off1 = O.fused_layout(H), O.fused_layout(1)
    p1 = torch.zeros(B, L, off1["NPAD"], dtype=proj.dtype, device=proj.device)
    for name, w in GROUPS:
        p1[..., off1[name]:off1[name] + w] = proj[..., off[name] + h * w:off[name] + (h + 1) * w]
    return p1, z[..., h:h + 1].contiguous(), lam[h:h + 1].contiguous(), dy[..., h * 64:(h + 1) * 64].contiguous()


def _run(proj, z, lam, dy, H, dev):
    from sisa_b200.kernels.fused import sisa_fused

    P = proj.to(dev).requires_grad_(True)
    Z = z.to(dev).requires_grad_(True)
    LAM = lam.to(dev).requires_grad_(True)
    y = sisa_fused(P, Z, LAM, H)
    y.backward(dy.to(dev))
    torch.cuda.synchronize()
    return y.detach(), P.grad, Z.grad, LAM.grad


def _check_heads_bitwise(B, H, seed, dev):
    proj, z, lam, dy = _inputs(B, H, L_BENCH, seed)
    y, dP, dZ, dLAM = _run(proj, z, lam, dy, H, dev)
    off, off1 = O.fused_layout(H), O.fused_layout(1)
    for h in range(H):
        y1, dP1, dZ1, dLAM1 = _run(*_head_slice(proj, z, lam, dy, H, h), 1, dev)
        assert torch.equal(y[..., h * 64:(h + 1) * 64], y1), f"head {h}: y"
        for name, w in GROUPS:
            full = dP[..., off[name] + h * w:off[name] + (h + 1) * w]
            assert torch.equal(full, dP1[..., off1[name]:off1[name] + w]), f"head {h}: d_proj {name}"
        assert torch.equal(dZ[..., h], dZ1[..., 0]), f"head {h}: dz"
        assert torch.equal(dLAM[h], dLAM1[0]), f"head {h}: dlam"
    assert bool((dP[..., off["NTOT"]:] == 0).all())
    return proj, z, lam, dy, (y.cpu(), dP.cpu(), dZ.cpu(), dLAM.cpu())


def _check_unit_oracle(proj, z, lam, dy, H, b, h, got, check_dlam):
    """fp64 truth of (batch b, head h) with c~/b~ rounded to bf16 as the reference's glue does."""
    y, dP, dZ, dLAM = got
    p1, z1, lam1, dy1 = _head_slice(proj[b:b + 1], z[b:b + 1], lam, dy[b:b + 1], H, h)
    y64, dp64, dz64, dlam64 = O.fused_layer_grads(p1.double(), z1.double(), lam1.double(), 1, dy1.double(),
                                                  lowp=torch.bfloat16)
    off, off1 = O.fused_layout(H), O.fused_layout(1)
    assert max_abs(y[b:b + 1, :, h * 64:(h + 1) * 64], y64) <= OUT_MAX_ABS, (b, h)
    for name, w in GROUPS:
        g = dP[b:b + 1, :, off[name] + h * w:off[name] + (h + 1) * w]
        assert rel_err(g, dp64[..., off1[name]:off1[name] + w]) <= GRAD_REL, (b, h, name)
    assert rel_err(dZ[b:b + 1, :, h:h + 1], dz64) <= GRAD_REL, (b, h)
    if check_dlam:
        assert rel_err(dLAM[h:h + 1], dlam64) <= GRAD_REL, (b, h)


def test_bench_shape_one_full_group_and_remainder(cuda_dev):
    """B=1, H=18, T=4096: heads 0-15 take the full-group branch, heads 16-17 the remainder."""
    B, H = 1, 18
    proj, z, lam, dy, got = _check_heads_bitwise(B, H, seed=41, dev=cuda_dev)
    for h in (5, 17):   # one head of each branch; with B=1 the unit's dlam is the head's dlam
        _check_unit_oracle(proj, z, lam, dy, H, 0, h, got, check_dlam=True)


def test_bench_shape_cfg1(cuda_dev):
    """B=8, H=16, T=4096: every head bitwise equal to its own run, two units
    against fp64."""
    B, H = 8, 16
    proj, z, lam, dy, got = _check_heads_bitwise(B, H, seed=43, dev=cuda_dev)
    for b, h in ((0, 0), (7, 13)):
        _check_unit_oracle(proj, z, lam, dy, H, b, h, got, check_dlam=False)
