"""Fused preparation kernel (sisa_prep_fwd) against the fp64 oracle, through the C ABI."""
from __future__ import annotations

import pytest
import torch

from oracle import sisa_oracle as O
from sisa_b200 import _lib
from tests.helpers import PREP_SCAN_REL, rel_err

pytestmark = pytest.mark.gpu


def _run(B, L, H, seed, with_z=True, dtype=torch.bfloat16):
    from sisa_b200.kernels.fused import prep_forward

    proj, z, _ = O.make_proj_inputs(B, L, H, seed=seed)
    proj = proj.to(dtype)
    dev = torch.device("cuda", 0)
    c_rot, b_rot, pos, tot = prep_forward(proj.to(dev), z.to(dev) if with_z else None, H)
    torch.cuda.synchronize()
    ref = O.prep(proj.double(), z.double() if with_z else None, H)
    return c_rot.cpu(), b_rot.cpu(), _lib.pos_records(pos, L).cpu(), ref


@pytest.mark.parametrize("L", [1, 2, 63, 64, 65, 130, 1000, 4096])
def test_prep_scans_and_rotation(cuda_dev, L):
    H = 3
    c_rot, b_rot, pos, ref = _run(2, L, H, seed=L)
    g, Fg, rowf, colf = pos[..., 0], pos[..., 1], pos[..., 2], pos[..., 3]
    assert rel_err(g, ref["g"]) <= PREP_SCAN_REL
    assert rel_err(Fg, ref["F"]) <= PREP_SCAN_REL
    assert (g.double() - ref["g"]).abs().max() <= PREP_SCAN_REL * ref["g"].abs().max() + 1e-6
    # one bf16 rounding of an fp32 rotation
    for got, want in ((c_rot, ref["c"]), (b_rot, ref["b"])):
        err = (got.double() - want).abs()
        assert bool((err <= 2.0 ** -8 * want.abs() + 1e-5).all())
    # g is non-increasing (within rounding) and the block factors follow from g
    if L > 1:
        assert float((g[..., 1:] - g[..., :-1]).max()) <= 1e-6
    t = torch.arange(L)
    start = (t // 64) * 64
    end = torch.clamp(start + 63, max=L - 1)
    gs = g.double()[..., start]
    ge = g.double()[..., end]
    assert torch.allclose(rowf.double(), torch.exp(torch.clamp(g.double() - gs, max=0)), rtol=2e-6, atol=1e-7)
    assert torch.allclose(colf.double(), torch.exp(torch.clamp(ge - g.double(), max=0)), rtol=2e-6, atol=1e-7)


def test_prep_without_forget_gate(cuda_dev):
    c_rot, b_rot, pos, ref = _run(1, 100, 2, seed=3, with_z=False)
    assert bool((pos[..., 1] == 0).all())
    assert rel_err(pos[..., 0], ref["g"]) <= PREP_SCAN_REL


def test_prep_fp16(cuda_dev):
    c_rot, b_rot, pos, ref = _run(1, 200, 2, seed=4, dtype=torch.float16)
    assert c_rot.dtype == torch.float16
    err = (c_rot.double() - ref["c"]).abs()
    assert bool((err <= 2.0 ** -10 * ref["c"].abs() + 1e-5).all())
