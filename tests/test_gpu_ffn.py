"""The SwiGLU gate/up GEMM with the activation in its epilogue (``sisa_gemm_swiglu``, kernels/ffn.py)
and the projection GEMM's bias epilogue, against the same computation split into its plain parts and
against fp64."""
from __future__ import annotations

import pytest
import torch

from tests.helpers import GRAD_REL, rel_err

pytestmark = pytest.mark.gpu


def _case(rows, d, d_ff, seed, dev):
    gen = torch.Generator().manual_seed(seed)
    h = torch.randn(rows, d, generator=gen).to(torch.bfloat16).to(dev)
    wg = (torch.randn(d_ff, d, generator=gen) * 0.05).to(dev)
    wu = (torch.randn(d_ff, d, generator=gen) * 0.05).to(dev)
    return h, wg, wu


@pytest.mark.parametrize("rows,d,d_ff", [(300, 768, 2744), (4096, 768, 2744), (77, 128, 40), (600, 256, 512)])
def test_gate_up_epilogue_matches_split_computation(cuda_dev, monkeypatch, rows, d, d_ff):
    """gu and a from the fused kernel equal the same GEMM's plain output and the separate SwiGLU kernel
    applied to it, bit for bit."""
    from types import SimpleNamespace

    from sisa_b200.kernels.ffn import gate_up_swiglu, interleave_gate_up
    from sisa_b200.kernels.gemm import matmul_t
    from sisa_b200.kernels.norm import swiglu

    monkeypatch.setenv("SISA_GEMM_TILE", "narrow")           # the fused kernel's tile shape
    h, wg, wu = _case(rows, d, d_ff, rows + d_ff, cuda_dev)
    owner = SimpleNamespace()
    a = gate_up_swiglu(h, wg, wu, torch.bfloat16, owner)
    w_il = interleave_gate_up(wg, wu, torch.bfloat16)
    gu = matmul_t(h, w_il, out_dtype=torch.bfloat16)
    blocks = gu.view(rows, d_ff // 8, 2, 8)
    g = blocks[:, :, 0].reshape(rows, d_ff)
    u = blocks[:, :, 1].reshape(rows, d_ff)
    with torch.no_grad():
        a_ref = swiglu(g.contiguous(), u.contiguous())
    torch.cuda.synchronize()
    assert torch.equal(a, a_ref)
    assert torch.equal(owner._gate_up_il[1], w_il)


def test_gate_up_gradients_against_fp64(cuda_dev):
    from types import SimpleNamespace

    from sisa_b200.kernels.ffn import gate_up_swiglu

    rows, d, d_ff = 1000, 256, 520
    h, wg, wu = _case(rows, d, d_ff, 5, cuda_dev)
    H, WG, WU = (t.clone().requires_grad_(True) for t in (h, wg, wu))
    a = gate_up_swiglu(H, WG, WU, torch.bfloat16, SimpleNamespace())
    da = torch.randn(rows, d_ff, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16).to(cuda_dev)
    (a.float() * da.float()).sum().backward()
    # fp64 truth on the bf16-rounded operands
    h64, wg64, wu64 = (t.detach().double().requires_grad_(True) for t in (h, wg.to(torch.bfloat16),
                                                                           wu.to(torch.bfloat16)))
    g64, u64 = h64 @ wg64.t(), h64 @ wu64.t()
    a64 = torch.nn.functional.silu(g64) * u64
    (a64 * da.double()).sum().backward()
    assert rel_err(a.float(), a64.detach()) <= 1e-2
    assert H.grad.dtype == torch.bfloat16 and WG.grad.dtype == torch.float32
    assert rel_err(H.grad.float(), h64.grad) <= GRAD_REL
    assert rel_err(WG.grad, wg64.grad) <= GRAD_REL
    assert rel_err(WU.grad, wu64.grad) <= GRAD_REL


def test_gate_up_weight_cache_follows_the_weights(cuda_dev):
    from types import SimpleNamespace

    from sisa_b200.kernels.ffn import gate_up_swiglu

    h, wg, wu = _case(256, 128, 64, 7, cuda_dev)
    owner = SimpleNamespace()
    with torch.no_grad():                                       # inference: the versions decide
        a1 = gate_up_swiglu(h, wg, wu, torch.bfloat16, owner)
        first = owner._gate_up_il[1]
        a2 = gate_up_swiglu(h, wg, wu, torch.bfloat16, owner)
        assert owner._gate_up_il[1] is first and torch.equal(a1, a2)
        wg.mul_(2.0)                                            # an in-place update bumps the version
        a3 = gate_up_swiglu(h, wg, wu, torch.bfloat16, owner)
        assert owner._gate_up_il[1] is not first and not torch.equal(a1, a3)
    # with gradients the copy is rebuilt on every call: an update that leaves the version alone (a fused
    # optimizer's) is seen too
    WU = wu.clone().requires_grad_(True)
    a4 = gate_up_swiglu(h, wg, WU, torch.bfloat16, owner)
    WU.data.mul_(0.5)
    a5 = gate_up_swiglu(h, wg, WU, torch.bfloat16, owner)
    with torch.no_grad():
        a6 = gate_up_swiglu(h, wg, wu * 0.5, torch.bfloat16, SimpleNamespace())
    assert torch.equal(a4.detach(), a3) and torch.equal(a5.detach(), a6)


def test_fused_block_uses_the_gate_up_kernel_and_matches_split_block(cuda_dev):
    """One block on the fused path (gate/up GEMM) against the same block with the split MLP path, under
    bf16 autocast: outputs and gradients agree within bf16 tolerance."""
    import sisa_b200 as sisa
    from sisa_b200.modeling import SISABlock

    cfg = sisa.SISAConfig(d_model=256, n_head=4, d_ff=520, n_layer=1, vocab_size=64, attn_impl="cuda")
    torch.manual_seed(0)
    blk = SISABlock(cfg).to(cuda_dev)
    x = torch.randn(2, 160, 256, device=cuda_dev)
    outs = []
    for fused in (True, False):
        import sisa_b200.kernels.ffn as ffn_mod

        orig = ffn_mod.supports
        if not fused:
            ffn_mod.supports = lambda *a, **k: False
        try:
            X = x.clone().requires_grad_(True)
            blk.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                xs, f = blk.forward_pair(X, None)
            ((xs + f).float().square().mean()).backward()
            outs.append((xs.detach().float(), f.detach().float(), X.grad.clone(), blk.ffn.w_gate.weight.grad.clone()))
        finally:
            ffn_mod.supports = orig
    for a, b in zip(outs[0], outs[1]):
        assert rel_err(a, b) <= 2e-2


def test_linear_cast_matches_autocast_linear(cuda_dev):
    """W_O / w_down: the output and dx equal autocast's F.linear bit for bit (the same bf16 GEMM); dW is
    the same product accumulated to fp32 instead of rounded to bf16 first, and the weight copy is kept
    while the weight is unchanged."""
    from types import SimpleNamespace

    from sisa_b200.kernels.linear import linear_cast

    gen = torch.Generator().manual_seed(12)
    x = torch.randn(4, 300, 768, generator=gen).to(torch.bfloat16).to(cuda_dev)
    w = (torch.randn(768, 768, generator=gen) * 0.02).to(cuda_dev)
    dy = torch.randn(4, 300, 768, generator=gen).to(torch.bfloat16).to(cuda_dev)
    owner = SimpleNamespace()
    X1, W1 = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    y1 = linear_cast(X1, W1, torch.bfloat16, owner, "W")
    y1.backward(dy)
    X2, W2 = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y2 = torch.nn.functional.linear(X2, W2)
    y2.backward(dy)
    assert y1.dtype == y2.dtype == torch.bfloat16
    assert torch.equal(y1, y2)
    assert torch.equal(X1.grad, X2.grad)
    assert W1.grad.dtype == torch.float32
    ref = (dy.double().reshape(-1, 768).t() @ x.double().reshape(-1, 768)).float()
    assert rel_err(W1.grad, ref) <= 1e-5
    assert rel_err(W2.grad, ref) <= 1e-2                       # autocast's bf16 dW, for scale
    with torch.no_grad():                                       # inference: kept while W is unchanged
        linear_cast(x, W1, torch.bfloat16, owner, "W")
        first = owner._lp_W[1]
        linear_cast(x, W1, torch.bfloat16, owner, "W")
    assert owner._lp_W[1] is first


def test_gate_up_inference_stores_only_the_activation(cuda_dev):
    """Without a gradient to compute the fused GEMM stores only a: bit for bit the training forward's a."""
    from types import SimpleNamespace

    from sisa_b200.kernels.ffn import gate_up_swiglu

    h, wg, wu = _case(1000, 768, 2744, 11, cuda_dev)
    with torch.no_grad():
        a_inf = gate_up_swiglu(h, wg, wu, torch.bfloat16, SimpleNamespace())
    a_tr = gate_up_swiglu(h, wg.clone().requires_grad_(True), wu, torch.bfloat16, SimpleNamespace())
    torch.cuda.synchronize()
    assert a_tr.requires_grad and torch.equal(a_inf, a_tr.detach())
