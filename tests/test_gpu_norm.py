"""Fused RMSNorm / SwiGLU kernels against the eager fp32 formulas (reference: src/sisa/modeling.py:26-49)."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _dev():
    from sisa_b200 import backends

    ok, why = backends.cuda_status(0)
    if not ok:
        pytest.fail(f"sisa_b200 CUDA kernels unavailable: {why}")
    return torch.device("cuda", 0)


def _ref_rms(x, w, eps):
    norm = torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + eps)
    return ((x.float() * norm) * w.float()).to(x.dtype)


@pytest.mark.parametrize("rows,d,dtype,pad", [(1, 768, torch.float32, 0), (333, 768, torch.float32, 0),
                                              (257, 100, torch.float32, 12), (64, 1024, torch.bfloat16, 0),
                                              (50, 37, torch.bfloat16, 5)])
def test_rms_norm_matches_eager(rows, d, dtype, pad):
    from sisa_b200.kernels.norm import rms_norm

    dev = _dev()
    g = torch.Generator(device=dev).manual_seed(rows + d)
    base = torch.randn((rows, d + pad), generator=g, device=dev) * 3
    x = base[:, :d].to(dtype)                       # row stride d + pad
    w = (torch.rand((d,), generator=g, device=dev) + 0.5)
    dy = torch.randn((rows, d), generator=g, device=dev).to(dtype)
    xr = x.detach().clone().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    yr = _ref_rms(xr.float(), wr, 1e-6)
    yr.backward(dy.float())
    xk = x.detach().clone().requires_grad_(True)
    wk = w.detach().clone().requires_grad_(True)
    yk = rms_norm(xk, wk, 1e-6)
    assert yk.dtype == dtype and yk.shape == x.shape
    yk.backward(dy)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert torch.allclose(yk.float(), yr.to(dtype).float(), rtol=tol, atol=tol)
    assert torch.allclose(xk.grad.float(), xr.grad.float(), rtol=1e-3 if dtype == torch.float32 else 2e-2,
                          atol=1e-4 if dtype == torch.float32 else 2e-2)
    assert torch.allclose(wk.grad, wr.grad, rtol=1e-4, atol=1e-3)
    # dw comes from a fixed reduction order: bitwise repeatable
    wk2 = w.detach().clone().requires_grad_(True)
    rms_norm(x.detach(), wk2, 1e-6).backward(dy)
    assert torch.equal(wk2.grad, wk.grad)


@pytest.mark.parametrize("rows,f,dtype", [(1, 2744, torch.bfloat16), (129, 2744, torch.bfloat16),
                                          (77, 37, torch.bfloat16), (40, 24, torch.float32)])
def test_swiglu_matches_eager(rows, f, dtype):
    from sisa_b200.kernels.norm import swiglu

    dev = _dev()
    gen = torch.Generator(device=dev).manual_seed(rows * 7 + f)
    g = (torch.randn((rows, f), generator=gen, device=dev) * 3).to(dtype)
    u = torch.randn((rows, f), generator=gen, device=dev).to(dtype)
    da = torch.randn((rows, f), generator=gen, device=dev).to(dtype)
    gr = g.detach().float().clone().requires_grad_(True)
    ur = u.detach().float().clone().requires_grad_(True)
    ar = torch.nn.functional.silu(gr) * ur
    ar.backward(da.float())
    gk = g.detach().clone().requires_grad_(True)
    uk = u.detach().clone().requires_grad_(True)
    ak = swiglu(gk, uk)
    ak.backward(da)
    assert ak.dtype == dtype
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert torch.allclose(ak.float(), ar, rtol=tol, atol=tol)
    assert torch.allclose(gk.grad.float(), gr.grad, rtol=tol, atol=tol)
    assert torch.allclose(uk.grad.float(), ur.grad, rtol=tol, atol=tol)


def test_model_blocks_use_the_fused_kernels_on_the_cuda_path():
    """attn_impl="cuda" routes the norms and the SwiGLU activation through kernels/norm.py; "torch" does not."""
    import sisa_b200 as sisa
    from sisa_b200 import modeling

    dev = _dev()
    cfg = sisa.SISAConfig.preset("sisa-152m", attn_impl="cuda")
    x = torch.randn((2, 8, cfg.d_model), device=dev)
    assert modeling._fused_kernels(x, cfg)
    cfg_t = sisa.SISAConfig.preset("sisa-152m", attn_impl="torch")
    assert not modeling._fused_kernels(x, cfg_t)
    assert not modeling._fused_kernels(x.cpu(), cfg)
