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


def _ref_block(x, res, w, pw, pb, eps, out_dtypes):
    """Eager reference of the block boundary: residual add, RMSNorm (modeling.py:25-36), the casts of
    the consumers and the fp32 forget projection (modeling.py:167-168)."""
    v = x + res if res is not None else x
    vf = v.float()
    h = ((vf * torch.rsqrt(vf.pow(2).mean(-1, keepdim=True) + eps)) * w.float()).to(v.dtype)
    ys = [h.to(dt) for dt in out_dtypes]
    z = torch.nn.functional.linear(h.float(), pw.float(), pb.float()) if pw is not None else None
    return v, ys, z


@pytest.mark.parametrize("rows,d,xdt,with_res,n_out,n_proj", [
    (300, 768, torch.float32, True, 1, 12),     # the attention norm of a cfg3 block
    (300, 768, torch.float32, True, 2, 0),      # the SwiGLU norm
    (129, 768, torch.float32, False, 1, 12),    # the first block (no residual add)
    (77, 100, torch.float32, True, 2, 3),       # d not a multiple of 4: scalar path
    (64, 256, torch.bfloat16, True, 1, 16),     # bf16 residual stream
    (300, 768, torch.bfloat16, True, 1, 12),    # the inference model's attention norm (staged kernel)
    (300, 768, torch.bfloat16, True, 1, 0),     # and its SwiGLU norm
    (129, 768, torch.bfloat16, False, 1, 12),   # its first block
    (33, 1280, torch.float32, True, 1, 20),     # row not cached in registers, 32 projection slots
])
def test_block_norm_matches_eager(rows, d, xdt, with_res, n_out, n_proj):
    from sisa_b200.kernels.norm import block_norm

    dev = _dev()
    gen = torch.Generator(device=dev).manual_seed(rows * 3 + d)
    rnd = lambda *s, sc=1.0: torch.randn(s, generator=gen, device=dev) * sc
    x = rnd(2, rows, d, sc=2.0).to(xdt)
    res = rnd(2, rows, d).to(torch.bfloat16) if with_res else None
    w = torch.rand((d,), generator=gen, device=dev) + 0.5
    pw = rnd(n_proj, d, sc=0.05) if n_proj else None
    pb = rnd(n_proj) if n_proj else None
    out_dtypes = (torch.bfloat16,) * n_out
    leaves = [t for t in (x, res, w, pw, pb) if t is not None]
    ref_in = [t.detach().clone().requires_grad_(True) for t in leaves]
    ker_in = [t.detach().clone().requires_grad_(True) for t in leaves]

    def unpack(ins):
        it = iter(ins)
        xx = next(it)
        rr = next(it) if with_res else None
        ww = next(it)
        pp = (next(it), next(it)) if n_proj else (None, None)
        return xx, rr, ww, pp

    xr, rr, wr, (pwr, pbr) = unpack(ref_in)
    v_ref, ys_ref, z_ref = _ref_block(xr, rr, wr, pwr, pbr, 1e-6, out_dtypes)
    xk, rk, wk, (pwk, pbk) = unpack(ker_in)
    outs = block_norm(xk, wk, 1e-6, res=rk, out_dtypes=out_dtypes, proj=(pwk, pbk) if n_proj else None)
    ref_outs = ([v_ref] if with_res else []) + ys_ref + ([z_ref] if n_proj else [])
    chk_outs = list(ref_outs)
    if n_proj and xdt != torch.float32:
        # a 16-bit stream rounds h to it before the projection; a one-ulp difference of the row's rstd
        # (summation order) can flip such a rounding, so z is checked against the projection of the
        # kernel's own rounded h (its last normalised output), and h against the reference at bf16
        # tolerance
        chk_outs[-1] = torch.nn.functional.linear(outs[-2].detach().float(), pwr.detach().float(),
                                                  pbr.detach().float())
    assert len(outs) == len(ref_outs)
    for o, r in zip(outs, chk_outs):
        assert o.dtype == r.dtype and o.shape == r.shape
        tol = 1e-5 if o.dtype == torch.float32 else 1e-2
        assert torch.allclose(o.float(), r.float(), rtol=tol, atol=tol)
    # independent upstream gradients for every output
    gouts = [rnd(*o.shape).to(o.dtype) for o in outs]
    torch.autograd.backward(ref_outs, gouts)
    torch.autograd.backward(list(outs), gouts)
    for a, b in zip(ker_in, ref_in):
        assert a.grad is not None and a.grad.dtype == b.grad.dtype
        lowp = a.grad.dtype != torch.float32 or xdt != torch.float32
        tol = 3e-2 if lowp else 2e-4
        err = (a.grad.float() - b.grad.float()).abs().max().item()
        assert err <= tol * (1 + b.grad.float().abs().max().item()), (tuple(a.shape), err)


def test_block_norm_weight_gradients_repeatable():
    from sisa_b200.kernels.norm import block_norm

    dev = _dev()
    gen = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn((4096, 768), generator=gen, device=dev)
    res = torch.randn((4096, 768), generator=gen, device=dev).to(torch.bfloat16)
    w = torch.rand((768,), generator=gen, device=dev)
    pw = torch.randn((12, 768), generator=gen, device=dev) * 0.05
    pb = torch.randn((12,), generator=gen, device=dev)
    gs = None
    grads = []
    for _ in range(2):
        ins = [t.detach().clone().requires_grad_(True) for t in (w, pw, pb)]
        outs = block_norm(x, ins[0], 1e-6, res=res, out_dtypes=(torch.bfloat16,), proj=(ins[1], ins[2]))
        if gs is None:
            gs = [torch.randn(o.shape, generator=gen, device=dev).to(o.dtype) for o in outs]
        torch.autograd.backward(list(outs), gs)
        grads.append([t.grad for t in ins])
    for a, b in zip(*grads):
        assert torch.equal(a, b)
