"""The CTA-pair tcgen05 GEMM (``sisa_gemm``) against an fp64 product of the same bf16/fp16 operands:
both tile shapes (256 x 256 and 256 x 512 pair tiles, forced through ``SISA_GEMM_TILE``), every operand
majorness, ragged M/N/K, the persistent tile loop (more tiles than CTA pairs), long K (the stage ring
wraps many times), fp32 accumulation into C and the rounded bf16/fp16 outputs."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _operands(M, N, K, a_mn, b_mn, dtype, dev, seed):
    gen = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=gen).to(dtype)
    b = torch.randn(N, K, generator=gen).to(dtype)
    # MN-major: store the transpose row-major (row stride padded to whole 16-byte units) and view it back
    def lay(x, mn):
        r, k = x.shape
        if mn:
            pad = -r % 8
            buf = torch.zeros(k, r + pad, dtype=dtype)
            buf[:, :r] = x.t()
            return buf.to(dev)[:, :r].t()
        pad = -k % 8
        buf = torch.zeros(r, k + pad, dtype=dtype)
        buf[:, :k] = x
        return buf.to(dev)[:, :k]
    return a, b, lay(a, a_mn), lay(b, b_mn)


def _check_f32(c, a, b, scale=1e-5):
    ref = a.double() @ b.double().t()
    bound = (a.double().abs() @ b.double().abs().t()) * scale + 1e-30
    err = (c.double().cpu() - ref).abs()
    assert bool((err <= bound).all()), float((err / bound).max())


SHAPES = [(256, 256, 64), (300, 520, 200), (1000, 130, 72), (17, 5, 8), (1, 300, 1000), (260, 1100, 136)]


@pytest.fixture(params=["narrow", "wide"])
def tile(request, monkeypatch):
    monkeypatch.setenv("SISA_GEMM_TILE", request.param)
    return request.param


@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("shape", SHAPES)
def test_gemm_fp32_out_all_majors(cuda_dev, tile, a_mn, b_mn, shape):
    from sisa_b200.kernels.gemm import matmul_t

    M, N, K = shape
    a, b, da, db = _operands(M, N, K, a_mn, b_mn, torch.bfloat16, cuda_dev, seed=M + N + K + 2 * a_mn + b_mn)
    c = matmul_t(da, db)
    torch.cuda.synchronize()
    _check_f32(c, a, b)
    from sisa_b200 import backends
    assert int(backends.status_word(cuda_dev).item()) == 0


def test_gemm_persistent_tiles_and_long_k(cuda_dev, tile):
    from sisa_b200.kernels.gemm import matmul_t

    # 16 x 8 = 128 pair tiles (more than the resident CTA pairs) and 3000 / 64 K stages (the six-stage
    # ring wraps ~8 times per tile)
    for (M, N, K, a_mn, b_mn) in ((4096, 2048, 256, 0, 0), (1024, 512, 3000, 1, 1), (2304, 1280, 1100, 0, 1)):
        a, b, da, db = _operands(M, N, K, a_mn, b_mn, torch.bfloat16, cuda_dev, seed=K)
        c = matmul_t(da, db)
        torch.cuda.synchronize()
        _check_f32(c, a, b)


def test_gemm_accumulate_and_strided_output(cuda_dev, tile):
    from sisa_b200.kernels.gemm import matmul_t

    M, N, K = 700, 600, 130
    a, b, da, db = _operands(M, N, K, 1, 1, torch.bfloat16, cuda_dev, seed=5)
    base = torch.randn(M, N + 12, generator=torch.Generator().manual_seed(6))
    out = base.clone().to(cuda_dev)
    view = out[:, 4:4 + N]
    matmul_t(da, db, view, accumulate=True)
    torch.cuda.synchronize()
    got = out.cpu()
    assert torch.equal(got[:, :4], base[:, :4]) and torch.equal(got[:, 4 + N:], base[:, 4 + N:])
    ref = base[:, 4:4 + N].double() + a.double() @ b.double().t()
    bound = (a.double().abs() @ b.double().abs().t() + base[:, 4:4 + N].double().abs()) * 1e-5
    assert bool(((got[:, 4:4 + N].double() - ref).abs() <= bound).all())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gemm_low_precision_out_rounds_once(cuda_dev, tile, dtype):
    from sisa_b200.kernels.gemm import matmul_t

    M, N, K = 520, 300, 264
    a, b, da, db = _operands(M, N, K, 0, 1, dtype, cuda_dev, seed=11)
    c32 = matmul_t(da, db)
    c = matmul_t(da, db, out_dtype=dtype)
    torch.cuda.synchronize()
    assert c.dtype == dtype
    # the low-precision output is the fp32 result rounded once (ties may differ only where the fp32
    # results themselves differ, which they do not: same kernel, same order)
    assert torch.equal(c, c32.to(dtype))
    _check_f32(c32, a, b)


def test_gemm_matches_torch_mm_within_fp32_order(cuda_dev):
    """The same product as torch.mm with an fp32 output (cuBLAS), up to summation order."""
    from sisa_b200.kernels.gemm import matmul_t

    gen = torch.Generator().manual_seed(8)
    G = torch.randn(1024, 2560, generator=gen).to(torch.bfloat16).to(cuda_dev)
    W = torch.randn(2560, 512, generator=gen).to(torch.bfloat16).to(cuda_dev)
    X = torch.randn(1024, 512, generator=gen).to(torch.bfloat16).to(cuda_dev)
    dx = matmul_t(G, W.t())                   # A K-major, B MN-major
    dw = matmul_t(G.t(), X.t())               # both MN-major
    ref_dx = torch.mm(G, W, out_dtype=torch.float32)
    ref_dw = torch.mm(G.t(), X, out_dtype=torch.float32)
    torch.testing.assert_close(dx, ref_dx, rtol=1e-4, atol=1e-3)
    torch.testing.assert_close(dw, ref_dw, rtol=1e-4, atol=1e-3)


def test_gemm_argument_errors(cuda_dev):
    from sisa_b200.kernels.gemm import matmul_t

    a = torch.randn(64, 70, device=cuda_dev).to(torch.bfloat16)[:, :66]   # row stride 70: not 16-byte units
    b = torch.randn(64, 66, device=cuda_dev).to(torch.bfloat16)
    with pytest.raises(ValueError):
        matmul_t(a, b)
    with pytest.raises(TypeError):
        matmul_t(b, b.half())
    out = torch.empty(64, 64, device=cuda_dev, dtype=torch.bfloat16)
    bb = torch.randn(64, 64, device=cuda_dev).to(torch.bfloat16)
    with pytest.raises(ValueError):
        matmul_t(bb, bb, out, accumulate=True)


@pytest.mark.parametrize("M,N,K,a_mn,b_mn", [(1040, 768, 8192, 1, 1), (768, 768, 16384, 1, 1), (300, 200, 5000, 0, 0),
                                             (520, 300, 3000, 1, 0)])
def test_gemm_split_k_is_ordered_and_deterministic(cuda_dev, monkeypatch, M, N, K, a_mn, b_mn):
    """Small fp32 problems with long K split K across CTA pairs; the slices add into C in a fixed order,
    so repeated runs agree bit for bit, and the result matches fp64 within fp32 summation error."""
    from sisa_b200.kernels.gemm import matmul_t

    monkeypatch.delenv("SISA_GEMM_TILE", raising=False)
    a, b, da, db = _operands(M, N, K, a_mn, b_mn, torch.bfloat16, cuda_dev, seed=M + K)
    c1 = matmul_t(da, db)
    c2 = matmul_t(da, db)
    base = torch.randn(M, N, generator=torch.Generator().manual_seed(1)).to(cuda_dev)
    c3 = base.clone()
    matmul_t(da, db, c3, accumulate=True)
    torch.cuda.synchronize()
    assert torch.equal(c1, c2)
    _check_f32(c1, a, b)
    ref = base.double().cpu() + a.double() @ b.double().t()
    bound = (a.double().abs() @ b.double().abs().t() + base.double().cpu().abs()) * 1e-5
    assert bool(((c3.double().cpu() - ref).abs() <= bound).all())
    monkeypatch.setenv("SISA_GEMM_TILE", "narrow")            # one slice: the same product, another order
    c4 = matmul_t(da, db)
    torch.cuda.synchronize()
    _check_f32(c4, a, b)
    from sisa_b200 import backends
    assert int(backends.status_word(cuda_dev).item()) == 0


@pytest.mark.parametrize("bias_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_gemm_bias_epilogue(cuda_dev, tile, bias_dtype, out_dtype):
    from sisa_b200.kernels.gemm import matmul_t

    M, N, K = 600, 3280, 768
    a, b, da, db = _operands(M, N, K, 0, 0, torch.bfloat16, cuda_dev, seed=21)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(22)).to(bias_dtype)
    c = matmul_t(da, db, out_dtype=out_dtype, bias=bias.to(cuda_dev))
    c32 = matmul_t(da, db)
    torch.cuda.synchronize()
    want = c32.cpu() + bias.float()                          # the fp32 result plus the bias, rounded once
    assert torch.equal(c.cpu(), want.to(out_dtype))


@pytest.mark.parametrize("dtype,bias_dtype,rnd", [(torch.bfloat16, torch.float32, True),
                                                  (torch.bfloat16, torch.bfloat16, False),
                                                  (torch.float16, torch.float32, True)])
@pytest.mark.parametrize("col0,n", [(0, 3280), (3100, 12), (248, 16), (1000, 0)])
def test_gemm_bias_columns(cuda_dev, tile, dtype, bias_dtype, rnd, col0, n):
    """``sisa_gemm_bias_cols``: a bias over columns [col0, col0 + n) only (the fused projection's alpha
    bias), optionally rounded to the output type first, equals the fp32 product plus that bias rounded
    once; ranges on and off 8-column boundaries, across a tile edge, and empty."""
    from sisa_b200.kernels.gemm import matmul_t

    M, N, K = 600, 3280, 768
    a, b, da, db = _operands(M, N, K, 0, 0, dtype, cuda_dev, seed=23)
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(24)) * 3).to(bias_dtype)
    c = matmul_t(da, db, out_dtype=dtype, bias=bias.to(cuda_dev), bias_col0=col0, bias_round=rnd)
    c32 = matmul_t(da, db)
    torch.cuda.synchronize()
    full = torch.zeros(N)
    full[col0:col0 + n] = bias.to(dtype).float() if rnd else bias.float()
    want = (c32.cpu() + full).to(dtype)
    assert torch.equal(c.cpu(), want)
    from sisa_b200 import backends
    assert int(backends.status_word(cuda_dev).item()) == 0
