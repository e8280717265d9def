"""The allocation-free decode entry point, sisa_decode_attn_noalloc, against sisa_decode_attn.

Some callers cannot allocate device memory at the moment they decode: host programs that bind only
the C ABI and have no device allocator of their own, and serving loops held to a fixed, pre-reserved
memory budget. For them the library keeps the decode kernel's split-K scratch in a fixed array of
its own, and the caller passes only inputs and outputs. These tests call both entry points through
the C ABI and require the same output within the decode tests' tolerance, on consecutive calls (the
array keeps the previous call's contents), and a clear error for sizes beyond the array.

This file is collected last so that a stop-at-first-failure run has already run every other test.
"""
from __future__ import annotations

import pytest
import torch

from tests.helpers import max_abs

pytestmark = pytest.mark.gpu

DECODE_TOL = 1e-2        # the max-abs tolerance of tests/test_gpu_decode.py


def _inputs(B, H, N, seed, dev):
    gen = torch.Generator().manual_seed(seed)
    cap = N + 40
    bf = torch.bfloat16
    k = torch.randn(B, H, cap, 64, generator=gen).to(bf)
    v = torch.randn(B, H, cap, 64, generator=gen).to(bf)
    b = torch.randn(B, H, cap, 32, generator=gen).to(bf)
    g = torch.cumsum(-torch.rand(B, H, cap, generator=gen) * 0.05, dim=2)
    f = torch.cumsum(-torch.rand(B, H, cap, generator=gen) * 0.02, dim=2)
    q = torch.randn(B, H, 1, 64, generator=gen).to(bf)
    c = torch.randn(B, H, 1, 32, generator=gen).to(bf)
    lam = torch.rand(H, generator=gen) + 0.2
    t = dict(k=k, v=v, b=b, g=g, f=f, q=q, c=c, lam=lam, gq=g[:, :, N - 1].contiguous(), fq=f[:, :, N - 1].contiguous())
    return {n: x.to(dev) for n, x in t.items()}


def _run(x, B, H, N, noalloc):
    from sisa_b200 import _lib, backends

    lib = _lib.load()
    dev = x["q"].device
    y = torch.empty(B, H, 1, 64, device=dev, dtype=torch.bfloat16)
    v = [_lib.view4(t) for t in (x["q"], x["c"], x["k"], x["v"], x["b"], y)]
    r = [_lib.vref(e) for e in v]
    st = backends.status_word(dev)
    stream = _lib.stream_ptr(dev)
    common = (r[0], r[1], x["gq"].data_ptr(), x["fq"].data_ptr(), r[2], r[3], r[4], x["g"].data_ptr(),
              x["f"].data_ptr(), x["g"].shape[2], x["lam"].data_ptr(), B, H, N, _lib.BF16, r[5])
    if noalloc:
        rc = lib.sisa_decode_attn_noalloc(*common, st.data_ptr(), stream)
    else:
        ws = torch.empty(lib.sisa_decode_workspace(B, H, N), dtype=torch.uint8, device=dev)
        rc = lib.sisa_decode_attn(*common, ws.data_ptr(), st.data_ptr(), stream)
    _lib.check(rc, "decode")
    torch.cuda.synchronize(dev)
    backends.check_status(dev)
    return y.cpu()


def test_noalloc_matches_workspace_entry_point(cuda_dev):
    # two calls in a row with different shapes: the second starts from the first call's leftover scratch
    for B, H, N, seed in ((2, 3, 1000, 1), (4, 2, 257, 2)):
        x = _inputs(B, H, N, seed, cuda_dev)
        ref = _run(x, B, H, N, noalloc=False)
        got = _run(x, B, H, N, noalloc=True)
        assert max_abs(got, ref) <= DECODE_TOL


def test_noalloc_repeated_calls_agree(cuda_dev):
    x = _inputs(3, 4, 3000, 3, cuda_dev)
    first = _run(x, 3, 4, 3000, noalloc=True)
    second = _run(x, 3, 4, 3000, noalloc=True)
    ref = _run(x, 3, 4, 3000, noalloc=False)
    assert torch.equal(first, second)
    assert max_abs(second, ref) <= DECODE_TOL


def test_noalloc_rejects_sizes_beyond_the_fixed_scratch(cuda_dev):
    from sisa_b200 import _lib

    x = _inputs(1, 1, 16, 4, cuda_dev)
    lib = _lib.load()
    y = torch.empty(1, 1, 1, 64, device=cuda_dev, dtype=torch.bfloat16)
    v = [_lib.vref(_lib.view4(t)) for t in (x["q"], x["c"], x["k"], x["v"], x["b"], y)]
    rc = lib.sisa_decode_attn_noalloc(v[0], v[1], x["gq"].data_ptr(), x["fq"].data_ptr(), v[2], v[3], v[4],
                                      x["g"].data_ptr(), x["f"].data_ptr(), x["g"].shape[2], x["lam"].data_ptr(),
                                      200, 100, 16, _lib.BF16, v[5], None, None)
    assert rc == _lib.ERR_VALUE
    assert "fixed scratch" in _lib.last_error()
