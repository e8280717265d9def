"""Run-time guards of the cuda path: the non-finite guard of the fused layer, the monotone check of
the unfused attention, and a bounded device wait that runs out.

The reference asserts on the device (``torch._assert_async``), which ends the CUDA context, so its
guard tests run every tripping case in a child process (tests/test_guards.py of tlstngud/sisa). Here
the kernels OR status bits into a device word that the host reads; the context survives, and every
case runs in this process:

* ``"async"`` (default): the call returns; ``backends.check_status()`` raises afterwards.
* ``"sync"``: the call itself raises.
* ``"off"``: nothing is read; the output must then be non-finite, never silently wrong.

The injection matrix follows the reference's (tests/test_guards.py:125-169): NaN at the first
element of head 0 in the alpha, theta, Q, K, B, C and V columns of ``proj``, in ``z`` and in lambda,
at rows 0.. (all), 100 and the last; +inf and -inf at row 100. Every case where a non-finite value
reaches a score must raise ``FloatingPointError``, except alpha = -inf (softplus = 0: no decay, finite),
z = +inf (log sigmoid = 0: no forgetting, finite) and V (not guarded: the output must be non-finite).
"""
from __future__ import annotations

import pytest
import torch

from oracle import sisa_oracle as O

pytestmark = pytest.mark.gpu

B_, H_, L_ = 2, 8, 512
VALUES = {"nan": float("nan"), "pinf": float("inf"), "ninf": float("-inf")}


def _cases():
    out = []
    for target in ("A", "TH", "Q", "K", "B", "C", "V", "z", "lam"):
        rows = ("all", "r100", "last") if target != "lam" else ("all",)
        for val in VALUES:
            for where in rows:
                if val != "nan" and where != "r100":
                    continue
                out.append(dict(target=target, val=val, where=where, forget=True, mode="async"))
    for target in ("A", "TH", "Q"):
        out.append(dict(target=target, val="nan", where="r100", forget=False, mode="async"))
    for mode in ("sync", "off"):
        out.append(dict(target="A", val="nan", where="all", forget=True, mode=mode))
    out.append(dict(target="none", val="nan", where="all", forget=True, mode="async"))
    return out


def _expect_raise(c):
    if c["mode"] == "off" or c["target"] in ("none", "V"):
        return False
    if (c["target"], c["val"]) in (("A", "ninf"), ("z", "pinf")):
        return False
    return True


def _case_id(c):
    return f"{c['target']}-{c['val']}-{c['where']}" + ("" if c["forget"] else "-noF") + \
        ("" if c["mode"] == "async" else f"-{c['mode']}")


def _layer(forget, dev):
    off = O.fused_layout(H_)
    gen = torch.Generator().manual_seed(11)
    proj = torch.randn(B_, L_, off["NPAD"], generator=gen) * 0.7
    proj[..., off["NTOT"]:] = 0
    z = torch.randn(B_, L_, H_, generator=gen) + 2 if forget else None
    lam = torch.rand(H_, generator=gen) + 0.2
    return proj.to(torch.bfloat16).to(dev), None if z is None else z.to(dev), lam.to(dev), off


@pytest.mark.parametrize("case", _cases(), ids=_case_id)
def test_nonfinite_guard(cuda_dev, case):
    from sisa_b200 import backends
    from sisa_b200.kernels.fused import sisa_fused

    backends.check_status(cuda_dev)          # start from a clear status word
    proj, z, lam, off = _layer(case["forget"], cuda_dev)
    val = VALUES[case["val"]]
    rows = {"all": slice(None), "r100": slice(100, 101), "last": slice(L_ - 1, L_)}[case["where"]]
    t = case["target"]
    if t in ("A", "TH", "Q", "K", "B", "C", "V"):
        proj[:, rows, off[t]] = val
    elif t == "z":
        z[:, rows, 0] = val
    elif t == "lam":
        lam[0] = val
    proj.requires_grad_(True)
    want = _expect_raise(case)
    old = backends.get_check_mode()
    backends.set_check_mode(case["mode"])
    try:
        if case["mode"] == "sync" and want:
            with pytest.raises(FloatingPointError):
                sisa_fused(proj, z, lam, H_)
            return
        y = sisa_fused(proj, z, lam, H_)
        torch.cuda.synchronize()
        finite = bool(torch.isfinite(y.float()).all())
        if case["mode"] == "off":
            backends.status_word(cuda_dev).zero_()      # bits set while nobody read them
            assert not finite, "check mode off: the output must be non-finite"
            return
        if want:
            with pytest.raises(FloatingPointError):
                backends.check_status(cuda_dev)
        else:
            backends.check_status(cuda_dev)          # must not raise
            assert finite == (t != "V"), f"output finite={finite}"
    finally:
        backends.set_check_mode(old)
        backends.status_word(cuda_dev).zero_()


def _rising_g(dev):
    gen = torch.Generator().manual_seed(3)
    Bm, Hm, Lm = 1, 2, 300
    q, k, v = (torch.randn(Bm, Hm, Lm, 64, generator=gen).to(torch.bfloat16).to(dev) for _ in range(3))
    c, b = (torch.randn(Bm, Hm, Lm, 32, generator=gen).to(torch.bfloat16).to(dev) for _ in range(2))
    g = torch.cumsum(-torch.rand(Bm, Hm, Lm, generator=gen) * 0.1, -1)
    g[:, :, 150:] += 0.5                      # one rise of +0.5 between positions 149 and 150
    lam = torch.full((Hm,), 0.3)
    return q, k, v, c, b, g.to(dev), lam.to(dev)


@pytest.mark.parametrize("mode", ["sync", "async"])
def test_monotone_check(cuda_dev, mode):
    from sisa_b200 import backends
    from sisa_b200.kernels.attention import sisa_attention_cuda

    backends.check_status(cuda_dev)
    args = _rising_g(cuda_dev)
    old = backends.get_check_mode()
    backends.set_check_mode(mode)
    try:
        if mode == "sync":
            with pytest.raises(ValueError, match="non-increasing"):
                sisa_attention_cuda(*args)
        else:
            sisa_attention_cuda(*args)
            with pytest.raises(ValueError, match="non-increasing"):
                backends.check_status(cuda_dev)
    finally:
        backends.set_check_mode(old)
        backends.status_word(cuda_dev).zero_()


def test_bounded_wait_times_out_and_context_survives(cuda_dev):
    """A producer that never arrives: the consumers' bounded waits run out after 20 ms, record
    SISA_ST_TIMEOUT, free the tensor memory and return; the context then runs real work."""
    from sisa_b200 import _lib, backends

    lib = _lib.load()
    backends.check_status(cuda_dev)
    st = backends.status_word(cuda_dev)
    res = torch.full((1,), -1, dtype=torch.int32, device=cuda_dev)
    _lib.check(lib.sisa_selftest_wait(0, 20_000_000, st.data_ptr(), res.data_ptr(), _lib.stream_ptr(cuda_dev)),
               "sisa_selftest_wait")
    torch.cuda.synchronize()
    assert int(res.item()) == 2
    assert int(st.item()) & _lib.ST_TIMEOUT
    with pytest.raises(RuntimeError, match="timed out"):
        backends.check_status(cuda_dev)
    # the same handshake with the producer arriving: no timeout
    _lib.check(lib.sisa_selftest_wait(1, 20_000_000, st.data_ptr(), res.data_ptr(), _lib.stream_ptr(cuda_dev)),
               "sisa_selftest_wait")
    torch.cuda.synchronize()
    assert int(res.item()) == 0 and int(st.item()) == 0
    # the context is intact: a real attention call still runs and passes its checks
    from tests.test_gpu_attention import check, make_inputs

    ins, dout = make_inputs(1, 2, 130, seed=21)
    check(ins, dout, cuda_dev)
    backends.check_status(cuda_dev)
