"""The C ABI library loads and exports every entry point declared in include/*.h (no GPU calls)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from sisa_b200 import _lib

INCLUDE = Path(__file__).resolve().parents[1] / "include"


def declared_symbols() -> list[str]:
    names = []
    for h in sorted(INCLUDE.glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(sisa_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    declared = declared_symbols()
    assert len(declared) >= 12
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing
    # the binding knows every declared symbol (argument types attached)
    assert set(declared) <= set(_lib.SIGNATURES), sorted(set(declared) - set(_lib.SIGNATURES))


def test_version_and_layout():
    lib = _lib.load()
    assert b"sm_100a" in lib.sisa_version()
    out = (ctypes.c_int64 * 9)()
    for h, npad in ((8, 2192), (12, 3280), (16, 4368)):
        assert lib.sisa_fused_layout(h, out) == 0
        assert list(out) == [0, 64 * h, 128 * h, 192 * h, 224 * h, 256 * h, 272 * h, 273 * h, npad]
    assert lib.sisa_fused_layout(0, out) == _lib.ERR_VALUE
    assert "n_head" in _lib.last_error()


def test_layout_agrees_with_python_and_oracle(golden):
    from oracle import sisa_oracle as O
    from sisa_b200.kernels.fused import fused_layout

    for h, lay in golden("known")["layouts"].items():
        assert fused_layout(h) == lay == O.fused_layout(h)


def test_workspace_sizes():
    lib = _lib.load()
    assert lib.sisa_prep_fwd_workspace(2, 3, 130) == 2 * 3 * 3 * 18 * 4
    # fp64 block totals (B*H, nch, 18) + per-token d Phi (B*H, L, 16) fp32
    assert lib.sisa_prep_bwd_workspace(2, 3, 130) == 2 * 3 * (3 * 18 * 8 + 130 * 16 * 4)
    # row-statistic planes (4 x Lp fp32) + three (L,) fp32 row parts per (batch, head)
    assert lib.sisa_attn_bwd_workspace(2, 3, 130) == 2 * 3 * (132 * 16 + 130 * 12)


def test_position_plane_length():
    lib = _lib.load()
    assert [lib.sisa_pos_len(L) for L in (1, 4, 5, 130, 4096)] == [4, 4, 8, 132, 4096]


def test_host_side_argument_errors_need_no_gpu():
    """Validation happens before any CUDA call: bad shapes return SISA_ERR_VALUE with a message."""
    lib = _lib.load()
    rc = lib.sisa_prep_fwd(None, 0, 10, 2, 0, 0, 0, None, 0, 0, None, None, None, None, None, None)
    assert rc == _lib.ERR_VALUE and "B, H and L" in _lib.last_error()
    with pytest.raises(ValueError):
        _lib.check(rc, "sisa_prep_fwd")
    rc = lib.sisa_prep_fwd(None, 1, 10, 2, 0, 0, 7, None, 0, 0, None, None, None, None, None, None)
    assert rc == _lib.ERR_TYPE
    with pytest.raises(TypeError):
        _lib.check(rc, "sisa_prep_fwd")
    # (batch, head) rows are a launch-grid dimension: at most 65535 of them
    rc = lib.sisa_prep_fwd(None, 65536, 10, 1, 0, 0, 0, None, 0, 0, None, None, None, None, None, None)
    assert rc == _lib.ERR_VALUE and "too large" in _lib.last_error()


def test_norm_args_structs_match_the_c_header(tmp_path):
    """The ctypes mirrors of sisa_norm_fwd_args / sisa_norm_bwd_args have the C layout (gcc, no GPU)."""
    import ctypes
    import shutil
    import subprocess

    from sisa_b200 import _lib

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not found")
    root = Path(__file__).resolve().parents[1]
    src = tmp_path / "layout.c"
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "sisa_b200.h"', 'int main(void) {']
    for cname, cls in (("sisa_norm_fwd_args", _lib.NormFwdArgs), ("sisa_norm_bwd_args", _lib.NormBwdArgs)):
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in cls._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["return 0;", "}"]
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-I", str(root / "include"), str(src), "-o", str(exe)], check=True)
    got = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], check=True, capture_output=True,
                                                              text=True).stdout.splitlines())
    for cname, cls in (("sisa_norm_fwd_args", _lib.NormFwdArgs), ("sisa_norm_bwd_args", _lib.NormBwdArgs)):
        assert int(got[f"{cname} size"]) == ctypes.sizeof(cls)
        for fname, _ in cls._fields_:
            assert int(got[f"{cname} {fname}"]) == getattr(cls, fname).offset, (cname, fname)


def test_selftest_wait_rejects_bad_limits():
    """Host-side argument checks of the diagnostic wait entry point (no kernel is launched)."""
    lib = _lib.load()
    assert lib.sisa_selftest_wait(0, 10, None, None, None) == _lib.ERR_VALUE
    assert "limit_ns" in _lib.last_error()
    assert lib.sisa_selftest_wait(0, 2_000_000_000, None, None, None) == _lib.ERR_VALUE


def test_gemm_entry_points_reject_bad_arguments_before_any_cuda_call():
    """sisa_gemm, sisa_gemm_swiglu and sisa_lce_seed_scale check pointers, layouts and dtypes on the host
    (fake 16-byte-aligned addresses: no call here reaches the device)."""
    lib = _lib.load()
    A, B, C = 0x10000, 0x20000, 0x30000
    ok = dict(a=A, lda=64, a_mn=0, b=B, ldb=64, b_mn=0, c=C, ldc=64, M=64, N=64, K=64, dtype=_lib.BF16,
              out=_lib.F32, acc=0, bias=None, bias_dtype=0, ws=None, ws_bytes=0)

    def gemm(**kw):
        a = dict(ok, **kw)
        return lib.sisa_gemm(a["a"], a["lda"], a["a_mn"], a["b"], a["ldb"], a["b_mn"], a["c"], a["ldc"], a["M"],
                             a["N"], a["K"], a["dtype"], a["out"], a["acc"], a["bias"], a["bias_dtype"], a["ws"],
                             a["ws_bytes"], None, None)

    assert gemm(a=None) == _lib.ERR_VALUE and "null" in _lib.last_error()
    assert gemm(a_mn=2) == _lib.ERR_VALUE
    assert gemm(dtype=_lib.F32) == _lib.ERR_TYPE                  # operands are bf16 / fp16
    assert gemm(out=7) == _lib.ERR_TYPE
    assert gemm(out=_lib.BF16, acc=1) == _lib.ERR_VALUE and "accumulate" in _lib.last_error()
    assert gemm(M=0) == _lib.ERR_VALUE
    assert gemm(K=(1 << 30) + 1) == _lib.ERR_VALUE
    assert gemm(lda=60) == _lib.ERR_ALIGN                         # not whole 16-byte units
    assert gemm(lda=56) == _lib.ERR_ALIGN                         # K-major rows shorter than K
    assert gemm(a=A + 8) == _lib.ERR_ALIGN
    assert gemm(out=_lib.BF16, ldc=68) == _lib.ERR_ALIGN          # 136-byte rows
    assert gemm(bias=A + 4, bias_dtype=_lib.F32) == _lib.ERR_VALUE
    assert gemm(bias=A, bias_dtype=9) == _lib.ERR_VALUE
    assert gemm(ws=A + 8, ws_bytes=4096) == _lib.ERR_VALUE

    def swiglu(**kw):
        a = dict(dict(x=A, xld=64, w=B, wld=64, gu=C, guld=80, a=C + 0x8000, ald=40, rows=64, dff=40, K=64,
                      dtype=_lib.BF16), **kw)
        return lib.sisa_gemm_swiglu(a["x"], a["xld"], a["w"], a["wld"], a["gu"], a["guld"], a["a"], a["ald"],
                                    a["rows"], a["dff"], a["K"], a["dtype"], None, None)

    def gemm_cols(bias=A, bias_dtype=_lib.F32, col0=0, n=8, rnd=0, **kw):
        a = dict(ok, **kw)
        return lib.sisa_gemm_bias_cols(a["a"], a["lda"], a["a_mn"], a["b"], a["ldb"], a["b_mn"], a["c"], a["ldc"],
                                       a["M"], a["N"], a["K"], a["dtype"], a["out"], a["acc"], bias, bias_dtype,
                                       col0, n, rnd, a["ws"], a["ws_bytes"], None, None)

    # each call below fails a host check before anything could reach the device
    assert gemm_cols(bias=None) == _lib.ERR_VALUE and "null bias" in _lib.last_error()
    assert gemm_cols(bias_dtype=7) == _lib.ERR_TYPE
    assert gemm_cols(bias=A + 2) == _lib.ERR_ALIGN                   # fp32 bias off a 4-byte boundary
    assert gemm_cols(col0=60, n=8) == _lib.ERR_VALUE and "outside" in _lib.last_error()   # past N = 64
    assert gemm_cols(col0=-1) == _lib.ERR_VALUE
    assert gemm_cols(rnd=2) == _lib.ERR_VALUE
    assert gemm_cols(rnd=1) == _lib.ERR_VALUE and "bias_round" in _lib.last_error()       # fp32 output
    assert gemm_cols(a=None) == _lib.ERR_VALUE and "sisa_gemm_bias_cols" in _lib.last_error()

    assert swiglu(dff=36) == _lib.ERR_VALUE and "multiple of 8" in _lib.last_error()
    assert swiglu(a=None) == _lib.ERR_VALUE                      # gu may be NULL (inference), a may not
    assert swiglu(guld=72) == _lib.ERR_ALIGN                      # gu rows must hold 2 d_ff
    assert swiglu(gu=None, ald=36) == _lib.ERR_ALIGN              # without gu, a is still checked
    assert swiglu(dtype=_lib.F32) == _lib.ERR_TYPE

    assert lib.sisa_lce_seed_scale(None, 16, A, None, _lib.F32, None, None) == _lib.ERR_VALUE
    assert lib.sisa_lce_seed_scale(A, 16, A, None, _lib.BF16, None, None) == _lib.ERR_VALUE   # in place is fp32
    assert lib.sisa_lce_seed_scale(A, 16, A, B, 5, None, None) == _lib.ERR_TYPE
    assert lib.sisa_lce_seed_scale(A + 4, 16, A, None, _lib.F32, None, None) == _lib.ERR_ALIGN


def test_split_rows_is_checked_on_the_host():
    """sisa_split_rows rejects bad shapes and alignment before any CUDA call (fake addresses)."""
    lib = _lib.load()
    A, B, C = 0x10000, 0x20000, 0x30000

    def split(src=A, sld=8, d0=B, d1=C, dld=8, rows=16, cols=8, block=8):
        return lib.sisa_split_rows(src, sld, d0, d1, dld, rows, cols, block, None)

    assert split(src=None) == _lib.ERR_VALUE and "null" in _lib.last_error()
    assert split(rows=12) == _lib.ERR_VALUE                       # not a multiple of the block
    assert split(cols=6) == _lib.ERR_VALUE
    assert split(block=0) == _lib.ERR_VALUE
    assert split(sld=6, cols=4) == _lib.ERR_ALIGN                  # row stride not a multiple of 4
    assert split(d1=C + 4) == _lib.ERR_ALIGN
    assert split(rows=0) == _lib.OK                                # nothing to do, no launch


def test_embedding_grad_is_checked_on_the_host():
    """sisa_embedding_bwd rejects bad sizes and alignment before any CUDA call (fake addresses)."""
    lib = _lib.load()
    A, B, C = 0x10000, 0x20000, 0x30000

    def bwd(ids=A, n=16, grad=B, ld=8, dw=C, V=10, D=8):
        return lib.sisa_embedding_bwd(ids, n, grad, ld, dw, V, D, None)

    assert bwd(dw=None) == _lib.ERR_VALUE and "null" in _lib.last_error()
    assert bwd(ids=None) == _lib.ERR_VALUE
    assert bwd(n=262145) == _lib.ERR_VALUE                         # past SISA_EMBED_MAX_IDS
    assert bwd(D=6, ld=8) == _lib.ERR_VALUE                        # D a multiple of 4
    assert bwd(ld=4) == _lib.ERR_VALUE                             # row stride below D
    assert bwd(V=0) == _lib.ERR_VALUE
    assert bwd(ld=10, D=8) == _lib.ERR_ALIGN
    assert bwd(grad=B + 8) == _lib.ERR_ALIGN
    assert bwd(ids=A + 4) == _lib.ERR_ALIGN


def test_row_copy_jobs_are_checked_on_the_host():
    """sisa_row_copy_check accepts well-formed jobs and names what is wrong with the others;
    sisa_copy_rows rejects a bad table pointer or dtype before any CUDA call (fake addresses)."""
    import ctypes

    lib = _lib.load()
    ok = dict(src=0x10000, dst=0x20000, rows=64, cols=256, src_ld=256, dst_ld=256, block_rows=64,
              dst_block_stride=0)

    def check(**kw):
        job = _lib.RowCopy(**dict(ok, **kw))
        return lib.sisa_row_copy_check(ctypes.byref(job))

    assert check() == _lib.OK
    assert check(src=None) == _lib.OK                           # zero fill
    assert check(block_rows=8, dst_block_stride=16) == _lib.OK  # interleave
    assert check(dst=None) == _lib.ERR_VALUE
    assert check(cols=252) == _lib.ERR_VALUE and "multiple of 8" in _lib.last_error()
    assert check(rows=-1) == _lib.ERR_VALUE
    assert check(block_rows=0) == _lib.ERR_VALUE
    assert check(dst=0x20008) == _lib.ERR_ALIGN
    assert check(src=0x10004) == _lib.ERR_ALIGN
    assert check(dst_ld=260) == _lib.ERR_ALIGN
    assert check(src_ld=130) == _lib.ERR_ALIGN                  # shorter than a row
    assert lib.sisa_copy_rows(0x30008, 4, 100, _lib.BF16, None, None) == _lib.ERR_ALIGN
    assert lib.sisa_copy_rows(0x30000, 4, 100, 7, None, None) == _lib.ERR_TYPE
    assert lib.sisa_copy_rows(0x30000, -1, 100, _lib.BF16, None, None) == _lib.ERR_VALUE
    assert lib.sisa_copy_rows(None, 0, 0, _lib.BF16, None, None) == _lib.OK


def test_adamw_tensor_list_is_checked_on_the_host():
    """sisa_adamw_tensors checks its host table before any CUDA call (fake 16-byte-aligned addresses;
    every call here is invalid, so none reaches the device)."""
    lib = _lib.load()
    A = 0x10000

    def call(entries, n_state=4096, **kw):
        tab = (_lib.AdamTensor * max(1, len(entries)))()
        for e, (param, grad, off, n) in zip(tab, entries):
            e.param, e.grad, e.offset, e.n, e.lr, e.weight_decay = param, grad, off, n, 1e-3, 0.1
        a = dict(m=A, v=A + 0x4000, npart=296, b1=0.9, b2=0.95, eps=1e-8)
        a.update(kw)
        return lib.sisa_adamw_tensors(tab, len(entries), a["m"], a["v"], n_state, A, A, a["npart"], a["b1"], a["b2"],
                                      a["eps"], 1.0, None, None)

    assert call([(A, A, 2, 5)]) == _lib.ERR_VALUE                                # offset not a multiple of 4
    assert call([(A, A, 0, 5), (A, A, 4, 3)]) == _lib.ERR_VALUE                  # overlaps the previous tensor
    assert call([(A, A, 4092, 8)]) == _lib.ERR_VALUE                             # past n_state
    assert call([(A + 2, A, 0, 5)]) == _lib.ERR_ALIGN                            # not even 4-byte aligned
    assert call([(A, None, 0, 5)]) == _lib.ERR_VALUE
    assert call([(A, A, 0, 5)], n_state=4094) == _lib.ERR_VALUE
    assert call([(A, A, 0, 5)], eps=0.0) == _lib.ERR_VALUE
    assert call([(A, A, 0, 5)], m=A + 8) == _lib.ERR_ALIGN
    assert call([(A, A, 4 * k, 1) for k in range(385)], n_state=4 * 385) == _lib.ERR_VALUE
