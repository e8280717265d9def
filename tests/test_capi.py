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
