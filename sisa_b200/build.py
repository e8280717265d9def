"""Build ``libsisa_b200.so`` (the sm_100a kernels and their C ABI) in-tree with nvcc.

Usage: ``python -m sisa_b200.build [--verbose]``. The library lands in ``sisa_b200/_lib/`` so that it
travels with the source tree; nothing is installed elsewhere.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "libsisa_b200.so"
SOURCES = ["prep.cu", "attn_fwd.cu", "attn_bwd.cu", "lce.cu", "gemm.cu", "decode.cu", "norm.cu", "optim.cu", "copy.cu", "embed.cu", "selftest.cu", "capi.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include"), "-I", str(CSRC)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put CUDA's bin directory on PATH)")


def _compile(src: Path, obj: Path, verbose: bool) -> str:
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}")
    return res.stderr


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile every CUDA source for sm_100a and link the shared library. Returns its path."""
    srcs = [CSRC / s for s in SOURCES if (CSRC / s).exists()]
    deps = srcs + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [ROOT / "include" / "sisa_b200.h"]
    if not force and LIB.exists() and all(LIB.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return LIB
    obj_dir = OUT_DIR / "obj"
    obj_dir.mkdir(parents=True, exist_ok=True)
    objs = [obj_dir / (s.stem + ".o") for s in srcs]
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        logs = list(ex.map(lambda a: _compile(a[0], a[1], verbose), zip(srcs, objs)))
    if verbose:
        for s, log in zip(srcs, logs):
            print(f"== {s.name}\n{log}")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args(argv)
    path = build(verbose=args.verbose, force=args.force)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
