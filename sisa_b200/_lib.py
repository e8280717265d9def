"""ctypes binding of ``libsisa_b200.so`` (declared in ``include/sisa_b200.h``).

The library is loaded on first use. If it has not been built, every CUDA entry point raises
``RuntimeError``: there is no fallback implementation behind this module.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libsisa_b200.so"
_LOCK = threading.Lock()
_LIB = None

# return codes / status bits (sisa_b200.h)
OK, ERR_VALUE, ERR_TYPE, ERR_ALIGN, ERR_CUDA, ERR_UNSUPPORTED = 0, 1, 2, 3, 4, 5
ST_NONFINITE, ST_NONMONOTONE, ST_TIMEOUT, ST_BAD_SEED, ST_BAD_POS = 1, 2, 4, 8, 16
BF16, F16, F32 = 0, 1, 2


class View4(ctypes.Structure):
    """``sisa_view4``: a (B, H, L, X) view with element strides of the first three axes."""

    _fields_ = [("data", ctypes.c_void_p), ("stride_b", ctypes.c_int64), ("stride_h", ctypes.c_int64),
                ("stride_l", ctypes.c_int64)]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int
_VP = ctypes.POINTER(View4)


class AdamTensor(ctypes.Structure):
    """``sisa_adam_tensor``: one parameter tensor of the tensor-list AdamW."""

    _fields_ = [("param", _P), ("grad", _P), ("offset", _I64), ("n", _I64), ("lr", ctypes.c_float),
                ("weight_decay", ctypes.c_float)]


class RowCopy(ctypes.Structure):
    """``sisa_row_copy``: one row-block copy of fp32 rows into compute-dtype rows (or a zero fill)."""

    _fields_ = [("src", _P), ("dst", _P), ("rows", _I64), ("cols", _I64), ("src_ld", _I64), ("dst_ld", _I64),
                ("block_rows", _I64), ("dst_block_stride", _I64)]


class NormFwdArgs(ctypes.Structure):
    """``sisa_norm_fwd_args``: one RMSNorm at a block boundary (residual add, up to two output copies, an
    optional fp32 projection of the output)."""

    _fields_ = [("x", _P), ("x_ld", _I64), ("x_dtype", _I),
                ("res", _P), ("res_ld", _I64), ("res_dtype", _I),
                ("xsum", _P), ("xsum_ld", _I64),
                ("weight", _P),
                ("rows", _I64), ("d", _I64),
                ("eps", ctypes.c_float),
                ("n_out", _I),
                ("y", _P * 2), ("y_ld", _I64 * 2), ("y_dtype", _I * 2),
                ("rstd", _P),
                ("proj_w", _P), ("proj_b", _P), ("n_proj", _I64), ("proj_out", _P)]


class NormBwdArgs(ctypes.Structure):
    """``sisa_norm_bwd_args``: the backward of :class:`NormFwdArgs`."""

    _fields_ = [("v", _P), ("v_ld", _I64), ("v_dtype", _I),
                ("weight", _P), ("rstd", _P),
                ("rows", _I64), ("d", _I64),
                ("dy", _P * 2), ("dy_ld", _I64 * 2), ("dy_dtype", _I * 2),
                ("dv_in", _P), ("dv_in_ld", _I64), ("dv_in_dtype", _I),
                ("proj_w", _P), ("n_proj", _I64), ("dproj_out", _P),
                ("dx", _P), ("dx_ld", _I64), ("dx_dtype", _I),
                ("dres", _P), ("dres_ld", _I64), ("dres_dtype", _I),
                ("dweight", _P), ("dproj_w", _P), ("dproj_b", _P),
                ("workspace", _P)]

# name -> (restype, argtypes); every symbol declared in include/sisa_b200.h
SIGNATURES = {
    "sisa_version": (ctypes.c_char_p, []),
    "sisa_last_error": (ctypes.c_char_p, []),
    "sisa_device_check": (_I, [_I]),
    "sisa_fused_layout": (_I, [_I64, ctypes.POINTER(_I64)]),
    "sisa_prep_fwd_workspace": (_I64, [_I64, _I64, _I64]),
    "sisa_prep_bwd_workspace": (_I64, [_I64, _I64, _I64]),
    "sisa_attn_bwd_workspace": (_I64, [_I64, _I64, _I64]),
    "sisa_pos_len": (_I64, [_I64]),
    "sisa_prep_fwd": (_I, [_P, _I64, _I64, _I64, _I64, _I64, _I, _P, _I64, _I64, _P, _P, _P, _P, _P, _P]),
    "sisa_pack_positions": (_I, [_P, _I64, _I64, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _P]),
    "sisa_attn_fwd": (_I, [_VP, _VP, _VP, _VP, _VP, _P, _P, _I64, _I64, _I64, _I, _VP, _P, _P, _P, _P]),
    "sisa_attn_bwd": (_I, [_VP, _VP, _VP, _VP, _VP, _P, _P, _VP, _VP, _P, _P, _I64, _I64, _I64, _I,
                           _VP, _VP, _VP, _VP, _VP, _P, _P, _P, _P, _P, _P]),
    "sisa_prep_bwd": (_I, [_P, _I64, _I64, _I64, _I64, _I64, _I, _P, _I64, _I64, _P, _P, _P, _P, _P,
                           _P, _I64, _I64, _P, _P, _P, _P]),
    "sisa_lce_workspace": (_I64, [_I64, _I64]),
    "sisa_lce_logits": (_I, [_P, _I64, _I64, _I64, _P, _I64, _I64, _I64, _I, _P, _P, _I64, _P, _P, _P]),
    "sisa_lce_grad": (_I, [_P, _I64, _I64, _I64, _I64, _I, _P, _I64, _P, ctypes.c_float, _I, _P, _P, _P, _P]),
    "sisa_lce_seed_scale": (_I, [_P, _I64, _P, _P, _I, _P, _P]),
    "sisa_adamw_flat": (_I, [_P, _P, _P, _P, _I64, _P, _I, _P, _P, _I, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                             ctypes.c_float, _P, _P]),
    "sisa_adamw_tensors": (_I, [ctypes.POINTER(AdamTensor), _I, _P, _P, _I64, _P, _P, _I, ctypes.c_float,
                                ctypes.c_float, ctypes.c_float, ctypes.c_float, _P, _P]),
    "sisa_row_copy_check": (_I, [ctypes.POINTER(RowCopy)]),
    "sisa_copy_heads": (_I, [_P, _I64, _I64, _I64, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _P]),
    "sisa_copy_rows": (_I, [_P, _I, _I64, _I, _P, _P]),
    "sisa_gemm_swiglu": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I64, _I, _P, _P]),
    "sisa_gemm_workspace": (_I64, [_I64, _I64, _I64, _I]),
    "sisa_split_rows": (_I, [_P, _I64, _P, _P, _I64, _I64, _I64, _I64, _P]),
    "sisa_embedding_bwd": (_I, [_P, _I64, _P, _I64, _P, _I64, _I64, _P]),
    "sisa_gemm": (_I, [_P, _I64, _I, _P, _I64, _I, _P, _I64, _I64, _I64, _I64, _I, _I, _I, _P, _I, _P, _I64, _P, _P]),
    "sisa_gemm_bias_cols": (_I, [_P, _I64, _I, _P, _I64, _I, _P, _I64, _I64, _I64, _I64, _I, _I, _I, _P, _I, _I64, _I64,
                                 _I, _P, _I64, _P, _P]),
    "sisa_decode_attn": (_I, [_VP, _VP, _P, _P, _VP, _VP, _VP, _P, _P, _I64, _P, _I64, _I64, _I64, _I, _VP, _P,
                              _P, _P]),
    "sisa_decode_workspace": (_I64, [_I64, _I64, _I64]),
    "sisa_decode_attn_noalloc": (_I, [_VP, _VP, _P, _P, _VP, _VP, _VP, _P, _P, _I64, _P, _I64, _I64, _I64, _I, _VP,
                                      _P, _P]),
    "sisa_decode_prep": (_I, [_P, _I64, _P, _I64, _I64, _I64, _I, _VP, _VP, _VP, _P, _P, _I64, _I64, _P, _P, _P, _P,
                              _P, _P]),
    "sisa_decode_prep_dpos": (_I, [_P, _I64, _P, _I64, _I64, _I64, _I, _VP, _VP, _VP, _P, _P, _I64, _P, _I64, _P, _P,
                                   _P, _P, _P, _P]),
    "sisa_decode_attn_dpos": (_I, [_VP, _VP, _P, _P, _VP, _VP, _VP, _P, _P, _I64, _P, _I64, _I64, _P, _I64, _I, _VP,
                                   _P, _P, _P]),
    "sisa_rmsnorm_bwd_workspace": (_I64, [_I64, _I64]),
    "sisa_rmsnorm_fwd": (_I, [_P, _I64, _I, _P, _I64, _I64, ctypes.c_float, _P, _I64, _I, _P, _P, _P]),
    "sisa_rmsnorm_bwd": (_I, [_P, _I64, _I, _P, _I64, _I, _P, _P, _I64, _I64, _P, _I64, _I, _P, _P, _P, _P]),
    "sisa_norm_bwd_workspace": (_I64, [_I64, _I64, _I64]),
    "sisa_norm_fwd": (_I, [ctypes.POINTER(NormFwdArgs), _P, _P]),
    "sisa_norm_bwd": (_I, [ctypes.POINTER(NormBwdArgs), _P, _P]),
    "sisa_swiglu_fwd": (_I, [_P, _I64, _P, _I64, _I64, _I64, _I, _P, _I64, _P, _P]),
    "sisa_swiglu_bwd": (_I, [_P, _I64, _P, _I64, _P, _I64, _I64, _I64, _I, _P, _I64, _P, _I64, _P, _P]),
    "sisa_selftest_wait": (_I, [_I, _I64, _P, _P, _P]),
}


def lib_path() -> Path:
    return _LIB_PATH


def load():
    """Load the shared library (once) and attach the prototypes. Raises RuntimeError if it is missing."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        if not _LIB_PATH.exists():
            raise RuntimeError(f"{_LIB_PATH} is not built; run `python -m sisa_b200.build` (nvcc, sm_100a)")
        lib = ctypes.CDLL(str(_LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
        return lib


def exported_symbols() -> list[str]:
    lib = load()
    return [n for n in SIGNATURES if hasattr(lib, n)]


def pos_planes(B: int, H: int, L: int, device) -> "torch.Tensor":
    """Allocate the planar position records (B, H, 4, Lp) fp32 that sisa_prep_fwd / sisa_pack_positions
    fill (planes g, F, rowf, colf; Lp = sisa_pos_len(L))."""
    import torch

    return torch.empty((B, H, 4, load().sisa_pos_len(L)), device=device, dtype=torch.float32)


def pos_records(pos, L: int):
    """(B, H, L, 4) view {g, F, rowf, colf} of planar position records."""
    return pos[..., :L].transpose(-1, -2)


def last_error() -> str:
    return load().sisa_last_error().decode()


def check(rc: int, what: str) -> None:
    """Map a C return code to the reference's exception types."""
    if rc == OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == ERR_TYPE:
        raise TypeError(msg)
    if rc in (ERR_VALUE, ERR_ALIGN):
        raise ValueError(msg)
    raise RuntimeError(msg)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def view4(t: torch.Tensor) -> View4:
    """View4 of a (B, H, L, X) tensor whose last axis is contiguous."""
    if t.dim() != 4 or t.stride(-1) != 1:
        raise ValueError(f"expected a 4-D tensor with a contiguous last axis, got {tuple(t.shape)} {t.stride()}")
    return View4(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def vref(v: View4):
    return ctypes.byref(v)


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return BF16
    if dt == torch.float16:
        return F16
    raise TypeError(f"the CUDA kernels take bf16 or fp16 operands, got {dt}")
