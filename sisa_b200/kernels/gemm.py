"""``C (+)= A B^T`` on the CTA-pair tcgen05 GEMM of libsisa_b200 (``sisa_gemm``).

The linear-CE gradient GEMMs (dX = G W and dW += G^T X, the ``torch.matmul`` calls of
src/sisa/kernels/linear_ce.py:170-178) run here: bf16/fp16 operands of either majorness, fp32
accumulation, an fp32 output that can be accumulated into, or a bf16/fp16 output rounded once.
"""
from __future__ import annotations

import torch
from torch import Tensor

from .. import _lib, backends

__all__ = ["matmul_t"]

_OUT_CODES = {torch.float32: 2, torch.bfloat16: 0, torch.float16: 1}
_WS_BYTES: dict[tuple, int] = {}


def _workspace(dev: torch.device, M: int, N: int, K: int, out_code: int) -> Tensor | None:
    """Split-K workspace for this problem on ``dev`` (None when the kernel would not split it), taken
    from the caching allocator on the current stream for the one launch."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    key = (idx, M, N, K, out_code)
    nbytes = _WS_BYTES.get(key)
    if nbytes is None:
        with torch.cuda.device(idx):
            nbytes = int(_lib.load().sisa_gemm_workspace(M, N, K, out_code))
        if len(_WS_BYTES) >= 4096:          # shapes of a long-running process with varying sizes
            _WS_BYTES.clear()
        _WS_BYTES[key] = nbytes
    return torch.empty(nbytes, dtype=torch.uint8, device=dev) if nbytes > 0 else None


def _operand(t: Tensor, name: str) -> tuple[int, int]:
    """(mn, ld) of a 2-D operand viewed as rows x K: K-major when the K stride is 1, MN-major when the
    row stride is 1."""
    if t.dim() != 2:
        raise ValueError(f"{name} must be 2-D, got shape {tuple(t.shape)}")
    rows, k = t.shape
    if t.stride(1) == 1 or k == 1:
        ld = t.stride(0) if rows > 1 else -(-k // 8) * 8          # one row: any whole-unit stride
        if ld % 8 == 0 and ld >= k:
            return 0, ld
    if t.stride(0) == 1 or rows == 1:
        ld = t.stride(1) if k > 1 else -(-rows // 8) * 8
        if ld % 8 == 0 and ld >= rows:
            return 1, ld
    raise ValueError(f"{name} {tuple(t.shape)} needs a unit stride along one dimension and a stride of whole "
                     f"16-byte units along the other, got strides {t.stride()}")


def matmul_t(a: Tensor, b: Tensor, out: Tensor | None = None, *, accumulate: bool = False,
             out_dtype: torch.dtype = torch.float32, bias: Tensor | None = None, bias_col0: int | None = None,
             bias_round: bool = False) -> Tensor:
    """``out (+)= a @ b.T (+ bias)`` for ``a`` (M, K) and ``b`` (N, K) CUDA tensors of one dtype (bf16 or
    fp16), each with a unit stride along K or along its rows (so ``x.t()`` of a row-major tensor is
    taken as it lies). ``out`` (M, N) with unit column stride; ``accumulate`` adds to it (fp32 only);
    ``bias`` (N,) contiguous bf16/fp16/fp32 is added in fp32 before the output's rounding. With
    ``bias_col0``, ``bias`` (n,) covers only columns [bias_col0, bias_col0 + n) and the others get no bias
    (``sisa_gemm_bias_cols``: tiles away from those columns skip the bias); ``bias_round`` then rounds
    each bias value to the output's 16-bit type first, as autocast casts a linear's bias. Row strides
    must be whole 16-byte units and pointers 16-byte aligned (errors come back from the C ABI)."""
    if a.dtype != b.dtype:
        raise TypeError(f"operands differ in dtype: {a.dtype} and {b.dtype}")
    M, K = a.shape
    N, Kb = b.shape
    if K != Kb:
        raise ValueError(f"inner dimensions differ: a is {tuple(a.shape)}, b is {tuple(b.shape)}")
    if out is None:
        if accumulate:
            raise ValueError("accumulate needs an output tensor")
        per16 = 16 // torch.empty((), dtype=out_dtype).element_size()
        out = torch.empty((M, N + (-N % per16)), dtype=out_dtype, device=a.device)[:, :N]   # rows in 16-byte units
    if out.shape != (M, N) or (out.stride(1) != 1 and N > 1):
        raise ValueError(f"out must be ({M}, {N}) with unit column stride, got {tuple(out.shape)} {out.stride()}")
    if out.dtype not in _OUT_CODES:
        raise TypeError(f"out dtype must be fp32, bf16 or fp16, got {out.dtype}")
    a_mn, lda = _operand(a, "a")
    b_mn, ldb = _operand(b, "b")
    ldc = out.stride(0) if M > 1 else -(-N // 8) * 8
    lib = _lib.load()
    dev = a.device
    ws = _workspace(dev, M, N, K, _OUT_CODES[out.dtype])
    ws_ptr, ws_n = (None, 0) if ws is None else (ws.data_ptr(), ws.numel())
    if bias_col0 is not None:
        if bias is None or bias.dim() != 1 or not bias.is_contiguous() or bias.dtype not in _OUT_CODES:
            raise ValueError("bias_col0 needs a contiguous 1-D bf16/fp16/fp32 bias")
        _lib.check(lib.sisa_gemm_bias_cols(a.data_ptr(), lda, a_mn, b.data_ptr(), ldb, b_mn, out.data_ptr(), ldc, M, N,
                                           K, _lib.dtype_code(a.dtype), _OUT_CODES[out.dtype], int(accumulate),
                                           bias.data_ptr(), _OUT_CODES[bias.dtype], bias_col0, bias.numel(),
                                           int(bias_round), ws_ptr, ws_n, backends.status_word(dev).data_ptr(),
                                           _lib.stream_ptr(dev)), "sisa_gemm_bias_cols")
        backends.after_call(dev)
        return out
    if bias is not None and (bias.shape != (N,) or not bias.is_contiguous() or bias.dtype not in _OUT_CODES):
        raise ValueError(f"bias must be a contiguous ({N},) bf16/fp16/fp32 tensor, got {tuple(bias.shape)} {bias.dtype}")
    _lib.check(lib.sisa_gemm(a.data_ptr(), lda, a_mn, b.data_ptr(), ldb, b_mn, out.data_ptr(), ldc, M, N, K,
                             _lib.dtype_code(a.dtype), _OUT_CODES[out.dtype], int(accumulate),
                             None if bias is None else bias.data_ptr(), 0 if bias is None else _OUT_CODES[bias.dtype],
                             ws_ptr, ws_n, backends.status_word(dev).data_ptr(), _lib.stream_ptr(dev)), "sisa_gemm")
    backends.after_call(dev)
    return out
