"""Functional SISA attention with a selectable implementation (mirrors src/sisa/functional.py).

For each head the score of query i and key j <= i is::

    s_ij = q_i.k_j / sqrt(d_head) + lam_h exp(g_i - g_j)(c_i.b_j) + (F_i - F_j)

``impl="torch"`` is exact blocked attention in plain PyTorch (any device, d_head, even d_state),
``impl="cuda"`` the sm_100a kernels (:func:`sisa_b200.kernels.attention.sisa_attention_cuda`),
``impl="auto"`` the kernels when they can take the inputs, else torch.
"""
from __future__ import annotations

import contextlib
import math
import warnings

import torch
from torch import Tensor
from torch.utils.checkpoint import checkpoint

__all__ = ["rotate_pairs", "sisa_attention_torch", "sisa_attention"]


def rotate_pairs(z: Tensor, phi: Tensor) -> Tensor:
    """Rotate interleaved channel pairs (0, 1), (2, 3), ... of ``z`` (..., d_state) by ``phi`` (..., d_state/2)."""
    ze, zo = z[..., 0::2], z[..., 1::2]
    c, s = torch.cos(phi), torch.sin(phi)
    return torch.stack([ze * c - zo * s, ze * s + zo * c], dim=-1).flatten(-2)


def _work_dtype(dtype: torch.dtype) -> torch.dtype:
    return torch.promote_types(dtype, torch.float32)


_AUTOCAST_DEVICE_TYPES = frozenset(d for d in ("cuda", "cpu", "xpu", "hpu", "mps") if torch.amp.is_autocast_available(d))


def _autocast_off(device_type: str):
    if device_type in _AUTOCAST_DEVICE_TYPES:
        return torch.autocast(device_type=device_type, enabled=False)
    return contextlib.nullcontext()


def attend_rows(q, k, v, c, b, g_q, g_k, lam, f_q, f_k, q_start: int) -> Tensor:
    """Exact attention of M query rows at positions q_start.. against N keys 0..N-1, in the inputs' dtype
    (autocast off). Shapes: q, c (B, H, M, .); k, v, b (B, H, N, .); g_q, f_q (B, H, M); g_k, f_k (B, H, N)."""
    with _autocast_off(q.device.type):
        m, n = q.shape[-2], k.shape[-2]
        scale = 1.0 / math.sqrt(q.shape[-1])
        causal = torch.arange(n, device=q.device).unsqueeze(0) <= torch.arange(q_start, q_start + m,
                                                                                device=q.device).unsqueeze(1)
        s = torch.matmul(q, k.transpose(-1, -2)) * scale
        delta = (g_q.unsqueeze(-1) - g_k.unsqueeze(-2)).masked_fill(~causal, 0.0)
        s = s + lam.view(1, -1, 1, 1) * torch.exp(delta) * torch.matmul(c, b.transpose(-1, -2))
        if f_q is not None:
            s = s + (f_q.unsqueeze(-1) - f_k.unsqueeze(-2))
        s = s.masked_fill(~causal, float("-inf"))
        return torch.matmul(torch.softmax(s, dim=-1), v)


def sisa_attention_torch(q: Tensor, k: Tensor, v: Tensor, c: Tensor, b: Tensor, g: Tensor, lam: Tensor,
                         fgate: Tensor | None = None, block_q: int = 256) -> Tensor:
    """Exact SISA attention in plain PyTorch, computed in fp32 (fp64 inputs stay fp64), query blocks of
    ``block_q`` rows, each checkpointed when gradients are needed. Returns (B, H, L, d_head) in q.dtype."""
    if q.dim() != 4:
        raise ValueError(f"q must be (B, H, L, d_head), got shape {tuple(q.shape)}")
    bsz, n_head, seq_len, _ = q.shape
    if k.shape != q.shape or v.shape[:3] != q.shape[:3]:
        raise ValueError(f"q, k, v shapes do not match: {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    if c.shape[:3] != q.shape[:3] or b.shape != c.shape or c.shape[-1] % 2 != 0:
        raise ValueError(f"c and b must be (B, H, L, d_state) with even d_state, got {tuple(c.shape)}, {tuple(b.shape)}")
    if g.shape != q.shape[:3] or (fgate is not None and fgate.shape != g.shape):
        raise ValueError("g and fgate must be (B, H, L)")
    if lam.shape != (n_head,):
        raise ValueError(f"lam must be ({n_head},), got {tuple(lam.shape)}")
    if block_q <= 0:
        raise ValueError("block_q must be positive")
    out_dtype = q.dtype
    wd = _work_dtype(q.dtype)
    q, k, v, c, b = (t.to(wd) for t in (q, k, v, c, b))
    g, lam = g.to(wd), lam.to(wd)
    fgate = None if fgate is None else fgate.to(wd)
    use_ckpt = torch.is_grad_enabled() and any(t is not None and t.requires_grad
                                               for t in (q, k, v, c, b, g, lam, fgate))
    outs = []
    for start in range(0, seq_len, block_q):
        end = min(start + block_q, seq_len)
        args = (q[:, :, start:end], k[:, :, :end], v[:, :, :end], c[:, :, start:end], b[:, :, :end],
                g[:, :, start:end], g[:, :, :end], lam, None if fgate is None else fgate[:, :, start:end],
                None if fgate is None else fgate[:, :, :end], start)
        if use_ckpt and seq_len > block_q:
            outs.append(checkpoint(attend_rows, *args, use_reentrant=False))
        else:
            outs.append(attend_rows(*args))
    out = outs[0] if len(outs) == 1 else torch.cat(outs, dim=2)
    return out.to(out_dtype)


def _cuda_problem(q, k, v, c, g, fgate) -> str | None:
    from . import backends
    from .config import CUDA_D_HEAD, CUDA_D_STATE

    if q.device.type != "cuda":
        return f"inputs are on {q.device.type}, the cuda kernels need CUDA"
    if q.shape[-1] != CUDA_D_HEAD or c.shape[-1] != CUDA_D_STATE:
        return f"the cuda kernels need d_head={CUDA_D_HEAD} and d_state={CUDA_D_STATE}"
    if q.dtype not in (torch.bfloat16, torch.float16):
        return f"unsupported dtype {q.dtype} (the cuda kernels take bf16 or fp16)"
    if k.dtype != q.dtype or v.dtype != q.dtype:
        return f"q, k and v must share one dtype, got {q.dtype}, {k.dtype}, {v.dtype}"
    if g.dtype != torch.float32 or (fgate is not None and fgate.dtype != torch.float32):
        return "g and fgate must be float32"
    ok, why = backends.cuda_status(q.device)
    return None if ok else why


def sisa_attention(q: Tensor, k: Tensor, v: Tensor, c: Tensor, b: Tensor, g: Tensor, lam: Tensor,
                   fgate: Tensor | None = None, impl: str = "auto", block_q: int = 256) -> Tensor:
    """SISA attention with a selectable backend (src/sisa/functional.py:181-220). ``impl`` is ``"torch"``,
    ``"cuda"`` (``"triton"`` is accepted as an alias) or ``"auto"``. Returns (B, H, L, d_head) in q.dtype."""
    if impl == "triton":
        impl = "cuda"
    if impl == "auto":
        why = _cuda_problem(q, k, v, c, g, fgate)
        impl = "cuda" if why is None else "torch"
        if why is not None and q.device.type == "cuda":
            from . import backends

            key = (q.device.index, why)
            if key not in backends._WARNED:
                backends._WARNED.add(key)
                warnings.warn(f"SISA: using the torch attention implementation on CUDA because {why}", stacklevel=2)
    if impl == "torch":
        return sisa_attention_torch(q, k, v, c, b, g, lam, fgate, block_q=block_q)
    if impl == "cuda":
        why = _cuda_problem(q, k, v, c, g, fgate)
        if why is not None:
            raise ValueError(f"impl='cuda' is not available: {why}")
        from .kernels.attention import sisa_attention_cuda

        return sisa_attention_cuda(q, k, v, c, b, g, lam, fgate)
    if impl == "triton_fused":
        raise ValueError("impl='triton_fused' fuses the input projections and is only available through "
                         "SISAAttention / SISAConfig.attn_impl")
    raise ValueError(f"unknown impl {impl!r}; expected 'auto', 'torch' or 'cuda'")
