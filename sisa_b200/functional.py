"""Functional SISA attention with a selectable implementation (the interface of src/sisa/functional.py).

For each head the score of query i and key j <= i is::

    s_ij = q_i.k_j / sqrt(d_head) + lam_h exp(g_i - g_j)(c_i.b_j) + (F_i - F_j)

and o_i = sum_j softmax_j(s_ij) v_j.

``impl="torch"`` runs :func:`sisa_attention_torch`, an exact plain-PyTorch implementation for any
device, d_head and even d_state; ``impl="cuda"`` runs the sm_100a kernels
(:func:`sisa_b200.kernels.attention.sisa_attention_cuda`); ``impl="auto"`` takes the kernels when they
can take the inputs, else torch.

The torch implementation streams over (query block, key block) tiles with an online softmax, so no
score matrix larger than one tile exists, and its backward is written out by hand from the score
formula rather than recorded by autograd: it recomputes each tile's probabilities from the saved
log-sum-exp and accumulates every input gradient tile by tile. Work happens in fp32 (fp64 inputs stay
fp64) with autocast off; the output comes back in q.dtype.
"""
from __future__ import annotations

import contextlib
import math
import warnings

import torch
from torch import Tensor
from torch.autograd.function import once_differentiable

__all__ = ["rotate_pairs", "sisa_attention_torch", "sisa_attention", "attention_rows"]


def rotate_pairs(z: Tensor, phi: Tensor) -> Tensor:
    """Rotate the channel pairs (0, 1), (2, 3), ... of ``z`` (..., d_state) by the angles ``phi``
    (..., d_state / 2): each pair (x, y) becomes (x cos - y sin, x sin + y cos)."""
    x, y = z.unflatten(-1, (-1, 2)).unbind(-1)
    cos, sin = torch.cos(phi), torch.sin(phi)
    return torch.stack((x * cos - y * sin, x * sin + y * cos), dim=-1).flatten(-2)


def compute_dtype(dtype: torch.dtype) -> torch.dtype:
    """The dtype the torch implementation works in: fp64 for fp64 inputs, fp32 otherwise."""
    return torch.float64 if dtype == torch.float64 else torch.float32


def no_autocast(device_type: str):
    """A context with autocast disabled on ``device_type`` (nothing to disable where it does not exist)."""
    try:
        return torch.autocast(device_type=device_type, enabled=False)
    except RuntimeError:
        return contextlib.nullcontext()


class _Tile:
    """Scores of one (query block, key block) tile.

    ``keep`` masks keys after the query; ``e`` = exp(g_i - g_j) on kept entries and 0 elsewhere (the
    exponent is zeroed before exp, since for j > i it only grows and would overflow); ``u`` = c_i.b_j;
    ``s`` the score with -inf on masked entries."""

    __slots__ = ("keep", "e", "u", "s")

    def __init__(self, q, k, c, b, g_q, g_k, f_q, f_k, lam4, scale, rows, cols):
        self.keep = cols.unsqueeze(0) <= rows.unsqueeze(1)
        diff = g_q.unsqueeze(-1) - g_k.unsqueeze(-2)
        self.e = torch.exp(torch.where(self.keep, diff, diff.new_zeros(()))) * self.keep
        self.u = torch.matmul(c, b.transpose(-1, -2))
        s = torch.matmul(q, k.transpose(-1, -2)) * scale + lam4 * self.e * self.u
        if f_q is not None:
            s = s + (f_q.unsqueeze(-1) - f_k.unsqueeze(-2))
        self.s = s.masked_fill(~self.keep, float("-inf"))


def attention_rows(q, k, v, c, b, g_q, g_k, lam, f_q, f_k, q_start: int, block: int = 256):
    """Exact attention of M query rows at absolute positions q_start.. against keys 0..N-1, in the
    inputs' dtype with autocast off, streamed over key blocks with an online softmax.

    Shapes: q, c (B, H, M, .); k, v, b (B, H, N, .); g_q, f_q (B, H, M); g_k, f_k (B, H, N); lam (H,).
    Returns (o, lse) with lse the natural-log log-sum-exp of each row."""
    with no_autocast(q.device.type):
        M, N = q.shape[-2], k.shape[-2]
        scale = 1.0 / math.sqrt(q.shape[-1])
        lam4 = lam.view(1, -1, 1, 1)
        rows = torch.arange(q_start, q_start + M, device=q.device)
        shape = q.shape[:-1]
        m = torch.full(shape, float("-inf"), dtype=q.dtype, device=q.device)
        l = torch.zeros(shape, dtype=q.dtype, device=q.device)
        acc = torch.zeros(shape + (v.shape[-1],), dtype=q.dtype, device=q.device)
        last = min(N, q_start + M)                    # keys after the last query are never attended
        for j0 in range(0, last, block):
            j1 = min(j0 + block, last)
            t = _Tile(q, k[:, :, j0:j1], c, b[:, :, j0:j1], g_q, g_k[:, :, j0:j1], f_q,
                      None if f_k is None else f_k[:, :, j0:j1], lam4, scale, rows,
                      torch.arange(j0, j1, device=q.device))
            m_new = torch.maximum(m, t.s.amax(-1))
            # rows with no kept key in this block yet keep m = -inf; their rescale factor is then 1
            m_safe = torch.where(torch.isinf(m_new) & (m_new < 0), torch.zeros_like(m_new), m_new)
            alpha = torch.exp(m - m_safe)
            p = torch.exp(t.s - m_safe.unsqueeze(-1))
            l = l * alpha + p.sum(-1)
            acc = acc * alpha.unsqueeze(-1) + torch.matmul(p, v[:, :, j0:j1])
            m = m_new
        return acc / l.unsqueeze(-1), m + torch.log(l)


class _TorchAttention(torch.autograd.Function):
    """Exact SISA attention over (query block, key block) tiles; the backward is derived by hand.

    With P = softmax(S), dP = dO V^T, D_i = sum_d dO_id O_id and dS = P (dP - D):
    dq = dS k / sqrt(d), dk = dS^T q / sqrt(d), dv = P^T dO; with W = dS * exp(g_i - g_j) (masked):
    dc = lam W b, db = lam W^T c, dlam_h = sum W * (c.b), and g and F enter the score as
    (lam W (c.b)) and dS through differences, so each takes its row sums minus its column sums."""

    @staticmethod
    def forward(ctx, q, k, v, c, b, g, lam, fgate, block):
        L = q.shape[2]
        outs, lses = [], []
        for i0 in range(0, L, block):
            i1 = min(i0 + block, L)
            o, lse = attention_rows(q[:, :, i0:i1], k[:, :, :i1], v[:, :, :i1], c[:, :, i0:i1], b[:, :, :i1],
                                    g[:, :, i0:i1], g[:, :, :i1], lam,
                                    None if fgate is None else fgate[:, :, i0:i1],
                                    None if fgate is None else fgate[:, :, :i1], i0, block)
            outs.append(o)
            lses.append(lse)
        o = torch.cat(outs, dim=2)
        ctx.save_for_backward(q, k, v, c, b, g, lam, fgate, o, torch.cat(lses, dim=2))
        ctx.block = block
        return o

    @staticmethod
    @once_differentiable
    def backward(ctx, do):
        q, k, v, c, b, g, lam, fgate, o, lse = ctx.saved_tensors
        block = ctx.block
        with no_autocast(q.device.type):
            do = do.to(q.dtype)
            L = q.shape[2]
            scale = 1.0 / math.sqrt(q.shape[-1])
            lam4 = lam.view(1, -1, 1, 1)
            D = (do * o).sum(-1)
            dq, dk, dv, dc, db = (torch.zeros_like(t) for t in (q, k, v, c, b))
            dg = torch.zeros_like(g)
            dF = None if fgate is None else torch.zeros_like(fgate)
            dlam = torch.zeros_like(lam)
            dev = q.device
            for i0 in range(0, L, block):
                i1 = min(i0 + block, L)
                rows = torch.arange(i0, i1, device=dev)
                qi, ci, doi = q[:, :, i0:i1], c[:, :, i0:i1], do[:, :, i0:i1]
                for j0 in range(0, i1, block):
                    j1 = min(j0 + block, i1)
                    t = _Tile(qi, k[:, :, j0:j1], ci, b[:, :, j0:j1], g[:, :, i0:i1], g[:, :, j0:j1],
                              None if fgate is None else fgate[:, :, i0:i1],
                              None if fgate is None else fgate[:, :, j0:j1], lam4, scale, rows,
                              torch.arange(j0, j1, device=dev))
                    p = torch.exp(t.s - lse[:, :, i0:i1].unsqueeze(-1))
                    dp = torch.matmul(doi, v[:, :, j0:j1].transpose(-1, -2))
                    ds = p * (dp - D[:, :, i0:i1].unsqueeze(-1))
                    dq[:, :, i0:i1] += torch.matmul(ds, k[:, :, j0:j1]) * scale
                    dk[:, :, j0:j1] += torch.matmul(ds.transpose(-1, -2), qi) * scale
                    dv[:, :, j0:j1] += torch.matmul(p.transpose(-1, -2), doi)
                    w = ds * t.e
                    dc[:, :, i0:i1] += torch.matmul(w, b[:, :, j0:j1]) * lam4
                    db[:, :, j0:j1] += torch.matmul(w.transpose(-1, -2), ci) * lam4
                    wu = w * t.u
                    dlam += wu.sum(dim=(0, 2, 3))
                    lwu = wu * lam4
                    dg[:, :, i0:i1] += lwu.sum(-1)
                    dg[:, :, j0:j1] -= lwu.sum(-2)
                    if dF is not None:
                        dF[:, :, i0:i1] += ds.sum(-1)
                        dF[:, :, j0:j1] -= ds.sum(-2)
        return dq, dk, dv, dc, db, dg, dlam, dF, None


def sisa_attention_torch(q: Tensor, k: Tensor, v: Tensor, c: Tensor, b: Tensor, g: Tensor, lam: Tensor,
                         fgate: Tensor | None = None, block_q: int = 256) -> Tensor:
    """Exact SISA attention in plain PyTorch (src/sisa/functional.py:106), on any device, d_head and even
    d_state, differentiable w.r.t. every tensor argument.

    Works in fp32 (fp64 inputs stay fp64) with autocast off, over tiles of ``block_q`` queries by
    ``block_q`` keys, so memory grows with L * block_q rather than L^2 in both passes. Returns
    (B, H, L, d_head) in q.dtype."""
    if q.dim() != 4:
        raise ValueError(f"q must be (B, H, L, d_head), got shape {tuple(q.shape)}")
    B, H, L, _ = q.shape
    if k.shape != q.shape or v.shape[:3] != q.shape[:3]:
        raise ValueError(f"q, k, v shapes do not match: {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    if c.shape[:3] != q.shape[:3] or b.shape != c.shape or c.shape[-1] % 2 != 0:
        raise ValueError(f"c and b must be (B, H, L, d_state) with even d_state, got {tuple(c.shape)}, "
                         f"{tuple(b.shape)}")
    if g.shape != q.shape[:3] or (fgate is not None and fgate.shape != g.shape):
        raise ValueError("g and fgate must be (B, H, L)")
    if lam.shape != (H,):
        raise ValueError(f"lam must be ({H},), got {tuple(lam.shape)}")
    if block_q <= 0:
        raise ValueError("block_q must be positive")
    wd = compute_dtype(q.dtype)
    args = [t.to(wd) for t in (q, k, v, c, b, g, lam)] + [None if fgate is None else fgate.to(wd)]
    with no_autocast(q.device.type):
        out = _TorchAttention.apply(*args, int(block_q))
    return out.to(q.dtype)


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
