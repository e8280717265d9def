"""CPU oracle of the SISA hot path - TEST INFRASTRUCTURE, not part of the product.

A plain-PyTorch (CPU, fp64 by default) restatement of tlstngud/sisa's pure-PyTorch reference for the
path the B200 kernels implement. It is the checker the GPU parity tests compare against, and the
CPU baseline that ``bench.py`` times; the product package ``sisa_b200`` never imports it.

Pinned against fixtures produced by the reference itself (``tests/golden/make_golden.py`` imports
the reference package from its source tree in the build container and stores inputs/outputs under
``tests/golden/``); ``tests/test_oracle_golden.py`` checks this module against them.

Every function cites the reference file:line (paths inside the reference project) it restates.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

D_HEAD = 64
D_STATE = 32
LOG2E = 1.4426950408889634


def fused_layout(n_head: int) -> dict:
    """Column layout of the fused projection (src/sisa/kernels/fused_prep.py:71-96)."""
    H = int(n_head)
    o = {"Q": 0, "K": H * 64, "V": 2 * H * 64, "B": 3 * H * 64, "C": 3 * H * 64 + H * 32,
         "TH": 3 * H * 64 + 2 * H * 32}
    o["A"] = o["TH"] + H * 16
    o["NTOT"] = o["A"] + H
    o["NPAD"] = (o["NTOT"] + 15) // 16 * 16
    return o


def rotate_pairs(z: torch.Tensor, phi: torch.Tensor) -> torch.Tensor:
    """Rotate interleaved pairs (0,1),(2,3),... of z by phi (src/sisa/functional.py:38-50)."""
    ze, zo = z[..., 0::2], z[..., 1::2]
    c, s = torch.cos(phi), torch.sin(phi)
    return torch.stack([ze * c - zo * s, ze * s + zo * c], dim=-1).flatten(-2)


def prep(proj: torch.Tensor, z: torch.Tensor | None, n_head: int, dtype=torch.float64) -> dict:
    """g, F, Phi and the rotated C/B from the fused projection, in ``dtype`` with no rounding.

    Restates the torch glue src/sisa/modeling.py:171-199 on the fused column layout of
    src/sisa/kernels/fused_prep.py:71-96 (the fused kernels compute the same functions,
    fused_prep.py:277-352): g = cumsum(-softplus(alpha)), Phi = cumsum(theta),
    F = cumsum(logsigmoid(z)), c~ = R(Phi) c, b~ = R(Phi) b. Returns (B, H, L, .) tensors.
    """
    B, L, _ = proj.shape
    H = n_head
    off = fused_layout(H)
    P = proj.to(dtype)

    def cols(name, w):
        return P[..., off[name]:off[name] + H * w].reshape(B, L, H, w).transpose(1, 2)

    alpha = P[..., off["A"]:off["A"] + H].transpose(1, 2)
    theta = cols("TH", D_STATE // 2)
    g = torch.cumsum(-F.softplus(alpha), dim=2)
    phi = torch.cumsum(theta, dim=2)
    out = dict(q=cols("Q", 64), k=cols("K", 64), v=cols("V", 64), g=g, phi=phi,
               c=rotate_pairs(cols("C", 32), phi), b=rotate_pairs(cols("B", 32), phi))
    out["F"] = None if z is None else torch.cumsum(F.logsigmoid(z.to(dtype)).transpose(1, 2), dim=2)
    return out


def attention(q, k, v, c, b, g, lam, fgate=None, block_q: int = 512):
    """Exact SISA attention, dense and blocked over queries (src/sisa/functional.py:69-155).

    s_ij = q_i.k_j / sqrt(d) + lam_h exp(g_i - g_j)(c_i.b_j) + (F_i - F_j), j <= i; o = softmax(s) v.
    Works in the inputs' dtype (callers pass fp64). Returns (o, lse2) with lse2 = log2 sum_j exp(s_ij),
    the statistic the kernels store.
    """
    Bz, H, L, D = q.shape
    scale = 1.0 / math.sqrt(D)
    outs, lses = [], []
    for start in range(0, L, block_q):
        end = min(start + block_q, L)
        qi, ci, gi = q[:, :, start:end], c[:, :, start:end], g[:, :, start:end]
        kk, vv, bb, gk = k[:, :, :end], v[:, :, :end], b[:, :, :end], g[:, :, :end]
        pos_q = torch.arange(start, end).unsqueeze(1)
        causal = torch.arange(end).unsqueeze(0) <= pos_q
        s = torch.matmul(qi, kk.transpose(-1, -2)) * scale
        delta = (gi.unsqueeze(-1) - gk.unsqueeze(-2)).masked_fill(~causal, 0.0)
        s = s + lam.view(1, -1, 1, 1).to(q.dtype) * torch.exp(delta) * torch.matmul(ci, bb.transpose(-1, -2))
        if fgate is not None:
            s = s + (fgate[:, :, start:end].unsqueeze(-1) - fgate[:, :, :end].unsqueeze(-2))
        s = s.masked_fill(~causal, float("-inf"))
        lse = torch.logsumexp(s, dim=-1)
        outs.append(torch.matmul(torch.exp(s - lse.unsqueeze(-1)), vv))
        lses.append(lse * LOG2E)
    return torch.cat(outs, dim=2), torch.cat(lses, dim=2)


def attention_grads(q, k, v, c, b, g, lam, fgate, dout, dtype=torch.float64):
    """fp64 autograd truth of every attention input gradient (the reference's truth64 pattern,
    tests/test_attention_kernel.py:194-212). Returns dict o, dq, dk, dv, dc, db, dg, dlam, dF."""
    xs = [t.detach().to(dtype).requires_grad_(True) for t in (q, k, v, c, b, g, lam)]
    fg = None if fgate is None else fgate.detach().to(dtype).requires_grad_(True)
    o, _ = attention(*xs, fgate=fg)
    ins = xs + ([fg] if fg is not None else [])
    gr = torch.autograd.grad(o, ins, dout.to(dtype))
    names = ["dq", "dk", "dv", "dc", "db", "dg", "dlam"] + (["dF"] if fg is not None else [])
    res = dict(zip(names, gr))
    res["o"] = o.detach()
    if fg is None:
        res["dF"] = None
    return res


def _round_through(x: torch.Tensor, lowp) -> torch.Tensor:
    """Value rounded to ``lowp``, gradient passed through: the ``.to(compute_dtype)`` of the reference's
    torch glue under autocast (src/sisa/modeling.py:197-199)."""
    if lowp is None:
        return x
    return x + (x.detach().to(lowp).to(x.dtype) - x.detach())


def fused_layer(proj, z, lam, n_head, dtype=torch.float64, lowp=None):
    """y = heads-concatenated attention output of the fused layer core (src/sisa/kernels/fused_prep.py:637-683).

    ``lowp`` (e.g. torch.bfloat16) rounds the rotated c/b to the compute dtype as the reference's glue does
    before the attention; everything else stays in ``dtype``."""
    pr = prep(proj, z, n_head, dtype)
    c, b = _round_through(pr["c"], lowp), _round_through(pr["b"], lowp)
    o, lse = attention(pr["q"], pr["k"], pr["v"], c, b, pr["g"], lam.to(dtype), pr["F"])
    B, H, L, D = o.shape
    return o.transpose(1, 2).reshape(B, L, H * D), lse, pr


def fused_layer_grads(proj, z, lam, n_head, dy, dtype=torch.float64, lowp=None):
    """fp64 gradients of the fused layer w.r.t. proj, z and lam (the reference's ref64_fused pattern,
    tests/test_fused_prep.py:173-201). Returns y, dproj, dz, dlam."""
    P = proj.detach().to(dtype).requires_grad_(True)
    Z = None if z is None else z.detach().to(dtype).requires_grad_(True)
    LAM = lam.detach().to(dtype).requires_grad_(True)
    y, _, _ = fused_layer(P, Z, LAM, n_head, dtype, lowp=lowp)
    ins = [P, LAM] + ([Z] if Z is not None else [])
    gr = torch.autograd.grad(y, ins, dy.to(dtype))
    return y.detach(), gr[0], (gr[2] if Z is not None else None), gr[1]


def linear_cross_entropy(hidden, weight, labels, ignore_index: int = -100, dtype=torch.float64):
    """Mean CE of hidden @ weight^T over non-ignored rows and its gradients
    (src/sisa/kernels/linear_ce.py:220-224; labels are not shifted). Returns loss, dh, dw."""
    h = hidden.detach().to(dtype).requires_grad_(True)
    w = weight.detach().to(dtype).requires_grad_(True)
    logits = h @ w.t()
    loss = F.cross_entropy(logits, labels.reshape(-1), ignore_index=ignore_index)
    dh, dw = torch.autograd.grad(loss, [h, w])
    return loss.detach(), dh, dw


def decode_rows(q, c, g_q, f_q, k_cache, v_cache, b_cache, g_cache, f_cache, lam, start: int):
    """Attention of new rows at absolute positions start.. against a cache of keys 0..start+M-1
    (src/sisa/modeling.py:224-238 via src/sisa/functional.py:69-103)."""
    M = q.shape[2]
    N = k_cache.shape[2]
    scale = 1.0 / math.sqrt(q.shape[-1])
    pos_q = torch.arange(start, start + M).unsqueeze(1)
    causal = torch.arange(N).unsqueeze(0) <= pos_q
    s = torch.matmul(q, k_cache.transpose(-1, -2)) * scale
    delta = (g_q.unsqueeze(-1) - g_cache.unsqueeze(-2)).masked_fill(~causal, 0.0)
    s = s + lam.view(1, -1, 1, 1) * torch.exp(delta) * torch.matmul(c, b_cache.transpose(-1, -2))
    if f_q is not None:
        s = s + (f_q.unsqueeze(-1) - f_cache.unsqueeze(-2))
    s = s.masked_fill(~causal, float("-inf"))
    return torch.matmul(torch.softmax(s, dim=-1), v_cache)


# ---------------------------------------------------------------------------------------------
# Seeded inputs with the benchmark distributions: q,k,v ~ N(0,1);
# B,C ~ N(0,1); theta ~ N(0, 0.2^2); a ~ N(-5, 0.45^2); z ~ N(4, 0.45^2); lambda_raw = -1.
# ---------------------------------------------------------------------------------------------
def make_proj_inputs(B: int, L: int, H: int, seed: int = 0, dtype=torch.float32, theta_std: float = 0.2,
                     a_mean: float = -5.0, z_mean: float = 4.0, spread: float = 0.45):
    """(proj, z, lam) in the fused layout, generated in the fixed order q, k, v, B, C, theta, a, z."""
    gen = torch.Generator().manual_seed(seed)
    off = fused_layout(H)
    proj = torch.zeros(B, L, off["NPAD"], dtype=torch.float32)
    proj[..., off["Q"]:off["Q"] + H * 64] = torch.randn(B, L, H * 64, generator=gen)
    proj[..., off["K"]:off["K"] + H * 64] = torch.randn(B, L, H * 64, generator=gen)
    proj[..., off["V"]:off["V"] + H * 64] = torch.randn(B, L, H * 64, generator=gen)
    proj[..., off["B"]:off["B"] + H * 32] = torch.randn(B, L, H * 32, generator=gen)
    proj[..., off["C"]:off["C"] + H * 32] = torch.randn(B, L, H * 32, generator=gen)
    proj[..., off["TH"]:off["TH"] + H * 16] = torch.randn(B, L, H * 16, generator=gen) * theta_std
    proj[..., off["A"]:off["A"] + H] = torch.randn(B, L, H, generator=gen) * spread + a_mean
    z = torch.randn(B, L, H, generator=gen) * spread + z_mean
    lam = F.softplus(torch.full((H,), -1.0))
    return proj.to(dtype), z, lam
