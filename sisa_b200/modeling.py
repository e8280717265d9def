"""SISA language model: pre-norm blocks of SISA attention and SwiGLU, tied embedding
(mirrors src/sisa/modeling.py; state-dict keys and initialisation are the reference's).

The ``cuda`` implementation runs the fused layer core: one projection GEMM (cuBLAS through
``F.linear``) into the fused column layout, then the sm_100a preparation and attention kernels
(:func:`sisa_b200.kernels.fused.sisa_fused`). ``fused_ce=True`` computes the loss with the chunked
linear + cross-entropy kernels; decoding with a cache uses the incremental-decode kernel.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING, Any, Iterable

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch import Tensor
from torch.utils.checkpoint import checkpoint

from .config import ATTN_IMPLS, SISAConfig
from .functional import attention_rows, compute_dtype, no_autocast, rotate_pairs, sisa_attention

if TYPE_CHECKING:  # pragma: no cover
    from .generation import SISACache

__all__ = ["RMSNorm", "SwiGLU", "SISAAttention", "SISABlock", "SISAModel", "SISAForCausalLM", "SISAOutput"]

IGNORE_INDEX = -100


def _fused_kernels(x: Tensor, config: SISAConfig | None) -> bool:
    """The sm_100a RMSNorm/SwiGLU kernels serve a block when its attention path is not ``"torch"`` and
    ``x`` is on a device those kernels run on; everything else takes the eager reference code."""
    if config is None or config.attn_impl == "torch" or not x.is_cuda:
        return False
    from . import backends

    return backends.cuda_status(x.device)[0]


class RMSNorm(nn.Module):
    """RMSNorm computed in fp32; output in the input's dtype (modeling.py:26-36). With a ``config`` whose
    attention path is not ``"torch"``, CUDA inputs take the fused kernel (kernels/norm.py)."""

    def __init__(self, dim: int, eps: float = 1e-6, config: SISAConfig | None = None):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps
        self._config = config

    def forward(self, x: Tensor) -> Tensor:
        if _fused_kernels(x, self._config):
            from .kernels.norm import rms_norm

            return rms_norm(x, self.weight, self.eps)
        norm = torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + self.eps)
        return ((x.float() * norm) * self.weight.float()).to(x.dtype)


class SwiGLU(nn.Module):
    """``w_down(silu(w_gate x) * w_up x)`` without biases (modeling.py:39-49); the activation takes the
    fused kernel under the same rule as RMSNorm."""

    def __init__(self, d_model: int, d_ff: int, config: SISAConfig | None = None):
        super().__init__()
        self.w_gate = nn.Linear(d_model, d_ff, bias=False)
        self.w_up = nn.Linear(d_model, d_ff, bias=False)
        self.w_down = nn.Linear(d_ff, d_model, bias=False)
        self._config = config

    def forward(self, x: Tensor) -> Tensor:
        return self.forward_split(x, x)

    def forward_fused(self, h: Tensor, dtype: torch.dtype) -> Tensor:
        """The forward with the gate and up projections and the activation in one tcgen05 GEMM
        (kernels/ffn.py), then ``w_down`` under autocast."""
        from .kernels.ffn import gate_up_swiglu
        from .kernels.linear import linear_cast, supports

        a = gate_up_swiglu(h, self.w_gate.weight, self.w_up.weight, dtype, self)
        if supports(a, self.w_down.weight, dtype):
            return linear_cast(a, self.w_down.weight, dtype, self, "w_down")
        return self.w_down(a)

    def forward_split(self, x_gate: Tensor, x_up: Tensor) -> Tensor:
        """The forward with the gate and up projections fed from separate copies of the input (the fused
        block path hands each its own copy, so that their gradients are summed in fp32)."""
        g, u = self.w_gate(x_gate), self.w_up(x_up)
        if _fused_kernels(x_gate, self._config) and g.dtype == u.dtype:
            from .kernels.norm import swiglu

            return self.w_down(swiglu(g, u))
        return self.w_down(F.silu(g) * u)


def _cast_keep_fp32(fn: Any, t: Tensor) -> Tensor:
    """``fn(t)``, except that a result in fp16/bf16 is replaced by ``t`` in fp32 on the result's device."""
    out = fn(t)
    if out.dtype in (torch.float16, torch.bfloat16):
        out = t.to(device=out.device, dtype=torch.float32)
    return out


def _static(owner: nn.Module, name: str, make, *tensors: Tensor):
    """``make(*tensors)``, kept on ``owner`` under ``name`` while none of ``tensors`` changed (same storage,
    version and dtype). For the decode step, which runs without autograd and would otherwise recompute
    these weight-only values (fp32 copies, concatenations) every token; a captured decode graph reads
    the kept tensors, which stay valid while the weights are unchanged. A fused optimizer changes the
    weights without advancing their versions: after its steps (our Trainer does this itself) call
    ``torch.autograd.graph.increment_version`` on the parameters before decoding."""
    key = tuple((t.data_ptr(), t._version, t.dtype) for t in tensors)
    hit = owner.__dict__.get(name)
    if hit is None or hit[0] != key:
        hit = (key, make(*tensors))
        owner.__dict__[name] = hit
    return hit[1]


def _fp32(*tensors: Tensor) -> tuple[Tensor, ...]:
    return tuple(t.float().contiguous() for t in tensors)


def _compute_dtype(x: Tensor) -> torch.dtype:
    dt = x.device.type
    try:
        if torch.is_autocast_enabled(dt):
            return torch.get_autocast_dtype(dt)
    except (TypeError, RuntimeError):
        pass
    return x.dtype


def _resolve_impl(requested: str, x: Tensor, config: SISAConfig) -> str:
    """``"torch"`` or ``"cuda"`` for layer input ``x`` (modeling.py:60-76)."""
    if requested not in ATTN_IMPLS:
        raise ValueError(f"attn_impl must be one of {ATTN_IMPLS}, got {requested!r}")
    if requested == "torch":
        return "torch"
    if x.device.type != "cuda":
        if requested == "auto":
            return "torch"
        raise ValueError(f"attn_impl={requested!r} needs a CUDA tensor, got one on {x.device.type}; "
                         "use attn_impl='torch' or 'auto'")
    from . import backends

    return backends.select_impl(requested, x, config)


class SISAAttention(nn.Module):
    """SISA attention sublayer: projections, recurrences, attention and output projection.

    Parameters (paper-checkpoint row layouts, modeling.py:79-141): ``W_Q, W_K, W_V, W_O`` (d -> d);
    ``W_B, W_C`` (d -> H*d_state); ``alpha_proj`` (d -> H, decay, with bias); ``theta_proj``
    (d -> H*d_state/2, rotation rate); ``forget_proj`` (d -> H, with bias); ``lambda_raw`` (H),
    ``lam = softplus(lambda_raw)``, kept in fp32 when the module is cast to bf16/fp16.
    """

    def __init__(self, config: SISAConfig, layer_idx: int = 0):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        d, h, s = config.d_model, config.n_head, config.d_state
        self.W_Q = nn.Linear(d, d, bias=False)
        self.W_K = nn.Linear(d, d, bias=False)
        self.W_V = nn.Linear(d, d, bias=False)
        self.W_O = nn.Linear(d, d, bias=False)
        self.W_B = nn.Linear(d, h * s, bias=False)
        self.W_C = nn.Linear(d, h * s, bias=False)
        self.alpha_proj = nn.Linear(d, h, bias=True)
        self.theta_proj = nn.Linear(d, h * (s // 2), bias=False)
        self.forget_proj = nn.Linear(d, h, bias=True)
        self.lambda_raw = nn.Parameter(torch.full((h,), float(config.lambda_raw_init)))
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self) -> None:
        """The SISA initialisation: weights ~ N(0, std) with std from the table below (W_C zero when
        zero_init_c), the decay and forget biases and lambda_raw at their configured constants."""
        cfg = self.config
        stds = {"W_Q": cfg.init_std, "W_K": cfg.init_std, "W_V": cfg.init_std, "W_O": cfg.init_std,
                "W_B": cfg.init_std, "W_C": 0.0 if cfg.zero_init_c else cfg.init_std,
                "alpha_proj": cfg.init_std, "theta_proj": cfg.theta_init_std, "forget_proj": cfg.init_std}
        for name, std in stds.items():
            w = getattr(self, name).weight
            if std > 0:
                w.normal_(0.0, std)
            else:
                w.zero_()
        self.alpha_proj.bias.fill_(cfg.decay_bias_init)
        self.forget_proj.bias.fill_(cfg.forget_bias_init)
        self.lambda_raw.fill_(cfg.lambda_raw_init)

    def _apply(self, fn: Any, recurse: bool = True) -> "SISAAttention":
        """Module-wide casts and moves (``.to``, ``.cuda``, ``.bfloat16`` ...) reach every tensor, but
        lambda_raw (and its gradient) never drops below fp32: a cast to fp16/bf16 only moves it to the
        target device with its fp32 value intact; other casts (fp64) apply as usual. The parameter stays
        the same object, so optimizers that hold it keep working."""
        lam = self._parameters.pop("lambda_raw")
        try:
            super()._apply(fn, recurse)
        finally:
            self._parameters["lambda_raw"] = lam
        with torch.no_grad():
            data = _cast_keep_fp32(fn, lam.data)
            grad = None if lam.grad is None else _cast_keep_fp32(fn, lam.grad)
            if torch._has_compatible_shallow_copy_type(lam, data):
                lam.data = data
                lam.grad = grad
            else:                                   # e.g. to_empty() from the meta device: a new parameter
                new = nn.Parameter(data, requires_grad=lam.requires_grad)
                new.grad = grad
                self._parameters["lambda_raw"] = new
        return self

    def lam(self) -> Tensor:
        return F.softplus(self.lambda_raw).float()

    def _forget_logits(self, x: Tensor) -> Tensor:
        with no_autocast(x.device.type):
            return F.linear(x.float(), self.forget_proj.weight.float(), self.forget_proj.bias.float())

    def projection_weights(self) -> list[Tensor]:
        """The weights of the fused projection in column order: W_Q, W_K, W_V, W_B, W_C, W_theta, W_alpha."""
        return [self.W_Q.weight, self.W_K.weight, self.W_V.weight, self.W_B.weight, self.W_C.weight,
                self.theta_proj.weight, self.alpha_proj.weight]

    def fused_weights(self) -> tuple[Tensor, Tensor]:
        from .kernels.fused import concat_fused_weights

        return concat_fused_weights(self.W_Q.weight, self.W_K.weight, self.W_V.weight, self.W_B.weight,
                                    self.W_C.weight, self.theta_proj.weight, self.alpha_proj.weight,
                                    self.alpha_proj.bias)

    def _prepare(self, x: Tensor, state: Any = None):
        """Inputs of the unfused attention (the glue of src/sisa/modeling.py:171-199), computed from one
        projection GEMM over the concatenated weights (columns Q | K | V | B | C | theta | alpha, the
        alpha bias the only bias), then the recurrences in fp32: g = cumsum(-softplus(alpha)),
        Phi = cumsum(theta), F = cumsum(log sigmoid(z)), continued from the last cached position when a
        decode ``state`` is given, and the rotation of c and b by Phi. Returns q, k, v, c~, b~ in the
        compute dtype and g, F, Phi in fp32, all (B, H, L, .)."""
        B, L, _ = x.shape
        H, dh, ds = self.config.n_head, self.config.d_head, self.config.d_state
        widths = (dh, dh, dh, ds, ds, ds // 2, 1)
        lins = (self.W_Q, self.W_K, self.W_V, self.W_B, self.W_C, self.theta_proj, self.alpha_proj)
        n = H * sum(widths)
        pad = -n % 16                     # zero rows: every row of proj starts 16-byte aligned (kernel views)
        ab = self.alpha_proj.bias
        weight = torch.cat([lin.weight for lin in lins] + [self.W_Q.weight.new_zeros(pad, x.shape[-1])])
        bias = torch.cat([ab.new_zeros(n - H), ab, ab.new_zeros(pad)])
        proj = F.linear(x, weight, bias)
        heads = [part.view(B, L, H, w).transpose(1, 2)
                 for part, w in zip(proj.split([H * w for w in widths] + [pad], dim=-1), widths)]
        q, k, v, b, c, theta, alpha = heads
        z = self._forget_logits(x)
        with no_autocast(x.device.type):
            g = torch.cumsum(-F.softplus(alpha[..., 0].float()), dim=2)
            phi = torch.cumsum(theta.float(), dim=2)
            fgate = torch.cumsum(F.logsigmoid(z).transpose(1, 2), dim=2)
            if state is not None:
                g = g + state.g_last()
                phi = phi + state.phi.unsqueeze(2)
                fgate = fgate + state.f_last()
            c = rotate_pairs(c.float(), phi)
            b = rotate_pairs(b.float(), phi)
        cd = _compute_dtype(x)
        return q.to(cd), k.to(cd), v.to(cd), c.to(cd), b.to(cd), g, fgate, phi

    def _output(self, y: Tensor) -> Tensor:
        bsz, h, seq_len, dh = y.shape
        return self.W_O(y.transpose(1, 2).reshape(bsz, seq_len, h * dh))

    def _forward_fused(self, x: Tensor, z: Tensor | None = None, lam: Tensor | None = None) -> Tensor:
        """Projection, layer core and output projection (modeling.py:213-222); ``z`` is the forget
        projection of ``x`` when the caller computed it already (the fused block norm does), ``lam``
        this layer's softplus(lambda_raw) when the caller computed every layer's at once."""
        from .kernels.fused import sisa_fused

        bsz, seq_len, d = x.shape
        cd = _compute_dtype(x)
        if x.is_cuda and (cd != x.dtype or cd != self.W_Q.weight.dtype):
            from .kernels.fused import fused_projection

            # autocast's linear over a cached compute-dtype concatenation, lean bias gradient
            proj = fused_projection(x, self.projection_weights(), self.alpha_proj.bias, cd, self)
        else:
            weight, bias = self.fused_weights()
            proj = F.linear(x, weight, bias)
        y = sisa_fused(proj, self._forget_logits(x) if z is None else z, self.lam() if lam is None else lam,
                       self.config.n_head)
        from .kernels.linear import linear_cast, supports

        if supports(y, self.W_O.weight, cd):
            return linear_cast(y.reshape(bsz, seq_len, d), self.W_O.weight, cd, self, "W_O")
        return self.W_O(y.reshape(bsz, seq_len, d))

    def _fused_weights_static(self) -> tuple[Tensor, Tensor]:
        """``fused_weights()``, kept between calls while no gradient is recorded and no weight changed
        (decode reuses it every step)."""
        if torch.is_grad_enabled():
            return self.fused_weights()
        parts = (self.W_Q.weight, self.W_K.weight, self.W_V.weight, self.W_B.weight, self.W_C.weight,
                 self.theta_proj.weight, self.alpha_proj.weight, self.alpha_proj.bias)
        key = tuple((t.data_ptr(), t._version, t.dtype) for t in parts)
        hit = getattr(self, "_wcat_static", None)
        if hit is None or hit[0] != key:
            hit = (key, self.fused_weights())
            self._wcat_static = hit
        return hit[1]

    def _decode_fused(self, x: Tensor, state, z: Tensor | None = None) -> Tensor:
        """One decode step on the CUDA path: one projection GEMM, one kernel for the recurrences, the
        rotation and the cache append (kernels/decode.py ``decode_prep``), then the decode attention.
        ``z`` is the forget projection of ``x`` when the caller computed it already (the block norm does)."""
        from .kernels.decode import decode_attention, decode_prep

        weight, bias = self._fused_weights_static()
        proj = F.linear(x, weight, bias)
        q, c, g, fgate = decode_prep(proj, self._forget_logits(x) if z is None else z, state, self.config.n_head)
        lam = _static(self, "_lam_static", lambda t: F.softplus(t).float(), self.lambda_raw)
        return self._output(decode_attention(q, c, g, fgate, state, lam))

    def _prefill_fused(self, x: Tensor, cache: "SISACache", z: Tensor | None = None) -> Tensor:
        """A prompt into an empty cache on the CUDA path: one projection GEMM over the concatenated
        weights, the preparation kernel and the tcgen05 forward (kernels/fused.py ``prefill_layer``), with
        the cache filled from their outputs. ``z`` is the forget projection of ``x`` when the caller
        computed it already (the block norm does)."""
        from .kernels.fused import prefill_layer

        weight, bias = self._fused_weights_static()
        proj = F.linear(x, weight, bias)
        lam = _static(self, "_lam_static", lambda t: F.softplus(t).float(), self.lambda_raw)
        y, (k, v, b, g, fgate, phi) = prefill_layer(proj, self._forget_logits(x) if z is None else z, lam,
                                                     self.config.n_head)
        cache.update(self.layer_idx, k=k, v=v, b=b, g=g, fgate=fgate, phi=phi)
        return self.W_O(y)

    def _use_fused_prefill(self, x: Tensor, state, requested: str) -> bool:
        """A prompt into an empty cache on the CUDA path without autograd, in a low-precision compute
        dtype (the cache takes the projection's dtype)."""
        return (state is None and x.is_cuda and not torch.is_grad_enabled()
                and _compute_dtype(x) in (torch.bfloat16, torch.float16)
                and _resolve_impl(requested, x, self.config) == "cuda")

    def _use_fused_decode(self, x: Tensor, state, requested: str) -> bool:
        """One new token on the CUDA path without autograd, into a cache of the compute dtype."""
        return (state is not None and x.shape[1] == 1 and x.is_cuda and not torch.is_grad_enabled()
                and _resolve_impl(requested, x, self.config) == "cuda" and _compute_dtype(x) == state.k_buf.dtype)

    def _forward_cached(self, x: Tensor, cache: "SISACache", requested: str) -> Tensor:
        state = cache.get(self.layer_idx)
        if self._use_fused_decode(x, state, requested):
            return self._decode_fused(x, state)
        if self._use_fused_prefill(x, state, requested):
            return self._prefill_fused(x, cache)
        q, k, v, c, b, g, fgate, phi = self._prepare(x, state)
        if state is None:
            impl = _resolve_impl(requested, x, self.config)
            y = sisa_attention(q, k, v, c, b, g, self.lam(), fgate, impl="cuda" if impl == "cuda" else "torch",
                               block_q=self.config.torch_block_q)
            cache.update(self.layer_idx, k=k, v=v, b=b, g=g, fgate=fgate, phi=phi[:, :, -1])
            return self._output(y)
        start = state.length
        state = cache.update(self.layer_idx, k=k, v=v, b=b, g=g, fgate=fgate, phi=phi[:, :, -1])
        impl = _resolve_impl(requested, x, self.config) if x.is_cuda else "torch"
        if impl == "cuda" and q.shape[2] == 1:
            from .kernels.decode import decode_attention

            y = decode_attention(q, c, g, fgate, state, self.lam())
            return self._output(y)
        wd = compute_dtype(q.dtype)
        y, _ = attention_rows(q.to(wd), state.k.to(wd), state.v.to(wd), c.to(wd), state.b.to(wd), g.to(wd),
                              state.g.to(wd), self.lam().to(wd), fgate.to(wd), state.fgate.to(wd), start,
                              block=self.config.torch_block_q)
        return self._output(y.to(q.dtype))

    def forward(self, x: Tensor, *, cache: "SISACache | None" = None, impl: str | None = None) -> Tensor:
        requested = impl or self.config.attn_impl
        if cache is not None:
            return self._forward_cached(x, cache, requested)
        impl = _resolve_impl(requested, x, self.config)
        if impl == "cuda":
            return self._forward_fused(x)
        q, k, v, c, b, g, fgate, _ = self._prepare(x)
        y = sisa_attention(q, k, v, c, b, g, self.lam(), fgate, impl="torch", block_q=self.config.torch_block_q)
        return self._output(y)


class SISABlock(nn.Module):
    """``x + attn(attn_norm(x))`` then ``x + ffn(ffn_norm(x))`` (modeling.py:258-290)."""

    def __init__(self, config: SISAConfig, layer_idx: int = 0):
        super().__init__()
        self.config = config
        self.attn_norm = RMSNorm(config.d_model, config.norm_eps, config)
        self.attn = SISAAttention(config, layer_idx)
        self.ffn_norm = RMSNorm(config.d_model, config.norm_eps, config)
        self.ffn = SwiGLU(config.d_model, config.d_ff, config)
        self._reset_ffn_and_norms()

    @torch.no_grad()
    def _reset_ffn_and_norms(self) -> None:
        for lin in (self.ffn.w_gate, self.ffn.w_up, self.ffn.w_down):
            nn.init.normal_(lin.weight, std=self.config.init_std)
        nn.init.ones_(self.attn_norm.weight)
        nn.init.ones_(self.ffn_norm.weight)

    @torch.no_grad()
    def reset_parameters(self) -> None:
        self._reset_ffn_and_norms()
        self.attn.reset_parameters()

    def forward(self, x: Tensor, cache: "SISACache | None" = None) -> Tensor:
        if cache is None and self.fused_path(x):
            xs, m = self.forward_pair(x, None)
            return xs + m
        x = x + self.attn(self.attn_norm(x), cache=cache)
        return x + self.ffn(self.ffn_norm(x))

    def fused_path(self, x: Tensor) -> bool:
        """Whether :meth:`forward_pair` serves input ``x``: the norm kernels run and the attention takes
        the fused CUDA layer core."""
        return _fused_kernels(x, self.config) and _resolve_impl(self.config.attn_impl, x, self.config) == "cuda"

    def decode_pair_path(self, x: Tensor, cache: "SISACache") -> bool:
        """Whether :meth:`decode_pair` serves the one-token input ``x``: the norm kernels run and the
        attention takes the fused decode step."""
        return (x.shape[1] == 1 and _fused_kernels(x, self.config)
                and self.attn._use_fused_decode(x, cache.get(self.attn.layer_idx), self.config.attn_impl))

    def prefill_pair_path(self, x: Tensor, cache: "SISACache") -> bool:
        """Whether :meth:`prefill_pair` serves the prompt ``x``: the norm kernels run and the attention
        fills an empty cache through the fused layer core."""
        return (_fused_kernels(x, self.config)
                and self.attn._use_fused_prefill(x, cache.get(self.attn.layer_idx), self.config.attn_impl))

    def prefill_pair(self, x: Tensor, m: Tensor | None, cache: "SISACache") -> tuple[Tensor, Tensor]:
        """The prompt pass of the block in :meth:`decode_pair`'s form, the attention through the fused
        layer core into an empty cache."""
        return self.decode_pair(x, m, cache, prefill=True)

    def decode_pair(self, x: Tensor, m: Tensor | None, cache: "SISACache",
                    prefill: bool = False) -> tuple[Tensor, Tensor]:
        """One decode step of the block in :meth:`forward_pair`'s form: the previous block's residual add
        is folded into the attention norm, which also computes the forget projection in fp32 from its
        rounded output (the value the eager step's ``F.linear(h.float(), ...)`` reads). With ``prefill``
        the rows are a prompt and the attention fills the empty cache instead of decoding one token."""
        from .kernels.norm import block_norm, swiglu

        attn, ffn = self.attn, self.ffn
        wa, pw, pb, wf = _static(self, "_decode_fp32", _fp32, self.attn_norm.weight, attn.forget_proj.weight,
                                 attn.forget_proj.bias, self.ffn_norm.weight)
        if m is None:
            h, z = block_norm(x, wa, self.attn_norm.eps, proj=(pw, pb))
            xs = x
        else:
            xs, h, z = block_norm(x, wa, self.attn_norm.eps, res=m, proj=(pw, pb))
        a = attn._prefill_fused(h, cache, z) if prefill else attn._decode_fused(h, cache.get(attn.layer_idx), z)
        xs, f_in = block_norm(xs, wf, self.ffn_norm.eps, res=a)
        from .kernels import ffn as ffn_kernels

        d_ff = ffn.w_gate.weight.shape[0]
        if prefill and ffn_kernels.supports(f_in, d_ff, f_in.dtype):
            # the prompt's MLP: gate and up on the CTA-pair GEMM with the activation in its epilogue,
            # storing only the activation
            return xs, ffn.w_down(ffn_kernels.gate_up_swiglu(f_in, ffn.w_gate.weight, ffn.w_up.weight, f_in.dtype, ffn))
        # gate and up projections as one GEMM over the concatenated weights, the activation on its halves
        w_gu = _static(ffn, "_gate_up_static", lambda g, u: torch.cat([g, u]), ffn.w_gate.weight, ffn.w_up.weight)
        gu = F.linear(f_in, w_gu)
        return xs, ffn.w_down(swiglu(gu[..., :d_ff], gu[..., d_ff:]))

    def forward_pair(self, x: Tensor, m: Tensor | None, lam: Tensor | None = None) -> tuple[Tensor, Tensor]:
        """The block on the fused path, with the previous block's last residual add ``x + m`` folded into
        this block's first norm. Returns ``(x + m + attn, ffn)``: the caller (the next block, or the
        final norm) adds the second term. Each norm also writes its output in the dtype of the linears
        that read it, and the attention norm computes the fp32 forget projection, so neither the casts
        nor the separate gradient sums of eager PyTorch run (kernels/norm.py ``block_norm``). The MLP's
        gate and up projections and its activation run as one GEMM (kernels/ffn.py) where the widths
        allow, else as two linears and the activation kernel, each linear fed its own copy of the norm
        output. ``lam``: the attention's softplus(lambda_raw), when the caller computed it."""
        from .kernels.norm import block_norm

        cd = _compute_dtype(x)
        attn = self.attn
        fp = (attn.forget_proj.weight, attn.forget_proj.bias)
        if m is None:
            h, z = block_norm(x, self.attn_norm.weight, self.attn_norm.eps, out_dtypes=(cd,), proj=fp)
            xs = x
        else:
            xs, h, z = block_norm(x, self.attn_norm.weight, self.attn_norm.eps, res=m, out_dtypes=(cd,), proj=fp)
        a = attn._forward_fused(h, z, lam)
        from .kernels.ffn import supports

        if supports(x, self.ffn.w_gate.weight.shape[0], cd):
            xs, f_in = block_norm(xs, self.ffn_norm.weight, self.ffn_norm.eps, res=a, out_dtypes=(cd,))
            return xs, self.ffn.forward_fused(f_in, cd)
        xs, f_gate, f_up = block_norm(xs, self.ffn_norm.weight, self.ffn_norm.eps, res=a, out_dtypes=(cd, cd))
        return xs, self.ffn.forward_split(f_gate, f_up)


@dataclass
class SISAOutput:
    loss: Tensor | None = None
    logits: Tensor | None = None


def _lm_logits(hidden: Tensor, weight: Tensor) -> Tensor:
    """``F.linear(hidden, weight)`` for inference. With 16-bit CUDA tensors and a vocabulary that is not a
    multiple of 8 the product is written into rows padded to a multiple of 8 and returned as a view:
    the same GEMM, but cuBLAS then takes an aligned kernel (an odd row stride of 50,277 made it fall
    back to an unaligned one at about a third of the bandwidth in the decode step)."""
    V = weight.shape[0]
    if (hidden.is_cuda and not torch.is_grad_enabled() and V % 8 and hidden.dtype == weight.dtype
            and hidden.dtype in (torch.bfloat16, torch.float16) and not torch.is_autocast_enabled("cuda")):
        h2 = hidden.reshape(-1, hidden.shape[-1])
        out = torch.empty((h2.shape[0], V + (-V % 8)), dtype=hidden.dtype, device=hidden.device)
        torch.mm(h2, weight.t(), out=out[:, :V])
        return out[:, :V].view(*hidden.shape[:-1], V)
    return F.linear(hidden, weight)


def _lm_head_loss(hidden: Tensor, weight: Tensor, labels: Tensor) -> Tensor:
    logits = F.linear(hidden, weight)
    return F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), labels.reshape(-1), ignore_index=IGNORE_INDEX)


class SISAModel(nn.Module):
    """Embedding, ``n_layer`` blocks and the final RMSNorm (modeling.py:308-414)."""

    def __init__(self, config: SISAConfig):
        super().__init__()
        self.config = config.replace()
        cfg = self.config
        self.embed = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.layers = nn.ModuleList([SISABlock(cfg, i) for i in range(cfg.n_layer)])
        self.final_norm = RMSNorm(cfg.d_model, cfg.norm_eps, cfg)
        self._reset_embedding_and_norm()

    @torch.no_grad()
    def _reset_embedding_and_norm(self) -> None:
        nn.init.normal_(self.embed.weight, std=self.config.init_std)
        nn.init.ones_(self.final_norm.weight)

    @torch.no_grad()
    def reset_parameters(self) -> None:
        self._reset_embedding_and_norm()
        for layer in self.layers:
            layer.reset_parameters()

    def _layer_lams(self) -> tuple[Tensor, ...] | None:
        """softplus(lambda_raw) of every layer in one launch (a stack and one softplus; one softplus
        backward for all of them), when the layers' lambda_raw share dtype and device; else None and
        each layer computes its own. The layers take their rows through ``unbind``, whose backward
        stacks the rows' gradients in one launch (indexing would zero-fill and add once per layer)."""
        raws = [layer.attn.lambda_raw for layer in self.layers]
        if len(raws) < 2 or any(r.dtype != raws[0].dtype or r.device != raws[0].device or r.shape != raws[0].shape
                                for r in raws):
            return None
        return F.softplus(torch.stack(raws)).float().unbind(0)

    def _lookup(self, input_ids: Tensor) -> Tensor:
        """The token embedding; a plain ``nn.Embedding`` (no padding index, norm limit or frequency
        scaling) takes its weight gradient from the deterministic CUDA kernel (``kernels.embedding``)."""
        e = self.embed
        if e.padding_idx is None and e.max_norm is None and not e.scale_grad_by_freq and not e.sparse:
            from .kernels.embedding import embedding

            return embedding(input_ids, e.weight)
        return e(input_ids)

    def forward(self, input_ids: Tensor, *, cache: "SISACache | None" = None) -> Tensor:
        x = self._lookup(input_ids)
        use_ckpt = self.config.gradient_checkpointing and self.training and cache is None and torch.is_grad_enabled()
        if cache is None and len(self.layers) and self.layers[0].fused_path(x):
            from .kernels.weights import refresh

            refresh(self, _compute_dtype(x))        # every stale compute-dtype weight copy, one launch
            lams = self._layer_lams()
            m = None
            for i, layer in enumerate(self.layers):
                lam = None if lams is None else lams[i]
                x, m = (checkpoint(layer.forward_pair, x, m, lam, use_reentrant=False) if use_ckpt
                        else layer.forward_pair(x, m, lam))
            from .kernels.norm import block_norm

            return block_norm(x, self.final_norm.weight, self.final_norm.eps, res=m, keep_sum=False)[0]
        if (cache is not None and len(self.layers) and x.shape[1] > 1
                and all(layer.prefill_pair_path(x, cache) for layer in self.layers)):
            from .kernels.norm import block_norm

            m = None
            for layer in self.layers:
                x, m = layer.prefill_pair(x, m, cache)
            (wn,) = _static(self, "_final_fp32", _fp32, self.final_norm.weight)
            return block_norm(x, wn, self.final_norm.eps, res=m, keep_sum=False)[0]
        if cache is not None and len(self.layers) and all(layer.decode_pair_path(x, cache) for layer in self.layers):
            from .kernels.norm import block_norm

            m = None
            for layer in self.layers:
                x, m = layer.decode_pair(x, m, cache)
            (wn,) = _static(self, "_final_fp32", _fp32, self.final_norm.weight)
            return block_norm(x, wn, self.final_norm.eps, res=m, keep_sum=False)[0]
        for layer in self.layers:
            x = checkpoint(layer, x, use_reentrant=False) if use_ckpt else layer(x, cache=cache)
        return self.final_norm(x)

    def set_attn_impl(self, impl: str) -> None:
        self.config.replace(attn_impl=impl)
        self.config.attn_impl = impl

    def num_parameters(self, exclude_embeddings: bool = False) -> int:
        n = sum(p.numel() for p in self.parameters())
        return n - self.embed.weight.numel() if exclude_embeddings else n

    def param_groups(self, lr: float, weight_decay: float = 0.1, lambda_lr: float | None = None,
                     no_decay_timescale_biases: bool = True) -> list[dict[str, Any]]:
        """Optimizer groups (the reference's groups, src/sisa/modeling.py:366-394): "default" (every other
        parameter, with weight decay), "timescale_biases" (the alpha and forget biases, no decay; only
        with ``no_decay_timescale_biases``) and "lambda" (lambda_raw, no decay, at ``lambda_lr``, which
        defaults to ``lr``). Empty groups are left out."""
        def group_of(name: str) -> str:
            if name.endswith("lambda_raw"):
                return "lambda"
            if no_decay_timescale_biases and name.rsplit(".", 2)[-2:] in (["alpha_proj", "bias"],
                                                                          ["forget_proj", "bias"]):
                return "timescale_biases"
            return "default"

        members: dict[str, list[nn.Parameter]] = {"default": [], "timescale_biases": [], "lambda": []}
        for name, p in self.named_parameters():
            if p.requires_grad:
                members[group_of(name)].append(p)
        settings = {"default": (lr, weight_decay), "timescale_biases": (lr, 0.0),
                    "lambda": (lr if lambda_lr is None else lambda_lr, 0.0)}
        return [{"params": ps, "lr": settings[g][0], "weight_decay": settings[g][1], "name": g}
                for g, ps in members.items() if ps or g == "default"]


class SISAForCausalLM(SISAModel):
    """:class:`SISAModel` with the tied LM head; labels are shifted internally (HF convention,
    modeling.py:417-481)."""

    def __init__(self, config: SISAConfig):
        super().__init__(config)
        self._loss_fn = _lm_head_loss

    def forward(self, input_ids: Tensor, labels: Tensor | None = None, *, cache: "SISACache | None" = None,
                fused_ce: bool = False, return_logits: bool = True, logits_to_keep: int = 0) -> SISAOutput:
        if labels is not None and labels.shape != input_ids.shape:
            raise ValueError(f"labels shape {tuple(labels.shape)} must match input_ids {tuple(input_ids.shape)}")
        if labels is not None and logits_to_keep:
            raise ValueError("logits_to_keep cannot be combined with labels")
        hidden = super().forward(input_ids, cache=cache)
        weight = self.embed.weight
        if labels is None:
            logits = None
            if return_logits:
                logits = _lm_logits(hidden[:, -logits_to_keep:] if logits_to_keep else hidden, weight)
            return SISAOutput(logits=logits)
        # position t predicts token t + 1: the last position has no target, the first token no prediction
        inputs, targets = hidden[:, :-1], labels[:, 1:]
        if fused_ce:
            if not hidden.is_cuda:
                raise ValueError("fused_ce=True needs CUDA tensors")
            from .kernels.linear_ce import linear_cross_entropy

            # every position with the next token as its label and the last position ignored: the same
            # rows and loss as hidden[:, :-1] against labels[:, 1:], without copying the sliced hidden
            # states forward and their gradient back
            shifted = F.pad(targets, (0, 1), value=IGNORE_INDEX)
            loss = linear_cross_entropy(hidden.reshape(-1, hidden.shape[-1]), weight, shifted.reshape(-1),
                                        ignore_index=IGNORE_INDEX)
            return SISAOutput(loss=loss)
        if not return_logits:
            return SISAOutput(loss=self._loss_fn(inputs, weight, targets))
        logits = F.linear(hidden, weight)
        loss = F.cross_entropy(logits[:, :-1].flatten(0, 1).float(), targets.flatten(), ignore_index=IGNORE_INDEX)
        return SISAOutput(loss=loss, logits=logits)

    def generate(self, input_ids: Tensor, max_new_tokens: int, temperature: float = 1.0, top_k: int | None = None,
                 eos_token_id: int | Iterable[int] | Tensor | None = None, do_sample: bool = False,
                 **kwargs: Any) -> Tensor:
        from .generation import generate

        return generate(self, input_ids, max_new_tokens, temperature=temperature, top_k=top_k,
                        eos_token_id=eos_token_id, do_sample=do_sample, **kwargs)

    def save_pretrained(self, path: str, *, safe_serialization: bool = True) -> None:
        """Write ``config.json`` and the weights to directory ``path`` (modeling.py:484-488)."""
        from .checkpoint import save_pretrained

        save_pretrained(self, path, safe_serialization=safe_serialization)

    @classmethod
    def from_pretrained(cls, path: str, *, dtype: torch.dtype | None = None,
                        **config_overrides: Any) -> "SISAForCausalLM":
        """Load a directory written by :meth:`save_pretrained` here or in the reference."""
        from .checkpoint import from_pretrained

        return from_pretrained(path, dtype=dtype, **config_overrides)
