"""Model configuration and the paper presets (mirrors src/sisa/config.py of tlstngud/sisa).

``attn_impl`` accepts the reference's values plus ``"cuda"``. ``"triton"`` and ``"triton_fused"``
are accepted as aliases of ``"cuda"`` so that configurations written for the reference load
unchanged; there is no Triton code in this package.
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass
from typing import Any, Mapping

__all__ = ["SISAConfig", "PRESETS", "ATTN_IMPLS", "CUDA_D_HEAD", "CUDA_D_STATE"]

#: Accepted values of :attr:`SISAConfig.attn_impl` (src/sisa/config.py:12 plus "cuda").
ATTN_IMPLS = ("auto", "torch", "cuda", "triton", "triton_fused")
#: Implementation names that select the CUDA kernels of this package.
CUDA_ALIASES = ("cuda", "triton", "triton_fused")

#: Head and state sizes the sm_100a kernels are compiled for.
CUDA_D_HEAD = 64
CUDA_D_STATE = 32


@dataclass
class SISAConfig:
    """Hyper-parameters of a SISA language model (defaults: the 50M paper model ``sisa-50m``).

    Field meanings and validation follow src/sisa/config.py:19-93.
    """

    vocab_size: int = 50277
    d_model: int = 512
    n_layer: int = 6
    n_head: int = 8
    d_ff: int = 1829
    d_state: int = 32
    norm_eps: float = 1e-6
    init_std: float = 0.02
    theta_init_std: float = 0.01
    decay_bias_init: float = -5.0
    forget_bias_init: float = 4.0
    lambda_raw_init: float = -1.0
    zero_init_c: bool = True
    max_seq_len: int = 2048
    attn_impl: str = "auto"
    torch_block_q: int = 256
    gradient_checkpointing: bool = False

    def __post_init__(self) -> None:
        for name in ("vocab_size", "d_model", "n_layer", "n_head", "d_ff", "d_state",
                     "max_seq_len", "torch_block_q"):
            value = getattr(self, name)
            if isinstance(value, bool) or not isinstance(value, int) or value <= 0:
                raise ValueError(f"{name} must be a positive integer, got {value!r}")
        if self.d_model % self.n_head != 0:
            raise ValueError(f"d_model ({self.d_model}) must be divisible by n_head ({self.n_head})")
        if self.d_state % 2 != 0:
            raise ValueError(f"d_state must be even (channels are rotated in pairs), got {self.d_state}")
        if self.norm_eps <= 0:
            raise ValueError(f"norm_eps must be positive, got {self.norm_eps}")
        if self.attn_impl not in ATTN_IMPLS:
            raise ValueError(f"attn_impl must be one of {ATTN_IMPLS}, got {self.attn_impl!r}")
        if self.attn_impl in CUDA_ALIASES:
            if self.d_head != CUDA_D_HEAD or self.d_state != CUDA_D_STATE:
                raise ValueError(
                    f"attn_impl={self.attn_impl!r} requires d_head={CUDA_D_HEAD} and d_state={CUDA_D_STATE} "
                    f"(got d_head={self.d_head}, d_state={self.d_state}); use attn_impl='torch' or 'auto'")

    @property
    def d_head(self) -> int:
        return self.d_model // self.n_head

    def num_parameters(self) -> int:
        """Analytic parameter count; the tied LM head is counted once (src/sisa/config.py:100-114)."""
        d, h, s, f = self.d_model, self.n_head, self.d_state, self.d_ff
        per_layer = (4 * d * d + 2 * h * s * d + h * (s // 2) * d + 2 * (h * d + h) + h + 2 * d + 3 * d * f)
        return self.n_layer * per_layer + self.vocab_size * d + d

    def to_dict(self) -> dict[str, Any]:
        return dataclasses.asdict(self)

    @classmethod
    def from_dict(cls, data: Mapping[str, Any], **overrides: Any) -> "SISAConfig":
        merged = {**dict(data), **overrides}
        known = {f.name for f in dataclasses.fields(cls)}
        unknown = sorted(set(merged) - known)
        if unknown:
            raise ValueError(f"unknown SISAConfig fields: {unknown}")
        return cls(**merged)

    @classmethod
    def preset(cls, name: str, **overrides: Any) -> "SISAConfig":
        try:
            base = PRESETS[name]
        except KeyError:
            raise ValueError(f"unknown preset {name!r}; available: {sorted(PRESETS)}") from None
        return cls.from_dict(base, **overrides)

    def replace(self, **changes: Any) -> "SISAConfig":
        return dataclasses.replace(self, **changes)


#: Paper model sizes (src/sisa/config.py:145-149). Parameter counts 50,911,376 / 151,878,576 / 369,278,080.
PRESETS: dict[str, dict[str, Any]] = {
    "sisa-50m": dict(d_model=512, n_layer=6, n_head=8, d_ff=1829),
    "sisa-152m": dict(d_model=768, n_layer=12, n_head=12, d_ff=2744),
    "sisa-369m": dict(d_model=1024, n_layer=24, n_head=16, d_ff=2507),
}
