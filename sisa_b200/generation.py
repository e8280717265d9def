"""Incremental decoding with a per-layer cache (mirrors src/sisa/generation.py).

Per head and cached token SISA keeps k, v, the rotated b~, the cumulative decay g and the cumulative
forget value F; the running phase Phi is kept for the last position only. Unlike the reference (which
re-concatenates every cached tensor at every step, generation.py:67-83), the cache here holds buffers
with spare capacity: an append copies only the new positions, and ``generate`` sizes the buffers for
prompt + max_new_tokens up front. On CUDA with the ``cuda`` implementation, the prompt runs through the
tcgen05 attention and each decode step through the split-K decode kernel
(:func:`sisa_b200.kernels.decode.decode_attention`).
"""
from __future__ import annotations

import numbers
from typing import TYPE_CHECKING, Iterable

import torch
from torch import Tensor

if TYPE_CHECKING:  # pragma: no cover
    from .modeling import SISAForCausalLM

__all__ = ["LayerState", "SISACache", "generate"]

_ROUND = 256


class LayerState:
    """Cached tensors of one layer: k, v ``(B, H, T, d_head)`` and b ``(B, H, T, d_state)`` in the compute
    dtype, g and fgate ``(B, H, T)`` fp32 (views of the first ``length`` positions of the buffers), phi
    ``(B, H, d_state/2)`` fp32 at the last position."""

    def __init__(self, k: Tensor, v: Tensor, b: Tensor, g: Tensor, fgate: Tensor, phi: Tensor,
                 capacity: int | None = None):
        B, H, T, D = k.shape
        cap = max(int(capacity or 0), T)
        cap = -(-cap // _ROUND) * _ROUND
        self._alloc(B, H, cap, D, b.shape[-1], k.dtype, k.device)
        self.length = 0
        self.phi = phi
        self.append(k, v, b, g, fgate, phi)

    def _alloc(self, B, H, cap, D, S, dtype, device):
        self.k_buf = torch.empty((B, H, cap, D), dtype=dtype, device=device)
        self.v_buf = torch.empty((B, H, cap, D), dtype=dtype, device=device)
        self.b_buf = torch.empty((B, H, cap, S), dtype=dtype, device=device)
        self.g_buf = torch.empty((B, H, cap), dtype=torch.float32, device=device)
        self.f_buf = torch.empty((B, H, cap), dtype=torch.float32, device=device)

    @property
    def capacity(self) -> int:
        return self.k_buf.shape[2]

    def reserve(self, n: int) -> None:
        """Make room for ``n`` more positions (the buffers grow by doubling)."""
        if self.length + n > self.capacity:
            old = (self.k_buf, self.v_buf, self.b_buf, self.g_buf, self.f_buf)
            B, H, _, D = self.k_buf.shape
            cap = -(-max(2 * self.capacity, self.length + n) // _ROUND) * _ROUND
            self._alloc(B, H, cap, D, self.b_buf.shape[-1], self.k_buf.dtype, self.k_buf.device)
            for dst, src in zip((self.k_buf, self.v_buf, self.b_buf, self.g_buf, self.f_buf), old):
                dst[:, :, :self.length].copy_(src[:, :, :self.length])

    def phi_buffer(self) -> Tensor:
        """``phi`` as an fp32 contiguous tensor this state owns (the fused decode step advances it in place)."""
        if not (self.phi.dtype == torch.float32 and self.phi.is_contiguous() and getattr(self, "_phi_owned", False)):
            self.phi = self.phi.float().contiguous().clone()
            self._phi_owned = True
        return self.phi

    def append(self, k: Tensor, v: Tensor, b: Tensor, g: Tensor, fgate: Tensor, phi: Tensor) -> None:
        n = k.shape[2]
        self.reserve(n)
        t0, t1 = self.length, self.length + n
        self.k_buf[:, :, t0:t1].copy_(k)
        self.v_buf[:, :, t0:t1].copy_(v)
        self.b_buf[:, :, t0:t1].copy_(b)
        self.g_buf[:, :, t0:t1].copy_(g)
        self.f_buf[:, :, t0:t1].copy_(fgate)
        self.phi = phi
        self._phi_owned = False
        self.length = t1

    @property
    def k(self) -> Tensor:
        return self.k_buf[:, :, :self.length]

    @property
    def v(self) -> Tensor:
        return self.v_buf[:, :, :self.length]

    @property
    def b(self) -> Tensor:
        return self.b_buf[:, :, :self.length]

    @property
    def g(self) -> Tensor:
        return self.g_buf[:, :, :self.length]

    @property
    def fgate(self) -> Tensor:
        return self.f_buf[:, :, :self.length]

    def g_last(self) -> Tensor:
        return self.g_buf[:, :, self.length - 1:self.length]

    def f_last(self) -> Tensor:
        return self.f_buf[:, :, self.length - 1:self.length]


class SISACache:
    """Decode cache holding one :class:`LayerState` per layer. ``capacity`` (positions) sizes the buffers."""

    def __init__(self, capacity: int | None = None) -> None:
        self._layers: dict[int, LayerState] = {}
        self.capacity = capacity

    def get(self, layer_idx: int) -> LayerState | None:
        return self._layers.get(layer_idx)

    def update(self, layer_idx: int, *, k: Tensor, v: Tensor, b: Tensor, g: Tensor, fgate: Tensor,
               phi: Tensor) -> LayerState:
        state = self._layers.get(layer_idx)
        if state is None:
            state = LayerState(k, v, b, g, fgate, phi, capacity=self.capacity)
            self._layers[layer_idx] = state
        else:
            state.append(k, v, b, g, fgate, phi)
        return state

    @property
    def seq_len(self) -> int:
        state = self._layers.get(0)
        return 0 if state is None else state.length

    def reset(self) -> None:
        self._layers.clear()

    def __len__(self) -> int:
        return len(self._layers)


def _eos_ids(eos_token_id) -> list[int]:
    """Normalise ``eos_token_id`` to a list of ints (generation.py:98-122)."""
    if eos_token_id is None:
        return []
    bad = TypeError(f"eos_token_id must be an integer or an iterable of integers, "
                    f"got {eos_token_id!r} ({type(eos_token_id).__name__})")
    if isinstance(eos_token_id, (bool, str, bytes)):
        raise bad
    if isinstance(eos_token_id, numbers.Integral):
        return [int(eos_token_id)]
    dtype = getattr(eos_token_id, "dtype", None)
    if dtype is not None:
        is_float = dtype.is_floating_point if torch.is_tensor(eos_token_id) else dtype.kind not in "iu"
        if is_float or getattr(eos_token_id, "ndim", 1) > 1:
            raise bad
        if getattr(eos_token_id, "ndim", None) == 0:
            return [int(eos_token_id)]
        return [int(t) for t in eos_token_id.tolist()]
    try:
        ids = list(eos_token_id)
    except TypeError:
        raise bad from None
    if not all(isinstance(t, numbers.Integral) and not isinstance(t, bool) for t in ids):
        raise bad
    return [int(t) for t in ids]


def _next_token(logits: Tensor, *, do_sample: bool, temperature: float, top_k: int | None,
                generator: torch.Generator | None) -> Tensor:
    logits = logits.float()
    if not do_sample:
        return logits.argmax(dim=-1)
    logits = logits / temperature
    if top_k is not None and top_k < logits.shape[-1]:
        kth = torch.topk(logits, top_k, dim=-1).values[..., -1:]
        logits = logits.masked_fill(logits < kth, float("-inf"))
    probs = torch.softmax(logits, dim=-1)
    return torch.multinomial(probs, num_samples=1, generator=generator).squeeze(-1)


@torch.no_grad()
def generate(model: "SISAForCausalLM", input_ids: Tensor, max_new_tokens: int, temperature: float = 1.0,
             top_k: int | None = None, eos_token_id: int | Iterable[int] | Tensor | None = None,
             do_sample: bool = False, *, generator: torch.Generator | None = None,
             eos_check_every: int = 16) -> Tensor:
    """Generate continuations of ``input_ids`` (generation.py:139-191).

    Same results as the reference. The all-finished check reads the device only every
    ``eos_check_every`` steps; the tokens generated past the step where every row had finished are
    cut off afterwards, so the returned length is the reference's.
    """
    if max_new_tokens < 0:
        raise ValueError("max_new_tokens must be >= 0")
    if do_sample and temperature <= 0:
        raise ValueError("temperature must be positive when do_sample=True")
    if top_k is not None and top_k <= 0:
        raise ValueError("top_k must be a positive integer")
    squeeze = input_ids.dim() == 1
    if squeeze:
        input_ids = input_ids.unsqueeze(0)
    if input_ids.dim() != 2 or input_ids.shape[1] == 0:
        raise ValueError("input_ids must be a non-empty (B, L) tensor")
    if max_new_tokens == 0:
        return input_ids.squeeze(0) if squeeze else input_ids
    eos = _eos_ids(eos_token_id)
    eos_t = torch.tensor(eos, device=input_ids.device, dtype=input_ids.dtype) if eos else None
    cache = SISACache(capacity=input_ids.shape[1] + max_new_tokens)
    logits = model(input_ids, cache=cache, logits_to_keep=1).logits[:, -1]
    pieces = [input_ids]
    done = torch.zeros(input_ids.shape[0], dtype=torch.bool, device=input_ids.device)
    all_done_at = []       # device flags: every row finished after step s
    for step in range(max_new_tokens):
        nxt = _next_token(logits, do_sample=do_sample, temperature=temperature, top_k=top_k,
                          generator=generator).to(input_ids.dtype)
        if eos_t is not None:
            nxt = torch.where(done, eos_t[0], nxt)
            done = done | torch.isin(nxt, eos_t)
            all_done_at.append(done.all())
        pieces.append(nxt.unsqueeze(1))
        if step + 1 == max_new_tokens:
            break
        if eos_t is not None and (step + 1) % eos_check_every == 0 and bool(all_done_at[-1]):
            break
        logits = model(nxt.unsqueeze(1), cache=cache, logits_to_keep=1).logits[:, -1]
    out = torch.cat(pieces, dim=1)
    if all_done_at:
        flags = torch.stack(all_done_at).cpu()
        hit = torch.nonzero(flags).flatten()
        if hit.numel():
            out = out[:, :input_ids.shape[1] + int(hit[0]) + 1]
    return out.squeeze(0) if squeeze else out
