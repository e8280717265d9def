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

__all__ = ["LayerState", "SISACache", "DecodeGraph", "generate"]

_ROUND = 256


def _copy_heads(dst: Tensor, src: Tensor) -> None:
    """``dst.copy_(src)`` for (B, H, T, width) tensors. Between 16-bit CUDA tensors whose last dimension is
    contiguous (the prompt's k and v are head views of the fused projection, strided by its row) one
    16-byte-vector kernel moves whole rows (``sisa_copy_heads``); anything else is torch's copy."""
    B, H, T, W = dst.shape
    ok = (dst.is_cuda and src.is_cuda and dst.dtype == src.dtype and dst.dtype in (torch.bfloat16, torch.float16)
          and tuple(src.shape) == (B, H, T, W) and dst.stride(-1) == 1 and src.stride(-1) == 1 and W % 8 == 0
          and H * W // 8 <= 256 and dst.data_ptr() % 16 == 0 and src.data_ptr() % 16 == 0
          and all(st % 8 == 0 for st in dst.stride()[:3] + src.stride()[:3]))
    if not ok:
        dst.copy_(src)
        return
    from . import _lib

    _lib.check(_lib.load().sisa_copy_heads(src.data_ptr(), *src.stride()[:3], dst.data_ptr(), *dst.stride()[:3],
                                           B, H, T, W, _lib.stream_ptr(dst.device)), "sisa_copy_heads")


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
        self.pos_dev: Tensor | None = None   # device position counter while a DecodeGraph drives this cache
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
        _copy_heads(self.k_buf[:, :, t0:t1], k)
        _copy_heads(self.v_buf[:, :, t0:t1], v)
        _copy_heads(self.b_buf[:, :, t0:t1], b)
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


class DecodeGraph:
    """One decode step of ``model`` captured once as a CUDA graph and replayed for every new token.

    The step is every layer's projection, recurrences, cache append, decode attention and MLP, then the
    final norm and the LM head of the new position. The reference's ``generate`` dispatches each of its
    kernels from Python for every token (generation.py:177-189); at decode batch sizes that host work,
    not the GPU, sets the step time. Here the kernels that depend on the position read it from an int32
    counter on the device (``pos_dev``, given to every layer state), and the graph advances the counter
    at its end, so one capture serves every position. :meth:`step` advances the host-side lengths of the
    layer states to match.

    Build it after at least one eager decode step into ``cache`` (that step creates the concatenated
    projection weights and the libraries' per-stream state), with room in the cache for every further
    step: the buffers must not move once captured. :meth:`close` detaches the counter from the cache.
    """

    def __init__(self, model: "SISAForCausalLM", cache: "SISACache", batch: int,
                 stream: "torch.cuda.Stream | None" = None):
        if not DecodeGraph.supported(model, cache):
            raise ValueError("DecodeGraph needs a CUDA model on the cuda attention path with a filled cache, no "
                             "autograd or autocast, and a check mode other than 'sync'")
        first = next(model.parameters())
        dev = first.device
        self.cache = cache
        self.states = [cache.get(i) for i in range(len(model.layers))]
        self.stream = stream if stream is not None else torch.cuda.Stream(dev)   # capture (and replay) stream
        self.ids = torch.zeros((batch, 1), dtype=torch.long, device=dev)
        self.pos_dev = torch.full((1,), cache.seq_len, dtype=torch.int32, device=dev)
        lengths = [st.length for st in self.states]
        for st in self.states:
            st.phi_buffer()
            st.pos_dev = self.pos_dev
        self.graph = torch.cuda.CUDAGraph()
        self.stream.wait_stream(torch.cuda.current_stream(dev))
        try:
            with torch.cuda.graph(self.graph, stream=self.stream):
                self.logits = model(self.ids, cache=cache, logits_to_keep=1).logits[:, -1]
                self.pos_dev.add_(1)
        except BaseException:
            self.close()
            raise
        finally:
            for st, n in zip(self.states, lengths):   # capture ran the host code once but no kernel
                st.length = n

    @staticmethod
    def supported(model: "SISAForCausalLM", cache: "SISACache") -> bool:
        from . import backends
        from .modeling import _resolve_impl

        first = next(model.parameters(), None)
        if first is None or not first.is_cuda or torch.is_grad_enabled() or torch.is_autocast_enabled("cuda"):
            return False
        if backends.get_check_mode() == "sync" or len(cache) != len(model.layers) or cache.seq_len < 1:
            return False
        dt = model.embed.weight.dtype
        if dt not in (torch.bfloat16, torch.float16):
            return False
        probe = torch.empty((1, 1, model.config.d_model), dtype=dt, device=first.device)
        return _resolve_impl(model.config.attn_impl, probe, model.config) == "cuda" and all(
            cache.get(i) is not None and cache.get(i).k_buf.dtype == dt for i in range(len(model.layers)))

    def room(self) -> int:
        """Steps left before the cache is full."""
        return min(st.capacity - st.length for st in self.states)

    def step(self, ids: Tensor) -> Tensor:
        """Feed one token per row (``ids``: (B,) or (B, 1)); returns the (B, vocab) logits of the new position
        (a buffer that the next step overwrites)."""
        if self.room() < 1:
            raise ValueError("DecodeGraph: the cache is full")
        self.ids.copy_(ids.reshape(-1, 1))
        self.graph.replay()
        for st in self.states:
            st.length += 1
        return self.logits

    def close(self) -> None:
        for st in self.states:
            if getattr(st, "pos_dev", None) is self.pos_dev:
                st.pos_dev = None


def _eos_ids(eos_token_id) -> list[int]:
    """The end-of-sequence ids as a list (the accepted forms of src/sisa/generation.py:98-122): None gives
    none; an integer, a 0-d or 1-d integer tensor or array, or an iterable of integers gives its values.
    Booleans, strings, bytes, floating-point or 2-d arrays raise TypeError."""
    if eos_token_id is None:
        return []
    x = eos_token_id
    err = TypeError(f"eos_token_id must be an integer or an iterable of integers, got {x!r} ({type(x).__name__})")
    if isinstance(x, (bool, str, bytes)):
        raise err
    if isinstance(x, numbers.Integral):
        return [int(x)]
    dtype = getattr(x, "dtype", None)
    if dtype is not None:                               # a torch tensor or a numpy array
        floating = dtype.is_floating_point if torch.is_tensor(x) else dtype.kind not in "iu"
        if floating or x.ndim > 1:
            raise err
        return [int(v) for v in x.reshape(-1).tolist()]
    if not isinstance(x, Iterable):
        raise err
    ids = list(x)
    if any(isinstance(t, bool) or not isinstance(t, numbers.Integral) for t in ids):
        raise err
    return [int(t) for t in ids]


def _next_token(logits: Tensor, *, do_sample: bool, temperature: float, top_k: int | None,
                generator: torch.Generator | None) -> Tensor:
    """Greedy argmax, or a sample from softmax(logits / temperature) restricted to the ``top_k`` largest
    logits. The sample is drawn among the k candidates only (a softmax over k values instead of the
    vocabulary), so it follows the reference's distribution but not its random stream."""
    scores = logits.float()
    if not do_sample:
        return scores.argmax(dim=-1)
    scores = scores / temperature
    if top_k is not None and top_k < scores.shape[-1]:
        vals, idx = torch.topk(scores, top_k, dim=-1)
        pick = torch.multinomial(torch.softmax(vals, dim=-1), num_samples=1, generator=generator)
        return idx.gather(-1, pick).squeeze(-1)
    return torch.multinomial(torch.softmax(scores, dim=-1), num_samples=1, generator=generator).squeeze(-1)


def _check_generate_args(input_ids: Tensor, max_new_tokens: int, do_sample: bool, temperature: float,
                         top_k: int | None) -> None:
    """The argument errors of the reference's generate (ValueError, same messages)."""
    problems = [
        (max_new_tokens < 0, "max_new_tokens must be >= 0"),
        (do_sample and temperature <= 0, "temperature must be positive when do_sample=True"),
        (top_k is not None and top_k <= 0, "top_k must be a positive integer"),
        (input_ids.dim() not in (1, 2) or input_ids.shape[-1] == 0, "input_ids must be a non-empty (B, L) tensor"),
    ]
    for bad, msg in problems:
        if bad:
            raise ValueError(msg)


@torch.no_grad()
def generate(model: "SISAForCausalLM", input_ids: Tensor, max_new_tokens: int, temperature: float = 1.0,
             top_k: int | None = None, eos_token_id: int | Iterable[int] | Tensor | None = None,
             do_sample: bool = False, *, generator: torch.Generator | None = None,
             eos_check_every: int = 16, cuda_graph: bool = True) -> Tensor:
    """Generate continuations of ``input_ids`` (generation.py:139-191).

    Same results as the reference. The all-finished check reads the device only every
    ``eos_check_every`` steps; the tokens generated past the step where every row had finished are
    cut off afterwards, so the returned length is the reference's. With ``cuda_graph`` (default) and a
    model that :meth:`DecodeGraph.supported` accepts, the first decode step runs eagerly and the rest
    replay it as one CUDA graph.
    """
    _check_generate_args(input_ids, max_new_tokens, do_sample, temperature, top_k)
    squeeze = input_ids.dim() == 1
    if squeeze:
        input_ids = input_ids.unsqueeze(0)
    if max_new_tokens == 0:
        return input_ids.squeeze(0) if squeeze else input_ids
    eos = _eos_ids(eos_token_id)
    eos_t = torch.tensor(eos, device=input_ids.device, dtype=input_ids.dtype) if eos else None
    cache = SISACache(capacity=input_ids.shape[1] + max_new_tokens)
    logits = model(input_ids, cache=cache, logits_to_keep=1).logits[:, -1]
    pieces = [input_ids]
    done = torch.zeros(input_ids.shape[0], dtype=torch.bool, device=input_ids.device)
    all_done_at = []       # device flags: every row finished after step s
    use_graph = cuda_graph and max_new_tokens > 2 and DecodeGraph.supported(model, cache)
    out = _decode_loop(model, input_ids, max_new_tokens, logits, cache, pieces, done, all_done_at, eos_t,
                       do_sample, temperature, top_k, generator, eos_check_every, use_graph)
    if all_done_at:
        flags = torch.stack(all_done_at).cpu()
        hit = torch.nonzero(flags).flatten()
        if hit.numel():
            out = out[:, :input_ids.shape[1] + int(hit[0]) + 1]
    return out.squeeze(0) if squeeze else out


def _decode_loop(model, input_ids, max_new_tokens, logits, cache, pieces, done, all_done_at, eos_t, do_sample,
                 temperature, top_k, generator, eos_check_every, use_graph) -> Tensor:
    """The token loop of :func:`generate`; with ``use_graph`` the second and later steps replay a
    :class:`DecodeGraph` captured after the first, which runs eagerly on the graph's stream."""
    side = torch.cuda.Stream(input_ids.device) if use_graph else None
    graphs: list[DecodeGraph] = []
    try:
        _token_steps(model, input_ids, max_new_tokens, logits, cache, pieces, done, all_done_at, eos_t, do_sample,
                     temperature, top_k, generator, eos_check_every, side, graphs)
    finally:
        for graph in graphs:
            graph.close()
    return torch.cat(pieces, dim=1)


def _token_steps(model, input_ids, max_new_tokens, logits, cache, pieces, done, all_done_at, eos_t, do_sample,
                 temperature, top_k, generator, eos_check_every, side, graphs) -> None:
    graph = None
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
        if graph is not None:
            logits = graph.step(nxt)
        elif side is not None:
            # eager step on the capture stream (libraries set up their per-stream state), then capture
            cur = torch.cuda.current_stream(input_ids.device)
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                logits = model(nxt.unsqueeze(1), cache=cache, logits_to_keep=1).logits[:, -1]
            cur.wait_stream(side)
            logits.record_stream(cur)
            if max_new_tokens - step > 2:
                graph = DecodeGraph(model, cache, input_ids.shape[0], stream=side)
                graphs.append(graph)
            side = None
        else:
            logits = model(nxt.unsqueeze(1), cache=cache, logits_to_keep=1).logits[:, -1]
