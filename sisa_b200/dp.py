"""Data-parallel training step of the SISA decoder (one process per GPU, NCCL gradient allreduce).

The reference has no distributed code (its README calls DDP untested); its training loop is
examples/train_minimal.py:253-301: fp32 master weights, bf16 autocast, fused AdamW with the model's
parameter groups (betas 0.9/0.95), gradient clipping at 1.0, chunked linear-CE loss. This module runs
that step data-parallel: every rank holds a replica, processes its own batch, and the gradients are
averaged across ranks; the optimizer stays replicated. Two forms:

* DDP (eager): bucketed NCCL allreduces overlap the backward pass (buckets are views of the
  gradients, so no extra copy).
* Flat gradients (``Trainer(cuda_graph=True)`` on several GPUs, or ``flat_grads=True``): every
  parameter's gradient is a view of one fp32 buffer, laid out in the order the backward produces
  them and cut into buckets, and the loss is scaled by 1/world (exact for world sizes that are powers
  of two). As the backward finishes a bucket, a SUM allreduce of it starts on a side stream, so the
  allreduces overlap the rest of the backward; buckets start strictly in bucket order, which keeps the
  collective order identical on every rank. On CUDA the whole step, allreduces included, is captured
  as one CUDA graph and replayed, as on one GPU.
"""
from __future__ import annotations

import datetime
import os
import warnings

import torch
import torch.distributed as dist

from .config import SISAConfig
from .modeling import SISAForCausalLM

__all__ = ["init_distributed", "build_model", "make_optimizer", "Trainer"]


def init_distributed(backend: str | None = None, timeout_s: float = 120.0) -> tuple[int, int, torch.device]:
    """Join the process group described by RANK / WORLD_SIZE / LOCAL_RANK / MASTER_* (torchrun).

    Returns (rank, world_size, device). Single process (no WORLD_SIZE) returns (0, 1, cuda:0 or cpu).
    """
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    use_cuda = torch.cuda.is_available() and backend != "gloo"
    dev = torch.device("cuda", local) if use_cuda else torch.device("cpu")
    if world <= 1:
        return 0, 1, dev
    if use_cuda:
        torch.cuda.set_device(dev)
    if not dist.is_initialized():
        dist.init_process_group(backend or ("nccl" if use_cuda else "gloo"),
                                timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=dev if use_cuda else None)
    return dist.get_rank(), dist.get_world_size(), dev


def build_model(config: SISAConfig, device: torch.device, seed: int = 0) -> SISAForCausalLM:
    """Reference initialisation (SISAConfig init fields) with the same seed on every rank; fp32 master weights."""
    torch.manual_seed(seed)
    return SISAForCausalLM(config).to(device)


def make_optimizer(model: SISAForCausalLM, lr: float = 6e-4, weight_decay: float = 0.1,
                   capturable: bool = False) -> torch.optim.Optimizer:
    """AdamW over the model's parameter groups (train_minimal.py:253-260). ``capturable`` keeps the step
    counters on the device so that the step can be captured in a CUDA graph."""
    cuda = next(model.parameters()).is_cuda
    return torch.optim.AdamW(model.param_groups(lr, weight_decay=weight_decay), lr=lr, betas=(0.9, 0.95),
                             weight_decay=weight_decay, fused=cuda, capturable=capturable and cuda)


class GradBuckets:
    """Flat fp32 gradients, allreduced bucket by bucket as the backward finishes them.

    Every trainable parameter's gradient is a view of one fp32 buffer. The buffer holds the
    parameters in reverse registration order, which is about the order the backward finishes them
    (last block first), and is cut at parameter boundaries into buckets of about ``cap_mb``. A
    post-accumulate-grad hook counts the finished parameters of each bucket. A bucket starts once it
    and every bucket before it are complete, so all ranks issue the same allreduces in the same order
    whatever order the hooks fire in. On CUDA each allreduce runs on a side stream that first waits for
    the stream the backward ran on; :meth:`finish` starts any bucket still pending (parameters that
    received no gradient this step) and makes the caller's stream wait for the side stream. Under CUDA
    graph capture the waits become graph dependencies, so a replay overlaps the allreduces with the
    backward in the same way.
    """

    def __init__(self, params: list[torch.nn.Parameter], device: torch.device, cap_mb: float = 40.0,
                 reduce: bool = True):
        self.device = device
        self.reduce = reduce
        order = list(reversed(params))
        self.order = order
        # each parameter at an offset of whole 16-byte units (the flat optimizer's float4 chunks)
        size = lambda p: -(-p.numel() // 4) * 4                       # noqa: E731
        self.buffer = torch.zeros(sum(size(p) for p in order), dtype=torch.float32, device=device)
        cap = max(1, int(cap_mb * 2**20 / 4))
        self.bounds: list[tuple[int, int]] = []       # [start, end) of each bucket in the buffer
        self.offset: dict[int, tuple[int, int]] = {}  # id(p) -> (offset, numel)
        self._bucket_of: dict[int, int] = {}
        off, start = 0, 0
        for p in order:
            p.grad = self.buffer[off:off + p.numel()].view_as(p)
            self.offset[id(p)] = (off, p.numel())
            if off > start and off + size(p) - start > cap:
                self.bounds.append((start, off))
                start = off
            self._bucket_of[id(p)] = len(self.bounds)
            off += size(p)
        self.bounds.append((start, off))
        self._size = [0] * len(self.bounds)
        for p in order:
            self._size[self._bucket_of[id(p)]] += 1
        self._left: list[int] = []
        self._next = 0
        self.side = torch.cuda.Stream(device) if (device.type == "cuda" and reduce) else None
        self._hooks = [p.register_post_accumulate_grad_hook(self._on_grad) for p in order] if reduce else []

    def __len__(self) -> int:
        return len(self.bounds)

    def start_step(self) -> None:
        """Zero the gradients and rearm the bucket counters (call before the backward)."""
        self.buffer.zero_()
        self._left = list(self._size) if self.reduce else []
        self._next = 0

    def _on_grad(self, p: torch.Tensor) -> None:
        if not self._left:
            return                                   # a backward outside a step (no allreduce wanted)
        k = self._bucket_of[id(p)]
        self._left[k] -= 1
        while self._next < len(self.bounds) and self._left[self._next] == 0:
            self._launch(self._next)
            self._next += 1

    def _launch(self, k: int) -> None:
        a, b = self.bounds[k]
        view = self.buffer[a:b]
        if self.side is None:
            dist.all_reduce(view, op=dist.ReduceOp.SUM)
            return
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(self.device))
        self.side.wait_event(ready)
        with torch.cuda.stream(self.side):
            dist.all_reduce(view, op=dist.ReduceOp.SUM)

    def finish(self) -> None:
        """Start the buckets still pending and order the caller's stream after every allreduce."""
        if not self.reduce:
            return
        while self._next < len(self.bounds):
            self._launch(self._next)
            self._next += 1
        self._left = []
        if self.side is not None:
            torch.cuda.current_stream(self.device).wait_stream(self.side)

    def remove(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks = []


class Trainer:
    """One optimizer step per call: forward (bf16 autocast on CUDA), loss, backward, gradient allreduce,
    clipping, AdamW.

    With ``cuda_graph=True`` (CUDA; on several GPUs with flat gradients and the allreduce inside) the
    whole step (forward, backward, clipping and the
    optimizer) is captured once as a CUDA graph and replayed from a static input buffer, which removes
    the launch gaps of its several hundred kernels and the host's dispatch work. The first call runs
    eagerly (it also creates the optimizer state, which a capture must not allocate); the second
    captures and replays; every call is exactly one optimizer step. A new input shape captures again.

    ``flat_optimizer=True`` (CUDA, fp32 parameters, no optimizer given) runs clipping and AdamW as the
    flat kernels of :class:`sisa_b200.optim.FlatAdamW` over the gradients' flat layout; by default the
    step uses ``torch.optim.AdamW`` (fused) and ``clip_grad_norm_``.
    """

    def __init__(self, model: SISAForCausalLM, optimizer: torch.optim.Optimizer | None = None, *,
                 fused_ce: bool = True, clip: float = 1.0, bucket_cap_mb: float = 40.0, cuda_graph: bool = False,
                 flat_grads: bool = False, flat_optimizer: bool | None = None, tensor_optimizer: bool = True):
        self.module = model
        self._params = list(model.parameters())
        dev = next(model.parameters()).device
        self.device = dev
        self.distributed = dist.is_initialized() and dist.get_world_size() > 1
        self.world = dist.get_world_size() if self.distributed else 1
        self.cuda_graph = cuda_graph and dev.type == "cuda"
        trainable = [p for p in model.parameters() if p.requires_grad]
        flat_dp = self.distributed and (self.cuda_graph or flat_grads)
        # The flat AdamW kernels (sisa_b200.optim) are opt-in: they need the gradients as views of one
        # buffer, and on one GPU autograd then adds every gradient into its slot instead of handing over
        # the fresh tensor, which costs about what the kernels save (measured: 29.1 vs 28.4-28.8 ms per
        # cfg3 step); in the data-parallel flat form they measured no gain either (31.34 vs 31.37 ms).
        self.flat_opt = bool(flat_optimizer) and optimizer is None and dev.type == "cuda" and \
            all(p.dtype == torch.float32 for p in trainable)
        self.flat = flat_dp or self.flat_opt
        # Otherwise the same kernels over the parameter tensors as they are (sisa_b200.optim.TensorAdamW):
        # clipping and AdamW in two launches instead of torch's fused AdamW plus clip_grad_norm_.
        from .optim import TensorAdamW

        self.list_opt = (tensor_optimizer and optimizer is None and not self.flat and dev.type == "cuda"
                         and all(p.dtype == torch.float32 for p in trainable)
                         and len(trainable) <= TensorAdamW.MAX_TENSORS)
        self._buckets: GradBuckets | None = None
        if self.flat:
            self.model = model
            self._make_flat_grads(bucket_cap_mb)
        elif self.distributed:
            self.model = torch.nn.parallel.DistributedDataParallel(
                model, device_ids=[dev.index] if dev.type == "cuda" else None, gradient_as_bucket_view=True,
                bucket_cap_mb=bucket_cap_mb, broadcast_buffers=False)
        else:
            self.model = model
        if self.flat_opt:
            from .optim import FlatAdamW

            self.opt = FlatAdamW(model.param_groups(6e-4, weight_decay=0.1), self._buckets, betas=(0.9, 0.95),
                                 max_norm=clip)
        elif self.list_opt:
            self.opt = TensorAdamW(model.param_groups(6e-4, weight_decay=0.1), betas=(0.9, 0.95), max_norm=clip)
        else:
            self.opt = optimizer or make_optimizer(model, capturable=self.cuda_graph)
        self.fused_ce = fused_ce and dev.type == "cuda"
        self.clip = clip
        self._graph = None
        self._static_ids = None
        self._static_loss = None

    def _make_flat_grads(self, cap_mb: float) -> None:
        """Rank 0's parameters on every rank, and every gradient a view of one bucketed fp32 buffer
        (autograd accumulates into existing gradients in place, so the views persist across steps)."""
        params = [p for p in self.module.parameters() if p.requires_grad]
        if any(p.dtype != torch.float32 for p in params):
            raise TypeError("flat gradients need fp32 parameters (the master weights)")
        if self.distributed:
            with torch.no_grad():
                for p in params:
                    dist.broadcast(p.data, 0)
        self._buckets = GradBuckets(params, self.device, cap_mb, reduce=self.distributed)

    def close(self) -> None:
        """Release the captured step. A graph that holds NCCL work must be released before
        ``destroy_process_group``; later calls to :meth:`step` capture again."""
        if self._graph is not None:
            torch.cuda.synchronize(self.device)
            self._graph.reset()
            self._graph = None
            self._static_ids = None

    def step(self, ids: torch.Tensor) -> torch.Tensor:
        """Train on ``ids`` (B, T) (labels = ids, shifted inside the model). Returns the loss (device)."""
        if self.cuda_graph:
            return self._graphed_step(ids)
        return self._eager_step(ids)

    def _graphed_step(self, ids: torch.Tensor) -> torch.Tensor:
        if self._static_ids is None or self._static_ids.shape != ids.shape:
            self._graph = None                       # first call for this shape: eager, capture on the next
            self._static_ids = ids.detach().clone()
            return self._eager_step(ids)
        if self._graph is None:
            self._capture()
            if self._graph is None:                  # a rank could not capture: eager steps from here on
                return self._eager_step(ids)
        self._static_ids.copy_(ids, non_blocking=True)
        self._graph.replay()
        self._mark_updated()
        return self._static_loss.clone()

    def _capture(self) -> None:
        if not self.flat:
            self.opt.zero_grad(set_to_none=True)     # the captured backward allocates the gradients
        graph = torch.cuda.CUDAGraph()
        ok = True
        try:
            # thread_local with NCCL: its watchdog thread may query events while this thread captures
            with torch.cuda.graph(graph, capture_error_mode="thread_local" if self.distributed else "global"):
                self._static_loss = self._forward_backward(self._static_ids)
                self._update()
        except Exception:
            ok = False
            if not self.distributed:
                raise
        if self.distributed:
            # every rank replays only if every rank captured (a lone replay would wait in its allreduce);
            # otherwise all ranks continue with eager steps of the same form
            flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=self.device)
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
            if int(flag.item()) == 0:
                warnings.warn("Trainer: CUDA graph capture of the data-parallel step failed on a rank; "
                              "continuing with eager steps", RuntimeWarning)
                self.cuda_graph = False
                self._graph = None
                return
        self._graph = graph

    def _mark_updated(self) -> None:
        """Advance the parameters' version counters after an update: the fused optimizers (and a graph
        replay) change the weights in place without doing so, and the compute-dtype weight copies kept
        for inference are keyed on them."""
        torch.autograd.graph.increment_version(self._params)

    def _update(self) -> None:
        """Clipping and the optimizer step (in the flat form the allreduces have run during the backward;
        the flat AdamW clips inside its kernels)."""
        if self.flat_opt or self.list_opt:
            self.opt.step()                          # clips inside its kernels
        else:
            if self.clip:
                torch.nn.utils.clip_grad_norm_(self.module.parameters(), self.clip)
            self.opt.step()
        self._mark_updated()

    def _loss(self, ids: torch.Tensor) -> torch.Tensor:
        if self.device.type == "cuda":
            with torch.autocast("cuda", dtype=torch.bfloat16):
                return self.model(ids, labels=ids, fused_ce=self.fused_ce).loss
        return self.model(ids, labels=ids).loss

    def _forward_backward(self, ids: torch.Tensor) -> torch.Tensor:
        self.model.train()
        if self.flat:
            self._buckets.start_step()
        loss = self._loss(ids)
        (loss * (1.0 / self.world) if self.flat else loss).backward()
        if self.flat:
            self._buckets.finish()
        return loss.detach()

    def _eager_step(self, ids: torch.Tensor) -> torch.Tensor:
        loss = self._forward_backward(ids)
        self._update()
        if not self.flat:
            self.opt.zero_grad(set_to_none=True)
        return loss
