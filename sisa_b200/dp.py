"""Data-parallel training step of the SISA decoder (one process per GPU, NCCL gradient allreduce).

The reference has no distributed code (its README calls DDP untested); its training loop is
examples/train_minimal.py:253-301: fp32 master weights, bf16 autocast, fused AdamW with the model's
parameter groups (betas 0.9/0.95), gradient clipping at 1.0, chunked linear-CE loss. This module runs
that step data-parallel: every rank holds a replica, processes its own batch, and DDP averages the
gradients with bucketed NCCL allreduces that overlap the backward pass (buckets are views of the
gradients, so no extra copy). The optimizer stays replicated.
"""
from __future__ import annotations

import datetime
import os

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


class Trainer:
    """One optimizer step per call: forward (bf16 autocast on CUDA), loss, backward with overlapped
    gradient allreduce, clipping, AdamW.

    With ``cuda_graph=True`` (one process, CUDA) the whole step (forward, backward, clipping and the
    optimizer) is captured once as a CUDA graph and replayed from a static input buffer, which removes
    the launch gaps of its several hundred kernels and the host's dispatch work. The first call runs
    eagerly (it also creates the optimizer state, which a capture must not allocate); the second
    captures and replays; every call is exactly one optimizer step. A new input shape captures again.
    """

    def __init__(self, model: SISAForCausalLM, optimizer: torch.optim.Optimizer | None = None, *,
                 fused_ce: bool = True, clip: float = 1.0, bucket_cap_mb: float = 64.0, cuda_graph: bool = False):
        self.module = model
        dev = next(model.parameters()).device
        self.device = dev
        self.distributed = dist.is_initialized() and dist.get_world_size() > 1
        if self.distributed:
            self.model = torch.nn.parallel.DistributedDataParallel(
                model, device_ids=[dev.index] if dev.type == "cuda" else None, gradient_as_bucket_view=True,
                bucket_cap_mb=bucket_cap_mb, broadcast_buffers=False)
        else:
            self.model = model
        self.cuda_graph = cuda_graph and dev.type == "cuda" and not self.distributed
        self.opt = optimizer or make_optimizer(model, capturable=self.cuda_graph)
        self.fused_ce = fused_ce and dev.type == "cuda"
        self.clip = clip
        self._graph = None
        self._static_ids = None
        self._static_loss = None

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
        self._static_ids.copy_(ids, non_blocking=True)
        self._graph.replay()
        return self._static_loss.clone()

    def _capture(self) -> None:
        self.opt.zero_grad(set_to_none=True)         # the captured backward allocates the gradients
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._static_loss = self._forward_backward(self._static_ids)
            if self.clip:
                torch.nn.utils.clip_grad_norm_(self.module.parameters(), self.clip)
            self.opt.step()
        self._graph = graph

    def _forward_backward(self, ids: torch.Tensor) -> torch.Tensor:
        self.model.train()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = self.model(ids, labels=ids, fused_ce=self.fused_ce).loss
        loss.backward()
        return loss.detach()

    def _eager_step(self, ids: torch.Tensor) -> torch.Tensor:
        self.model.train()
        if self.device.type == "cuda":
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = self.model(ids, labels=ids, fused_ce=self.fused_ce).loss
        else:
            loss = self.model(ids, labels=ids).loss
        loss.backward()
        if self.clip:
            torch.nn.utils.clip_grad_norm_(self.module.parameters(), self.clip)
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return loss.detach()
