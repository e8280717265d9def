"""Test helpers (tolerances stated once, reused by every parity test)."""
from __future__ import annotations

import torch

# Tolerances of the bf16 path against the fp64 oracle:
OUT_MAX_ABS = 2e-2        # max |o - o_ref| over every output element
GRAD_REL = 5e-2           # ||dx - dx_ref|| / ||dx_ref|| per gradient tensor
PREP_SCAN_REL = 1e-5      # fp32 scans g, F, Phi vs fp64


def rel_err(x: torch.Tensor, ref: torch.Tensor) -> float:
    x, ref = x.detach().double().cpu(), ref.detach().double().cpu()
    return float((x - ref).norm() / ref.norm().clamp_min(1e-300))


def max_abs(x: torch.Tensor, ref: torch.Tensor) -> float:
    return float((x.detach().double().cpu() - ref.detach().double().cpu()).abs().max())
