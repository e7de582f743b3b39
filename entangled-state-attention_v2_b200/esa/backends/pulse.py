"""Pulse backend on the B200 kernels.

``pulse_scan`` keeps the reference signature and errors (esa/backends/pulse.py:
12-31).  The reference evaluates the recurrence with a Python loop over T; here
the same exact recurrence runs in the chunked scan kernel, which reproduces the
sequential result up to fp32 summation order.  ``PulseESA`` keeps the reference
constructor (pulse.py:41-67), including its eps default of 1e-6.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .. import ops
from ..precision import resolve_scan_dtype
from ._layer import gated_layer_forward
from .thunder import _check_scan_args


def pulse_scan(A: torch.Tensor, B_write: torch.Tensor) -> torch.Tensor:
    """E_t = A_t * E_{t-1} + B_t over [B, T, H, D] (zero initial state)."""
    _check_scan_args(A, B_write)
    if A.dtype != B_write.dtype:
        B_write = B_write.to(A.dtype)
    E, _ = ops.scan(A, B_write, None, 16)
    return E


class PulseESA(nn.Module):
    """Pulse backend layer (reference pulse.py:34-98)."""

    def __init__(self, n_embd: int, n_head: int = 4, dropout: float = 0.0, precision: str = "fp16",
                 gate_min: float = 0.80, gate_max: float = 0.995, eps: float = 1e-6,
                 strict_precision: bool = False):
        super().__init__()
        if n_embd % n_head != 0:
            raise ValueError("n_embd must be divisible by n_head")
        self.n_embd = n_embd
        self.n_head = n_head
        self.head_dim = n_embd // n_head
        self.precision = precision
        self.gate_min = gate_min
        self.gate_max = gate_max
        self.eps = eps
        self.strict_precision = strict_precision
        self.qgv = nn.Linear(n_embd, 3 * n_embd, bias=False)
        self.out_proj = nn.Linear(n_embd, n_embd, bias=False)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        scan_dtype = resolve_scan_dtype(self.precision, x.device,
                                        strict_precision=self.strict_precision)
        return gated_layer_forward(self, x, scan_dtype, 16, "PulseESA")
