"""Flare backend on the B200 kernels (no Triton).

The reference's Flare backend (esa/backends/flare.py:9-225) runs two Triton
kernels: a per-channel sequential scan with an fp32 state, output stored in
the input dtype, and its reverse-time backward.  Here ``flare_scan`` keeps that
signature and semantics (fp32 accumulation, output in the input dtype,
``block_ch`` accepted for compatibility) on the chunked scan kernels, and
``FlareESA`` scans in the activations' dtype as the reference does (its state
dtype is the input dtype, generation.py:382-383).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .. import ops
from ._layer import gated_layer_forward, require_cuda_input
from .thunder import _check_scan_args

TRITON_AVAILABLE = True  # kept for API compatibility: this backend needs no Triton
TRITON_ERROR = None


def flare_scan(A: torch.Tensor, B_write: torch.Tensor, *, block_ch: int = 128) -> torch.Tensor:
    """E_t = A_t * E_{t-1} + B_t, fp32 state, output in A's dtype."""
    _check_scan_args(A, B_write)
    require_cuda_input(A, "flare_scan")
    if A.dtype != B_write.dtype:
        B_write = B_write.to(A.dtype)
    E, _ = ops.scan(A, B_write, None, 16)
    return E


class FlareESA(nn.Module):
    """Flare backend layer (reference flare.py:151-225)."""

    def __init__(self, n_embd: int, n_head: int = 4, dropout: float = 0.0, precision: str = "fp16",
                 gate_min: float = 0.80, gate_max: float = 0.995, eps: float = 1e-6,
                 block_ch: int = 128, strict_precision: bool = False):
        super().__init__()
        if n_embd % n_head != 0:
            raise ValueError("n_embd must be divisible by n_head")
        if precision not in {"fp16", "bf16", "fp32", "fp64", "fp8"}:
            raise ValueError(f"Unsupported precision={precision!r}")
        if precision == "fp8" and strict_precision:
            raise NotImplementedError("True FP8 Flare scan is not implemented yet.")
        self.n_embd = n_embd
        self.n_head = n_head
        self.head_dim = n_embd // n_head
        self.precision = precision
        self.gate_min = gate_min
        self.gate_max = gate_max
        self.eps = eps
        self.block_ch = block_ch
        self.strict_precision = strict_precision
        self.qgv = nn.Linear(n_embd, 3 * n_embd, bias=False)
        self.out_proj = nn.Linear(n_embd, n_embd, bias=False)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("backend='flare' requires CUDA tensors.")
        return gated_layer_forward(self, x, None, 16, "FlareESA")
