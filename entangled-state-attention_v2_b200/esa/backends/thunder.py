"""Thunder backend on the B200 kernels.

``thunder_scan`` keeps the reference signature and errors
(esa/backends/thunder.py:70-159): ``thunder_scan(A, B_write, compass=16, c=None)``
over contiguous [B, T, H, D] tensors, differentiable in A and B.  It runs the
single-pass chunked scan kernel (``esa_scan_fwd`` / ``esa_scan_rev``); ``compass``
picks the kernel's time tile and does not change results beyond fp32 summation
order.  ``ThunderESA`` keeps the reference constructor, attribute names and
state_dict keys (``qgv``, ``out_proj``, ``dropout``) so reference checkpoints load.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from .. import ops
from ..precision import resolve_scan_dtype
from ._layer import gated_layer_forward


def _check_scan_args(A: torch.Tensor, B_write: torch.Tensor) -> None:
    if A.shape != B_write.shape:
        raise ValueError(f"A and B_write must have same shape, got {A.shape} and {B_write.shape}")
    if A.dim() != 4:
        raise ValueError(f"expected A/B_write shape [B,T,H,D], got {A.shape}")


def _check_compass(compass) -> None:
    if not isinstance(compass, int) or isinstance(compass, bool) or compass <= 0:
        raise ValueError(f"compass must be a positive integer, got {compass!r}")


def thunder_scan(A: torch.Tensor, B_write: torch.Tensor, compass: int = 16,
                 c: int | None = None) -> torch.Tensor:
    """E_t = A_t * E_{t-1} + B_t over [B, T, H, D] (zero initial state)."""
    if c is not None:
        compass = c
    _check_scan_args(A, B_write)
    _check_compass(compass)
    if A.dtype != B_write.dtype:
        B_write = B_write.to(A.dtype)
    E, _ = ops.scan(A, B_write, None, int(compass))
    return E


class ThunderESA(nn.Module):
    """Thunder backend layer: reference constructor (thunder.py:186-261)."""

    def __init__(self, embd: int | None = None, head: int = 4, n_embd: int | None = None,
                 n_head: int | None = None, dropout: float = 0.0, compass: int = 16,
                 c: int | None = None, precision: str = "fp16", gate_min: float = 0.80,
                 gate_max: float = 0.995, eps: float = 1e-5, strict_precision: bool = False):
        super().__init__()
        if embd is None:
            embd = n_embd
        if n_head is not None:
            head = n_head
        if c is not None:
            compass = c
        if embd is None:
            raise ValueError("ThunderESA requires embd. Example: ThunderESA(embd=128, head=4)")
        if embd % head != 0:
            raise ValueError(f"embd must be divisible by head, got embd={embd}, head={head}")
        _check_compass(compass)
        self.embd = embd
        self.head = head
        self.head_dim = embd // head
        self.compass = compass
        self.n_embd = embd
        self.n_head = head
        self.c = compass
        self.precision = precision
        self.gate_min = gate_min
        self.gate_max = gate_max
        self.eps = eps
        self.strict_precision = strict_precision
        self.qgv = nn.Linear(embd, 3 * embd, bias=False)
        self.out_proj = nn.Linear(embd, embd, bias=False)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() != 3:
            raise ValueError(f"expected input shape [B,T,C], got {x.shape}")
        if x.shape[-1] != self.embd:
            raise ValueError(f"expected embedding dim {self.embd}, got input dim {x.shape[-1]}")
        scan_dtype = resolve_scan_dtype(self.precision, x.device,
                                        strict_precision=self.strict_precision)
        return gated_layer_forward(self, x, scan_dtype, self.compass, "ThunderESA")
