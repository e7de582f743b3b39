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


def thunder_scan_host(A: torch.Tensor, B_write: torch.Tensor, compass: int = 16,
                      c: int | None = None, *, out: torch.Tensor | None = None,
                      device: torch.device | int | None = None) -> torch.Tensor:
    """thunder_scan of CPU tensors, computed on a GPU: the result is a CPU tensor.

    A and B_write stay in host memory; the library streams them through the
    device in chunks, overlapping the host-to-device copies, the scans and the
    device-to-host copies (``esa_scan_fwd_host``).  Page-locked inputs and
    ``out`` (``tensor.pin_memory()``) let the copies run asynchronously;
    pageable memory works at a lower rate.  Returns when E is complete.  No
    autograd (the reference's CPU thunder_scan is differentiable; use
    thunder_scan on device tensors for training).
    """
    from .. import _lib

    if c is not None:
        compass = c
    _check_scan_args(A, B_write)
    _check_compass(compass)
    if A.device.type != "cpu" or B_write.device.type != "cpu":
        raise ValueError("thunder_scan_host takes CPU tensors; use thunder_scan for device tensors")
    if not torch.cuda.is_available():
        raise RuntimeError("thunder_scan_host needs a CUDA device (no CPU fallback)")
    if A.dtype != B_write.dtype:
        B_write = B_write.to(A.dtype)
    A = A.contiguous()
    B_write = B_write.contiguous()
    if out is None:
        out = torch.empty(A.shape, dtype=A.dtype, pin_memory=A.is_pinned())
    elif out.shape != A.shape or out.dtype != A.dtype or not out.is_contiguous() or out.device.type != "cpu":
        raise ValueError("out must be a contiguous CPU tensor of A's shape and dtype")
    if device is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    else:
        dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
    nb, T, H, D = A.shape
    code = ops.dtype_code(A.dtype)
    L = _lib.lib()
    nbytes = int(L.esa_scan_host_staging_bytes(nb, T, H * D, code, int(compass)))
    with torch.cuda.device(dev):
        staging = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream(dev)
        _lib.check(L.esa_scan_fwd_host(A.data_ptr(), B_write.data_ptr(), out.data_ptr(), nb, T, H * D,
                                       code, int(compass), staging.data_ptr(), nbytes,
                                       stream.cuda_stream), "esa_scan_fwd_host")
        stream.synchronize()
        ops.check_device_status(dev)
        del staging
    return out


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
