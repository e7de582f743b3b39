"""Scan dtype policy: the precision string -> dtype table of the reference
(esa/precision.py:12-64), kept identical because it decides the scan kernels'
storage type.

    fp16 -> float16 on CUDA (float32 on CPU unless strict_precision)
    bf16 -> bfloat16,  fp32 -> float32,  fp64 -> float64
    fp8  -> float16 on CUDA / float32 on CPU, with a RuntimeWarning
            (NotImplementedError when strict_precision)
"""

from __future__ import annotations

import warnings

import torch

from .constants import SUPPORTED_PRECISIONS

_FP8_MSG = (
    "precision='fp8' is experimental in ESA v2. The current safe implementation uses fp16 "
    "scan accumulation. A true FP8 Flare/Thunder kernel can be added later."
)


def resolve_scan_dtype(precision: str, device, *, strict_precision: bool = False) -> torch.dtype:
    """Map a user precision string to the dtype the scan stores its state in."""
    p = str(precision).lower()
    if p not in SUPPORTED_PRECISIONS:
        raise ValueError(
            f"Unsupported precision={precision!r}. Expected one of {sorted(SUPPORTED_PRECISIONS)}."
        )
    on_cuda = torch.device(device).type == "cuda"
    if p == "fp16":
        return torch.float16 if (on_cuda or strict_precision) else torch.float32
    if p == "bf16":
        return torch.bfloat16
    if p == "fp32":
        return torch.float32
    if p == "fp64":
        return torch.float64
    # fp8
    if strict_precision:
        raise NotImplementedError(_FP8_MSG)
    warnings.warn(_FP8_MSG, RuntimeWarning, stacklevel=2)
    return torch.float16 if on_cuda else torch.float32
