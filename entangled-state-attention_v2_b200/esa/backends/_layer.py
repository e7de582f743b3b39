"""Shared forward of the ESA backend layers on the B200 kernels.

Math of the reference layers (ThunderESA.forward, esa/backends/thunder.py:
264-316; PulseESA.forward, esa/backends/pulse.py:69-98; FlareESA.forward,
esa/backends/flare.py:198-225):

    qgv = x W_qgv^T;  q, g, v = split(qgv)
    A = gmin + (gmax - gmin) sigmoid(g);  B = (1 - A) tanh(v)      -- fused into the scan
    E = scan(A.to(scan_dtype), B.to(scan_dtype))                  -- kernel a (+ b backward)
    y = out_proj( (sigmoid(q) * E * rsqrt(mean_C(E^2) + eps)).to(x.dtype) )

The gate prologue and its chain rule run inside the scan kernels
(``esa_b200::gated_scan``), so A and B are never materialised in HBM.
"""

from __future__ import annotations

import torch

from .. import ops


def require_cuda_input(x: torch.Tensor, who: str) -> None:
    if not x.is_cuda:
        raise RuntimeError(
            f"{who}: this ESA build runs on CUDA (sm_100a) only and has no CPU fallback; "
            f"move the layer and input to a CUDA device (got {x.device})."
        )


def readout(q: torch.Tensor, E: torch.Tensor, eps: float, out_dtype: torch.dtype) -> torch.Tensor:
    """sigmoid(q) * E * rsqrt(mean(E^2) + eps) over the channel axis, in E's
    dtype, cast to out_dtype (thunder.py:304-311, generation.py:270-293)."""
    q = q.to(E.dtype)
    E = E * torch.rsqrt(E.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (torch.sigmoid(q) * E).to(out_dtype)


def gated_layer_forward(layer, x: torch.Tensor, scan_dtype: torch.dtype | None, compass: int,
                        who: str) -> torch.Tensor:
    """scan_dtype None: scan in the dtype of the qgv projection (Flare)."""
    require_cuda_input(x, who)
    B, T, C = x.shape
    qgv = layer.qgv(x)
    q, gate_raw, value_raw = qgv.split(C, dim=-1)
    if scan_dtype is None:
        scan_dtype = qgv.dtype
    E, _ = ops.gated_scan(gate_raw, value_raw, None, float(layer.gate_min),
                          float(layer.gate_max), int(compass), scan_dtype)
    y = readout(q, E, float(layer.eps), x.dtype)
    return layer.dropout(layer.out_proj(y))
