"""Shared forward of the ESA backend layers on the B200 kernels.

Math of the reference layers (ThunderESA.forward, esa/backends/thunder.py:
264-316; PulseESA.forward, esa/backends/pulse.py:69-98; FlareESA.forward,
esa/backends/flare.py:198-225):

    qgv = x W_qgv^T;  q, g, v = split(qgv)
    A = gmin + (gmax - gmin) sigmoid(g);  B = (1 - A) tanh(v)      -- fused into the scan
    E = scan(A.to(scan_dtype), B.to(scan_dtype))                  -- kernel a (+ b backward)
    y = out_proj( (sigmoid(q) * E * rsqrt(mean_C(E^2) + eps)).to(x.dtype) )

Everything between the qgv projection and out_proj is one op
(``esa_b200::layer_core``): the gated scan with the gate prologue fused, then
the fused readout kernel; its backward is the fused readout backward (which
writes the q third of d qgv and dE) and the gated reverse scan with the gate
chain rule (which writes the g and v thirds), so neither A, B nor the readout
intermediates are materialised and d qgv needs no concatenation.  Under
autocast the readout writes y directly in the autocast dtype that out_proj
would cast it to (the same value: rounding the fp32 result once).
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
    """sigmoid(q) * E * rsqrt(mean(E^2) + eps) over the channel axis, cast to
    out_dtype (thunder.py:304-311, generation.py:270-293).  Without autograd:
    the fused readout kernel (fp32 arithmetic, one rounding); when a gradient
    is needed: the same math in torch ops, in E's dtype."""
    if (not torch.is_grad_enabled() or not (q.requires_grad or E.requires_grad)) and q.is_cuda \
            and E.is_cuda and q.dim() == E.dim() == 3:
        return ops.readout(q, E, eps, out_dtype)
    q = q.to(E.dtype)
    E = E * torch.rsqrt(E.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (torch.sigmoid(q) * E).to(out_dtype)


def gated_layer_forward(layer, x: torch.Tensor, scan_dtype: torch.dtype | None, compass: int,
                        who: str) -> torch.Tensor:
    """scan_dtype None: scan in the dtype of the qgv projection (Flare)."""
    require_cuda_input(x, who)
    B, T, C = x.shape
    qgv = layer.qgv(x)
    if scan_dtype is None:
        scan_dtype = qgv.dtype
    out_dtype = x.dtype
    if torch.is_autocast_enabled("cuda"):
        out_dtype = torch.get_autocast_dtype("cuda")
    y, _, _ = ops.layer_core(qgv, float(layer.gate_min), float(layer.gate_max), float(layer.eps),
                             int(compass), scan_dtype, out_dtype)
    return layer.dropout(layer.out_proj(y))
