# Copyright 2026 Zameer Hussain and Akhtar Hussain
# Licensed under the Apache License, Version 2.0.
# Portions of this file reproduce the public interface of esa/generation.py of
# Entangled-State-Attention v2.1.1 (signatures, dataclasses, validation and
# error messages), under that licence.

"""Prefill and ESA-Lightning decode on the B200 kernels.

Public surface of the reference's esa/generation.py (:15-560): GenerationStats,
GenerationResult, EngineSpec, parse_engine_spec, lightning_init_state,
esa_prefill (alias lightning_prefill), lightning_decode_step and
sample_next_token, with the same arguments, shapes, dtypes and errors.

Hot paths:
* ``esa_prefill`` runs the gated scan kernel (gate prologue fused, optional
  initial state).  The reference's exact-recurrence Python loop for
  ``backend="lightning"`` or an explicit ``state`` (generation.py:369-395)
  becomes the same kernel with that state as its initial value.
* ``lightning_decode_step`` runs the fused one-token kernel (gates, state
  update, RMS readout) between the qgv GEMV and the out_proj GEMV
  (generation.py:443-458).
"""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Any

import torch
import torch.nn.functional as F

from . import ops
from .backends._layer import readout as _readout_math
from .backends._layer import require_cuda_input
from .precision import resolve_scan_dtype


@dataclass(frozen=True)
class GenerationStats:
    prompt_tokens: int
    prefill_tokens: int
    generated_tokens: int
    decode_steps: int
    prefill_seconds: float
    decode_seconds: float
    decode_tok_s: float
    total_seconds: float
    state_bytes: int
    state_mb: float

    def to_dict(self) -> dict[str, Any]:
        """Return generation statistics as a JSON-serializable dictionary."""
        return asdict(self)


@dataclass
class GenerationResult:
    sequences: torch.Tensor
    generated_ids: torch.Tensor
    stats: GenerationStats
    text: str | list[str] | None = None


@dataclass(frozen=True)
class EngineSpec:
    """Parsed ESA execution-engine specification."""

    backend: str
    compiled: bool = False
    compass: int | None = None


def parse_engine_spec(value: str, *, default_thunder_compass: int = 16) -> EngineSpec:
    """Parse names such as ``thunder_compiled_16``, ``pulse`` or ``lightning``
    (grammar of generation.py:50-92)."""
    name = str(value).strip().lower().replace("-", "_")
    if not name:
        raise ValueError("Engine name must not be empty.")
    if name in {"lightning", "lightning_compiled"}:
        return EngineSpec(backend="lightning", compiled=name.endswith("_compiled"), compass=None)
    parts = [p for p in name.split("_") if p]
    backend = parts[0]
    if backend not in {"thunder", "flare", "pulse"}:
        raise ValueError(
            f"Unknown ESA engine {value!r}. Supported engines are lightning, thunder, flare, and pulse."
        )
    compiled = "compiled" in parts[1:]
    numeric = [int(p) for p in parts[1:] if p.isdigit()]
    if backend == "thunder":
        if len(numeric) > 1:
            raise ValueError(f"Thunder engine has multiple compass values: {value!r}")
        compass = numeric[0] if numeric else int(default_thunder_compass)
        if compass <= 0:
            raise ValueError(f"Thunder compass must be positive, got {compass}.")
    else:
        if numeric:
            raise ValueError(f"Compass values are only valid for Thunder engines, got {value!r}.")
        compass = None
    return EngineSpec(backend=backend, compiled=compiled, compass=compass)


def _unwrap_backend(module: torch.nn.Module) -> torch.nn.Module:
    current = getattr(module, "layer", module)
    seen: set[int] = set()
    while hasattr(current, "_orig_mod") and id(current) not in seen:
        seen.add(id(current))
        current = current._orig_mod
    return current


def _backend_name(module: torch.nn.Module) -> str:
    if hasattr(module, "backend"):
        return str(module.backend).lower()
    name = _unwrap_backend(module).__class__.__name__.lower()
    for cand in ("flare", "thunder", "pulse"):
        if cand in name:
            return cand
    return name


def _dimensions(module: torch.nn.Module) -> tuple[int, int, int]:
    backend = _unwrap_backend(module)
    embd = getattr(backend, "embd", None)
    head = getattr(backend, "head", None)
    head_dim = getattr(backend, "head_dim", None)
    if embd is None or head is None:
        raise AttributeError("ESA backend must expose embd and head.")
    embd, head = int(embd), int(head)
    if head_dim is None:
        head_dim = embd // head
    return embd, head, int(head_dim)


def _state_dtype(module: torch.nn.Module, device: torch.device, input_dtype: torch.dtype, *,
                 backend_name: str | None = None) -> torch.dtype:
    """Flare keeps the input dtype; the others follow resolve_scan_dtype
    (generation.py:372-403)."""
    backend = _unwrap_backend(module)
    name = (backend_name or _backend_name(module)).lower()
    if name == "flare":
        return input_dtype
    precision = str(getattr(backend, "precision", getattr(module, "precision", "fp16")))
    return resolve_scan_dtype(precision, device,
                              strict_precision=bool(getattr(backend, "strict_precision", False)))


def _project_logits(module: torch.nn.Module, x: torch.Tensor):
    """(q, gate_raw, value_raw) as [B, T, C] views of the qgv projection."""
    backend = _unwrap_backend(module)
    embd, _, _ = _dimensions(module)
    if x.ndim != 3 or x.size(-1) != embd:
        raise ValueError(f"Expected x [B,T,{embd}], got {tuple(x.shape)}")
    return backend.qgv(x).split(x.size(-1), dim=-1)


def _project_affine_terms(module: torch.nn.Module, x: torch.Tensor):
    """(q, A, B_write) as [B, T, H, D] (generation.py:180-221); kept for API
    parity -- the engine itself never materialises A and B."""
    _, head, head_dim = _dimensions(module)
    backend = _unwrap_backend(module)
    q, g, v = _project_logits(module, x)
    B, T, _ = x.shape
    shape = (B, T, head, head_dim)
    A = backend.gate_min + (backend.gate_max - backend.gate_min) * torch.sigmoid(g)
    Bw = (1.0 - A) * torch.tanh(v)
    return q.reshape(shape), A.reshape(shape), Bw.reshape(shape)


def _backend_scan(module: torch.nn.Module, A: torch.Tensor, B_write: torch.Tensor, *,
                  backend_override: str | None = None, compass_override: int | None = None):
    """Scan materialised A, B with the module's (or the overridden) backend
    (generation.py:224-268)."""
    backend = _unwrap_backend(module)
    name = (backend_override or _backend_name(module)).lower()
    if name not in {"thunder", "pulse", "flare"}:
        raise ValueError(f"Unsupported ESA backend for prefill: {name!r}")
    if name != "flare":
        dtype = _state_dtype(module, A.device, A.dtype, backend_name=name)
        A, B_write = A.to(dtype), B_write.to(dtype)
    compass = (int(compass_override) if compass_override is not None
               else int(getattr(backend, "compass", 16) or 16)) if name == "thunder" else 16
    E, _ = ops.scan(A.contiguous(), B_write.contiguous(), None, compass)
    return E


def _readout(module: torch.nn.Module, q: torch.Tensor, states: torch.Tensor, *,
             output_dtype: torch.dtype) -> torch.Tensor:
    """out_proj(sigmoid(q) * E * rsqrt(mean(E^2) + eps)) over all C channels."""
    backend = _unwrap_backend(module)
    B, T = states.shape[0], states.shape[1]
    C = states[0, 0].numel()
    z = _readout_math(q.reshape(B, T, C), states.reshape(B, T, C), float(backend.eps), output_dtype)
    return backend.dropout(backend.out_proj(z))


def lightning_init_state(module: torch.nn.Module, batch: int, *, device=None, dtype=None,
                         layout: str = "heads") -> torch.Tensor:
    backend = _unwrap_backend(module)
    embd, head, head_dim = _dimensions(module)
    if device is None:
        device = backend.qgv.weight.device
    device = torch.device(device)
    if dtype is None:
        dtype = _state_dtype(module, device, backend.qgv.weight.dtype)
    if layout == "heads":
        shape = (batch, head, head_dim)
    elif layout == "flat":
        shape = (batch, embd)
    else:
        raise ValueError("layout must be 'heads' or 'flat'")
    return torch.zeros(shape, device=device, dtype=dtype)


@torch.no_grad()
def esa_prefill(module: torch.nn.Module, x: torch.Tensor, state: torch.Tensor | None = None, *,
                backend: str | None = None, compass: int | None = None):
    """Prompt prefill; returns (y [B,T,C], final state [B,H,D]).

    ``backend=None`` keeps the module's backend; ``backend="lightning"`` or an
    explicit ``state`` runs the exact recurrence from that state (zero if None).
    """
    if x.ndim != 3 or x.size(1) <= 0:
        raise ValueError(f"Prefill expects non-empty [B,T,C], got {tuple(x.shape)}")
    require_cuda_input(x, "esa_prefill")
    B, T, C = x.shape
    _, head, head_dim = _dimensions(module)
    bk = _unwrap_backend(module)
    q, g, v = _project_logits(module, x)
    requested = None if backend is None else str(backend).lower()
    if requested is not None and requested not in {"lightning", "thunder", "pulse", "flare"}:
        raise ValueError(f"Unsupported ESA backend for prefill: {requested!r}")

    if state is None and requested != "lightning":
        name = requested or _backend_name(module)
        dtype = g.dtype if name == "flare" else _state_dtype(module, x.device, g.dtype, backend_name=name)
        cps = (int(compass) if compass is not None
               else int(getattr(bk, "compass", 16) or 16)) if name == "thunder" else 16
        e0 = None
    else:
        if state is None:
            dtype = _state_dtype(module, x.device, g.dtype, backend_name=_backend_name(module))
            e0 = None
        else:
            e0 = state.reshape(B, head * head_dim)
            dtype = state.dtype
        cps = 16
    E, _ = ops.gated_scan(g, v, e0, float(bk.gate_min), float(bk.gate_max), cps, dtype)
    y = _readout(module, q, E, output_dtype=x.dtype)
    return y, E[:, -1].reshape(B, head, head_dim).contiguous()


lightning_prefill = esa_prefill


def lightning_decode_step(module: torch.nn.Module, x: torch.Tensor, state: torch.Tensor):
    """Exact one-token ESA-Lightning step; returns (y, new state).

    x is [B, C] or [B, 1, C]; state is [B, H, D] or flat [B, C] (layout kept).
    """
    if x.ndim == 2:
        x3, squeeze = x.unsqueeze(1), True
    elif x.ndim == 3 and x.size(1) == 1:
        x3, squeeze = x, False
    else:
        raise ValueError(f"decode_step expects [B,C] or [B,1,C], got {tuple(x.shape)}")
    require_cuda_input(x3, "lightning_decode_step")
    B = x3.size(0)
    embd, head, head_dim = _dimensions(module)
    bk = _unwrap_backend(module)
    flat_state = state.ndim == 2
    qgv = bk.qgv(x3)[:, 0]
    new_state, z = ops.lightning_step(qgv, state.reshape(B, embd), float(bk.gate_min),
                                      float(bk.gate_max), float(bk.eps), x3.dtype)
    y = bk.dropout(bk.out_proj(z))
    y = y if squeeze else y.unsqueeze(1)
    new_state = new_state if flat_state else new_state.reshape(B, head, head_dim)
    return y, new_state


def sample_next_token(logits: torch.Tensor, *, temperature: float = 1.0, top_k: int | None = None,
                      top_p: float | None = None) -> torch.Tensor:
    """Greedy (temperature <= 0), top-k / top-p filtered multinomial sampling
    (generation.py:472-560)."""
    if logits.ndim == 3:
        logits = logits[:, -1]
    if logits.ndim != 2:
        raise ValueError(f"Expected logits [B,V] or [B,T,V], got {tuple(logits.shape)}")
    if temperature <= 0:
        return torch.argmax(logits, dim=-1, keepdim=True)
    logits = logits / max(float(temperature), 1e-5)
    if top_k is not None:
        k = min(int(top_k), logits.size(-1))
        values, _ = torch.topk(logits, k)
        logits = logits.masked_fill(logits < values[:, [-1]], float("-inf"))
    if top_p is not None and 0.0 < float(top_p) < 1.0:
        sorted_logits, sorted_indices = torch.sort(logits, descending=True)
        cumulative = torch.cumsum(F.softmax(sorted_logits, dim=-1), dim=-1)
        remove = cumulative > float(top_p)
        remove[:, 1:] = remove[:, :-1].clone()
        remove[:, 0] = False
        sorted_logits = sorted_logits.masked_fill(remove, float("-inf"))
        logits = torch.full_like(logits, float("-inf"))
        logits.scatter_(1, sorted_indices, sorted_logits)
    return torch.multinomial(F.softmax(logits, dim=-1), num_samples=1)
