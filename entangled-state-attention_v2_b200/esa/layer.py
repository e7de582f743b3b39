# Copyright 2026 Zameer Hussain and Akhtar Hussain
# Licensed under the Apache License, Version 2.0.
# Portions of this file reproduce the public interface of esa/layer.py of
# Entangled-State-Attention v2.1.1 (signatures, dataclasses, validation and
# error messages), under that licence.

"""Public ESA layer -- the drop-in boundary.

Same constructor, attributes, validation messages and methods as the
reference's ``esa.ESA`` (esa/layer.py:10-226): backend selection between
thunder / flare / pulse (all three here run on the B200 kernels), device
placement, optional ``torch.compile``, ``forward``, ``prefill``,
``decode_step`` and the ESA-Lightning aliases.
"""

from __future__ import annotations

import torch
import torch.nn as nn


class ESA(nn.Module):
    """Entangled State Attention sequence-mixing layer.

    Canonical public names: embd, head, batch, block, compass.
    Backends: thunder (default, compass=16), flare and pulse (no compass).
    """

    def __init__(self, embd: int, head: int = 4, batch: int | None = None,
                 block: int | None = None, backend: str = "thunder", precision: str = "fp16", *,
                 compass: int | None = None, dropout: float = 0.0, gate_min: float = 0.80,
                 gate_max: float = 0.995, eps: float = 1e-5,
                 device: str | torch.device | None = "auto", auto_compile: bool = False,
                 compile_mode: str = "default", auto_move_input: bool = True,
                 strict_checks: bool = False):
        super().__init__()
        if embd <= 0:
            raise ValueError(f"embd must be positive, got {embd}.")
        if head <= 0:
            raise ValueError(f"head must be positive, got {head}.")
        if embd % head != 0:
            raise ValueError(f"embd must be divisible by head, got embd={embd}, head={head}.")
        if batch is not None and batch <= 0:
            raise ValueError(f"batch must be positive when set, got {batch}.")
        if block is not None and block <= 0:
            raise ValueError(f"block must be positive when set, got {block}.")

        self.embd = int(embd)
        self.head = int(head)
        self.batch = None if batch is None else int(batch)
        self.block = None if block is None else int(block)
        self.backend = str(backend).lower()
        self.precision = str(precision).lower()
        self.dropout = float(dropout)
        self.gate_min = float(gate_min)
        self.gate_max = float(gate_max)
        self.eps = float(eps)
        self.auto_move_input = bool(auto_move_input)
        self.strict_checks = bool(strict_checks)
        self.compiled = False

        if self.backend == "thunder":
            self.compass = 16 if compass is None else int(compass)
        elif self.backend in {"flare", "pulse"}:
            if compass is not None:
                raise ValueError("compass is only supported by backend='thunder'.")
            self.compass = None
        else:
            raise ValueError(
                f"Unknown ESA backend: {backend!r}. Supported backends: 'flare', 'thunder', 'pulse'."
            )
        if self.compass is not None and self.compass <= 0:
            raise ValueError(f"compass must be positive, got {self.compass}.")

        common = dict(dropout=self.dropout, precision=self.precision, gate_min=self.gate_min,
                      gate_max=self.gate_max, eps=self.eps)
        if self.backend == "flare":
            from .backends.flare import FlareESA
            self.layer = FlareESA(n_embd=self.embd, n_head=self.head, **common)
        elif self.backend == "thunder":
            from .backends.thunder import ThunderESA
            self.layer = ThunderESA(embd=self.embd, head=self.head, compass=self.compass, **common)
        else:
            from .backends.pulse import PulseESA
            self.layer = PulseESA(n_embd=self.embd, n_head=self.head, **common)

        # the generation engine reads embd/head from the backend
        if not hasattr(self.layer, "embd"):
            self.layer.embd = self.embd
        if not hasattr(self.layer, "head"):
            self.layer.head = self.head

        self.register_buffer("_esa_device_ref", torch.empty(0), persistent=False)

        if device == "auto":
            device = "cuda" if torch.cuda.is_available() else "cpu"
        if device is not None:
            self.to(device)
        if auto_compile:
            self.compile(mode=compile_mode)

    def compile(self, mode: str = "default"):
        """Wrap the backend in torch.compile (the ESA kernels are opaque custom ops)."""
        try:
            self.layer = torch.compile(self.layer, mode=mode, fullgraph=False)
            self.compiled = True
        except Exception:
            self.compiled = False
        return self

    def _prepare_input(self, x: torch.Tensor) -> torch.Tensor:
        if self.auto_move_input:
            target = self._esa_device_ref.device
            if x.device != target:
                x = x.to(target, non_blocking=True)
        if x.dim() != 3:
            raise ValueError(f"ESA input must be [batch, seq, embd], got {tuple(x.shape)}.")
        B, T, C = x.shape
        if C != self.embd:
            raise ValueError(f"ESA expected embd={self.embd}, got {C}.")
        if self.strict_checks:
            if self.batch is not None and B != self.batch:
                raise ValueError(f"ESA expected batch={self.batch}, got {B}.")
            if self.block is not None and T > self.block:
                raise ValueError(f"ESA block limit is {self.block}, got {T}.")
        return x

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.layer(self._prepare_input(x))

    def init_state(self, batch: int, *, device=None, dtype=None, layout: str = "heads") -> torch.Tensor:
        """Zero recurrent state for `batch` rows ([batch, head, head_dim] or flat)."""
        from .generation import lightning_init_state
        return lightning_init_state(self, batch, device=device, dtype=dtype, layout=layout)

    @torch.no_grad()
    def prefill(self, x: torch.Tensor, state: torch.Tensor | None = None, *,
                backend: str | None = None, compass: int | None = None):
        """Process a whole sequence; returns (outputs, final recurrent state)."""
        from .generation import esa_prefill
        return esa_prefill(self, self._prepare_input(x), state=state, backend=backend,
                           compass=compass)

    def decode_step(self, x: torch.Tensor, state: torch.Tensor):
        """Advance the recurrent state by one token; returns (output, next state)."""
        from .generation import lightning_decode_step
        return lightning_decode_step(self, x, state)

    lightning_prefill = prefill
    lightning_step = decode_step
