"""Seeded, platform-independent parameter values for model-level fixtures.

Both the fixture generator (which runs the reference ESAModel on the CPU) and
the GPU tests (which run this package's ESAModel) fill a model with the values
below, so the two see bit-identical weights without a stored checkpoint (the
24-layer, 1024-wide decode model has 336 M parameters: 1.3 GB in fp32).

Values come from numpy's PCG64 generator as uniform float32 draws (integer
arithmetic and one exact scaling, so every x86 host produces the same bits),
centred and scaled to the spread the reference's own initialisation uses
(esa/model.py: normal(0, 0.02) for Linear and Embedding weights, 0.02 /
sqrt(2 n_layer) for the projections into the residual stream; LayerNorm
weights around 1).  Biases and LayerNorm parameters get small random values
too, so that every parameter takes part in the parity checks.

Parameters are visited in sorted state_dict-key order; a tensor reachable
under two keys (the tied wte / lm_head weight) is filled once, under the
first key.  This module imports neither package, only torch and numpy.
"""

from __future__ import annotations

import math

import numpy as np
import torch

_SQRT12 = math.sqrt(12.0)


def _uniform(seed: int, index: int, shape, std: float, mean: float = 0.0) -> torch.Tensor:
    rng = np.random.Generator(np.random.PCG64([seed, index]))
    u = rng.random(size=int(np.prod(shape)) if shape else 1, dtype=np.float32)
    # uniform on [0,1) has std 1/sqrt(12): centre, scale to the target std
    vals = (u - np.float32(0.5)) * np.float32(std * _SQRT12) + np.float32(mean)
    return torch.from_numpy(vals.astype(np.float32)).reshape(shape)


def _spread(name: str, n_layer: int) -> tuple[float, float]:
    """(mean, std) of a parameter, from its state_dict key."""
    if name.endswith("bias"):
        return 0.0, 0.01
    if ".ln" in name or name.startswith("ln_"):
        return 1.0, 0.05  # LayerNorm weight
    if name.endswith("proj.weight"):
        return 0.0, 0.02 / math.sqrt(2 * n_layer)
    return 0.0, 0.02


@torch.no_grad()
def fill_model(model: torch.nn.Module, seed: int, n_layer: int) -> None:
    """Overwrite every parameter of `model` (any device, any float dtype) with
    the seeded values of its key."""
    sd = model.state_dict(keep_vars=True)
    done: set[int] = set()
    for index, name in enumerate(sorted(sd)):
        t = sd[name]
        if not torch.is_floating_point(t):
            continue
        key = t.data_ptr()
        if key in done:
            continue
        done.add(key)
        mean, std = _spread(name, n_layer)
        t.copy_(_uniform(seed, index, tuple(t.shape), std, mean).to(t.dtype))
