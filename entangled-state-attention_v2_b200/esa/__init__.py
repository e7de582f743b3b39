"""ESA (Entangled State Attention) on NVIDIA B200 -- drop-in for the reference
package's hot path (maxzameer/Entangled-State-Attention_v2 v2.1.1, ``esa``).

The gated diagonal recurrence E_t = A_t * E_{t-1} + B_t runs in hand-written
sm_100a CUDA kernels (``libesa_b200.so``, C ABI in include/esa_b200.h) behind
the reference's public Python surface: ``esa.ESA``, ``esa.ESAModel``,
``esa.backends.thunder.thunder_scan`` and friends.
"""

from __future__ import annotations

from .layer import ESA
from .model import ESAModel, ESAModelConfig
from .generation import GenerationResult, GenerationStats
from .backends import FlareESA, PulseESA, ThunderESA

__version__ = "2.1.1"
__b200_version__ = "0.1.0"

__all__ = [
    "ESA",
    "ESAModel",
    "ESAModelConfig",
    "GenerationResult",
    "GenerationStats",
    "FlareESA",
    "ThunderESA",
    "PulseESA",
]
