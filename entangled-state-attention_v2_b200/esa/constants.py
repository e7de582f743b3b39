# Copyright 2026 Zameer Hussain and Akhtar Hussain
# Licensed under the Apache License, Version 2.0.
# Portions of this file reproduce the public interface of esa/constants.py of
# Entangled-State-Attention v2.1.1 (signatures, dataclasses, validation and
# error messages), under that licence.

"""ESA algorithm constants (values of esa/constants.py:6-10 in the reference)."""

from __future__ import annotations

ESA_GATE_MIN = 0.80
ESA_GATE_MAX = 0.995
ESA_SCAN_EPS = 1e-6
SUPPORTED_BACKENDS = {"thunder", "flare", "pulse"}
SUPPORTED_PRECISIONS = {"fp8", "fp16", "bf16", "fp32", "fp64"}
