"""Shared pytest setup: the ``gpu`` marker and import paths.

The Python package ``esa`` (the drop-in mirror of the reference's package)
lives in ``entangled-state-attention_v2_b200/``; the CPU oracle in ``oracle/``.
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "entangled-state-attention_v2_b200"
for p in (str(PKG), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
