"""ESA backends on the B200 kernels (same import surface as the reference's
esa/backends/__init__.py:1-15)."""

from .flare import FlareESA, flare_scan
from .thunder import ThunderESA, thunder_scan, thunder_scan_host
from .pulse import PulseESA, pulse_scan

__all__ = ["FlareESA", "ThunderESA", "PulseESA", "flare_scan", "thunder_scan", "thunder_scan_host",
           "pulse_scan"]
