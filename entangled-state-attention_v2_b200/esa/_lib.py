"""Loader for the C-ABI library ``libesa_b200.so`` (include/esa_b200.h).

The library is built in-tree by ``esa/build.py`` (``nvcc -gencode
arch=compute_100a,code=sm_100a``).  There is no fallback: if the library is
missing every ESA operation raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("ESA_B200_LIB", str(_HERE / "libesa_b200.so")))

# element type codes (include/esa_b200.h)
DTYPE_F16, DTYPE_BF16, DTYPE_F32, DTYPE_F64 = 0, 1, 2, 3
ABI_VERSION = 1

STATUS_LOOKBACK_TIMEOUT = 1
STATUS_COPY_TIMEOUT = 2

_lock = threading.Lock()
_lib = None

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f64 = ctypes.c_double
_sz = ctypes.c_size_t

# name -> (restype, argtypes); the exact set of symbols include/esa_b200.h declares
SIGNATURES = {
    "esa_abi_version": (_int, []),
    "esa_last_error": (ctypes.c_char_p, []),
    "esa_scan_last_path": (_int, []),
    "esa_device_status": (_int, [_int, _int, ctypes.POINTER(ctypes.c_uint)]),
    "esa_readout_fwd": (_int, [_vp, _i64, _int, _vp, _i64, _int, _vp, _i64, _int, _vp, _i64, _i64,
                               _f64, _vp]),
    "esa_readout_bwd": (_int, [_vp, _i64, _int, _vp, _i64, _int, _vp, _i64, _int, _vp, _vp, _i64,
                               _int, _vp, _i64, _int, _i64, _i64, _f64, _vp]),
    "esa_layer_norm_fwd": (_int, [_vp, _int, _vp, _vp, _int, _vp, _int, _vp, _vp, _i64, _i64, _f64, _vp]),
    "esa_layer_norm_workspace_bytes": (_sz, [_i64, _i64]),
    "esa_add_layer_norm_fwd": (_int, [_vp, _int, _vp, _int, _vp, _vp, _vp, _int, _vp, _int, _vp, _vp, _i64,
                                      _i64, _f64, _vp]),
    "esa_add_layer_norm_bwd": (_int, [_vp, _int, _vp, _int, _vp, _int, _vp, _int, _vp, _vp, _vp, _vp, _int,
                                      _vp, _vp, _vp, _sz, _i64, _i64, _vp]),
    "esa_layer_norm_bwd": (_int, [_vp, _int, _vp, _int, _vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i64,
                                  _i64, _vp]),
    "esa_cross_entropy_fwd": (_int, [_vp, _i64, _int, _vp, _i64, _vp, _vp, _i64, _i64, _vp]),
    "esa_cross_entropy_bwd": (_int, [_vp, _i64, _int, _vp, _i64, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "esa_wait_selftest": (_int, [ctypes.POINTER(ctypes.c_uint), ctypes.POINTER(ctypes.c_uint), _vp]),
    "esa_scan_workspace_bytes": (_sz, [_i64, _i64, _i64, _int, _int]),
    "esa_scan_fwd": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _int, _int, _vp, _vp, _vp, _sz, _vp]),
    "esa_scan_fwd_noalloc": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _int, _int, _vp, _vp, _vp]),
    "esa_scan_host_staging_bytes": (_sz, [_i64, _i64, _i64, _int, _int]),
    "esa_scan_fwd_host": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _int, _int, _vp, _sz, _vp]),
    "esa_scan_fwd_resume": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _int, _int, _vp, _vp, _vp, _sz, _vp]),
    "esa_scan_summary": (_int, [_vp, _vp, _i64, _i64, _i64, _int, _vp, _vp, _vp, _vp, _sz, _vp]),
    "esa_scan_prod": (_int, [_vp, _vp, _i64, _i64, _i64, _int, _vp]),
    "esa_scan_fixup": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp]),
    "esa_scan_rev": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _int, _vp, _vp, _vp,
                            _sz, _vp]),
    "esa_gated_scan_fwd": (_int, [_vp, _vp, _i64, _int, _vp, _int, _i64, _i64, _i64, _f64, _f64,
                                  _int, _int, _vp, _vp, _vp, _sz, _vp]),
    "esa_gated_scan_bwd": (_int, [_vp, _vp, _i64, _int, _vp, _vp, _int, _vp, _vp, _i64, _int,
                                  _i64, _i64, _i64, _f64, _f64, _int, _int, _vp, _vp, _vp, _sz,
                                  _vp]),
    "esa_lightning_step": (_int, [_vp, _i64, _int, _vp, _vp, _int, _vp, _int, _i64, _i64, _f64,
                                  _f64, _f64, _vp]),
    "esa_decode_block_scratch_bytes": (_sz, [_i64, _i64, _int]),
    "esa_decode_block": (_int, [_vp] * 18 + [_i64, _i64, _int, _f64, _f64, _f64, _f64, _vp, _sz, _vp]),
    "esa_decode_head": (_int, [_vp, _vp, _vp, _vp, _f64, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp]),
    "esa_layer_workspace_bytes": (_sz, [_i64, _i64, _i64, _int, _int, _int]),
    "esa_layer_fwd": (_int, [_vp, _i64, _int, _vp, _int, _vp, _int, _vp, _i64, _i64, _i64, _f64, _f64, _f64,
                             _vp, _vp, _vp, _sz, _vp]),
    "esa_layer_bwd": (_int, [_vp, _int, _vp, _i64, _int, _vp, _int, _vp, _vp, _i64, _i64, _i64, _i64, _f64,
                             _f64, _f64, _vp, _vp, _vp, _sz, _vp]),
}


class ESALibraryError(RuntimeError):
    pass


def lib():
    """The loaded library (raises ESALibraryError if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ESALibraryError(
                    f"ESA CUDA library not found at {LIB_PATH}. Build it with "
                    "`python -c 'import __graft_entry__ as g; g.build()'` from the repository "
                    "root (nvcc for sm_100a). There is no CPU fallback."
                )
            L = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            v = L.esa_abi_version()
            if v != ABI_VERSION:
                raise ESALibraryError(f"libesa_b200.so ABI {v}, expected {ABI_VERSION}")
            _lib = L
    return _lib


def last_error() -> str:
    msg = lib().esa_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    if rc == 0:
        return
    msg = last_error()
    if rc == -1:
        raise ValueError(f"{what}: {msg}")
    if rc == -2:
        raise TypeError(f"{what}: {msg}")
    raise RuntimeError(f"{what} failed ({rc}): {msg}")


SCAN_PATHS = {0: "none", 1: "sequential", 2: "lookback", 3: "strip", 4: "lane", 5: "chain"}


def last_scan_path() -> str:
    """Kernel family of the last scan launch on this host thread: "sequential",
    "lookback", "strip" or "lane" ("none" before any)."""
    return SCAN_PATHS.get(int(lib().esa_scan_last_path()), "unknown")


def device_status(device: int, clear: bool = True) -> int:
    """Read (and by default clear) the device status word; synchronises the device."""
    out = ctypes.c_uint(0)
    check(lib().esa_device_status(int(device), int(bool(clear)), ctypes.byref(out)), "esa_device_status")
    return int(out.value)
