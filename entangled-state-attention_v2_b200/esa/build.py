"""Build libesa_b200.so in-tree with nvcc for sm_100a (no JIT cache).

    python -m esa.build          (from entangled-state-attention_v2_b200/)

Sources: ../csrc/*.cu.  cudart is linked statically so the library carries no
runtime-version coupling to the PyTorch wheel's own cudart.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
OUT = PKG / "libesa_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
         "--expt-relaxed-constexpr", "-cudart", "static"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def up_to_date() -> bool:
    if not OUT.exists():
        return False
    t = OUT.stat().st_mtime
    deps = sources() + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + \
        [PKG.parent.parent / "include" / "esa_b200.h", Path(__file__)]
    return all(p.stat().st_mtime <= t for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUT
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, *FLAGS, "-o", str(tmp), *map(str, sources())]
    if verbose:
        print(" ".join(cmd))
    # compile translation units in parallel
    subprocess.run(cmd + ["--threads", "0"], check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(OUT)
