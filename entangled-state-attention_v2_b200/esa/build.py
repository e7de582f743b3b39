"""Build libesa_b200.so in-tree with nvcc for sm_100a (no JIT cache).

    python -m esa.build [--force]      (from entangled-state-attention_v2_b200/)

Sources: ../csrc/*.cu, compiled to objects in parallel (one nvcc per
translation unit) and linked into esa/libesa_b200.so.  cudart is linked
statically so the library carries no runtime-version coupling to the PyTorch
wheel's own cudart.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
import tempfile
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG.parent / "csrc"
INCLUDE = PKG.parent.parent / "include"
OUT = PKG / "libesa_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
          "-Xcompiler", "-fvisibility=hidden"]


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
        [INCLUDE / "esa_b200.h", Path(__file__)]
    return all(p.stat().st_mtime <= t for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None,
          out: Path | None = None) -> Path:
    out = out or OUT
    if not force and out == OUT and up_to_date():
        return out
    exe = nvcc()
    flags = CFLAGS + list(extra_flags or [])
    with tempfile.TemporaryDirectory(prefix="esa_build_") as tmp:
        objs = []

        def compile_one(src: Path) -> Path:
            obj = Path(tmp) / (src.stem + ".o")
            cmd = [exe, *ARCH, *flags, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
            return obj

        with ThreadPoolExecutor(max_workers=max(1, min(len(sources()), os.cpu_count() or 1))) as ex:
            objs = list(ex.map(compile_one, sources()))
        tmp_out = Path(tmp) / out.name
        cmd = [exe, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp_out), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        shutil.copyfile(tmp_out, str(out) + ".tmp")
        os.replace(str(out) + ".tmp", out)
    return out


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(OUT)
