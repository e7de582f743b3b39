"""The lane-serial scan (one lane per channel vector, walking the steps in
order) against the fp64 oracle.

1. Shapes with enough channels for two consumer warps per SM: forward with
   initial and final states, reverse with the gradient of the initial state,
   fused gated forward/backward on qgv slices (row stride 3C), the summary
   pass, ragged time tiles and partial strips, both CTA widths (one and two
   consumer warps).  The automatic choice runs the lane kernel for the 16-bit
   plain forward (checked through esa_scan_last_path) and the strip kernel
   for the rest.
2. This file and every scan test file re-run in a child process with the lane
   path forced (ESA_SCAN_PATH=lane): there every case above must run the lane
   kernel, and the suites take it to few channels, time pieces of the split
   scan, summary passes, incoming states and the host pipeline.

Tolerance: relative Frobenius error ||got - ref|| / ||ref|| against the fp64
oracle on the same rounded inputs -- 1e-5 fp32, 2e-3 fp16 / bf16, 1e-12 fp64.
"""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 2e-3, torch.float64: 1e-12}
DEV = "cuda"
ROOT = Path(__file__).resolve().parent.parent


def rel(got, ref) -> float:
    got = np.asarray(got.detach().double().cpu() if torch.is_tensor(got) else got, dtype=np.float64)
    ref = np.asarray(ref.detach().double().cpu() if torch.is_tensor(ref) else ref, dtype=np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.isfinite(got).all()
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-300))


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    from esa import ops
    torch.cuda.synchronize()
    ops.check_device_status()


FORCED = os.environ.get("ESA_SCAN_PATH") == "lane"


def _expect_lane(automatic: bool) -> None:
    """The lane kernel ran if it is forced, or if the automatic choice takes it."""
    from esa import _lib
    if FORCED or automatic:
        assert _lib.last_scan_path() == "lane"


def _acc(dtype):
    return torch.float64 if dtype == torch.float64 else torch.float32


# (shape [B,T,H,D], dtype): enough channels for the automatic lane path on a
# 148-SM B200 (>= 296 warps of 64 16-bit or 32 wider channels); T not a
# multiple of the 32-step tile; H*D not a multiple of the strip width
FWD_CASES = [
    ((40, 77, 10, 56), torch.float16),   # 9 strips of 64 per row, the last one partial
    ((40, 70, 16, 64), torch.float16),   # two consumer warps per CTA (128-channel strips)
    ((40, 77, 10, 56), torch.bfloat16),
    ((24, 45, 8, 56), torch.float32),    # 14 strips of 32
    ((20, 33, 2, 264), torch.float64),   # 16.5 strips of 32
]


@pytest.mark.parametrize("shape,dtype", FWD_CASES)
def test_lane_forward_and_reverse_with_states(shape, dtype):
    from esa import ops
    g = torch.Generator().manual_seed(41)
    nb, T, H, D = shape
    A = torch.sigmoid(2 * torch.randn(shape, generator=g) + 2).to(dtype)
    B = torch.randn(shape, generator=g).to(dtype)
    e0 = torch.randn(nb, H * D, generator=g).to(_acc(dtype))
    E, e_last = ops.scan(A.to(DEV), B.to(DEV), e0.to(DEV), 16)
    _expect_lane(dtype in (torch.float16, torch.bfloat16))
    ref = oracle.scan_fwd(A.double(), B.double(), e0=e0.double())
    assert rel(E, ref) < TOL[dtype]
    assert rel(e_last, ref[:, -1].reshape(nb, H * D)) < TOL[dtype]
    # reverse: the stored (rounded) E, upstream dE, gradient of e0
    dE = torch.randn(shape, generator=g).to(dtype)
    dA, dB, de0 = ops.scan_backward(A.to(DEV), E, dE.to(DEV), e0.to(DEV), 16)
    _expect_lane(False)
    dA_ref, dB_ref, de0_ref = oracle.scan_rev(A.double(), E.double().cpu(), dE.double(), e0=e0.double())
    assert rel(dB, dB_ref) < TOL[dtype]
    assert rel(dA, dA_ref) < TOL[dtype]
    assert rel(de0, de0_ref) < TOL[dtype]


@pytest.mark.parametrize("raw_dtype,scan_dtype,C", [
    (torch.float16, torch.float16, 640),
    (torch.bfloat16, torch.bfloat16, 640),
    (torch.float32, torch.float32, 320),
    (torch.float32, torch.float16, 640),
])
def test_lane_gated_fwd_bwd_strided(raw_dtype, scan_dtype, C):
    """Gate prologue + scan + gate epilogue on qgv slices (row stride 3C)."""
    from esa import ops
    g = torch.Generator().manual_seed(42)
    Bsz, T = 32, 50
    qgv = torch.randn(Bsz, T, 3 * C, generator=g).to(raw_dtype)
    gr, vr = qgv[..., C:2 * C], qgv[..., 2 * C:]
    qd = qgv.to(DEV)
    grd, vrd = qd[..., C:2 * C], qd[..., 2 * C:]
    E, _ = ops.gated_scan(grd, vrd, None, 0.8, 0.995, 16, scan_dtype)
    _expect_lane(False)
    A64, B64 = oracle.gate(gr, vr)
    Ar = torch.from_numpy(A64).to(scan_dtype).double()
    Br = torch.from_numpy(B64).to(scan_dtype).double()
    ref = oracle.scan_fwd(Ar.reshape(Bsz, T, 1, C), Br.reshape(Bsz, T, 1, C)).reshape(Bsz, T, C)
    tol = max(TOL[scan_dtype], TOL[raw_dtype])
    assert rel(E, ref) < tol
    dE = torch.randn(Bsz, T, C, generator=g).to(scan_dtype)
    dg, dv, _ = ops.gated_scan_backward(grd, vrd, E, dE.to(DEV), None, 0.8, 0.995, 16)
    _expect_lane(False)
    dA, dB, _ = oracle.scan_rev(Ar.reshape(Bsz, T, 1, C), E.double().cpu().reshape(Bsz, T, 1, C),
                                dE.double().reshape(Bsz, T, 1, C))
    dg_ref, dv_ref = oracle.gate_bwd(gr, vr, dA.reshape(Bsz, T, C), dB.reshape(Bsz, T, C))
    assert rel(dg, dg_ref) < tol * 2
    assert rel(dv, dv_ref) < tol * 2


def test_lane_summary_matches_oracle():
    """The summary pass (end state and coefficient product, no per-step
    outputs) on a lane-sized slice."""
    from esa import ops
    g = torch.Generator().manual_seed(43)
    shape = (40, 200, 16, 64)
    A = torch.sigmoid(torch.randn(shape, generator=g) + 3)
    B = torch.randn(shape, generator=g)
    e0 = torch.randn(40, 1024, generator=g)
    e_last, prod = ops.scan_summary(A.to(DEV), B.to(DEV), e0.to(DEV))
    _expect_lane(False)
    ref = oracle.scan_fwd(A.double(), B.double(), e0=e0.double())
    assert rel(e_last, ref[:, -1].reshape(40, 1024)) < 1e-5
    assert rel(prod, A.double().prod(dim=1).reshape(40, 1024)) < 1e-5


@pytest.mark.skipif(FORCED, reason="already the forced child")
def test_scan_suites_with_the_lane_path_forced():
    env = dict(os.environ, ESA_SCAN_PATH="lane")
    files = ["tests/test_gpu_lane.py", "tests/test_gpu_scan.py", "tests/test_gpu_chain.py",
             "tests/test_parallel.py", "tests/test_gpu_layer.py"]
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                        *files], cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, (r.stdout + r.stderr)[-4000:]
