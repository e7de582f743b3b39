"""Parity of the scan kernels (forward, reverse, gated) with the fp64 oracle.

Tolerance (the build's parity bar): relative Frobenius error
||got - ref||_2 / ||ref||_2 against the fp64 oracle evaluated on the same
rounded inputs -- 1e-5 for fp32, 2e-3 for fp16 / bf16, 1e-12 for fp64.  Per
element relative error is not used: near zero it measures only the output
rounding (e.g. 4e-2 for fp16 from rounding alone).
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 2e-3, torch.float64: 1e-12}
DTYPES = [torch.float32, torch.float16, torch.bfloat16, torch.float64]
DEV = "cuda"


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


def _shapes():
    z = np.load(GOLDEN / "scan_shapes.npz")
    return {n: (torch.from_numpy(z[f"{n}_A"]), torch.from_numpy(z[f"{n}_B"]))
            for n in ("t1", "t9", "t33_hd15", "t130", "t64_hd1024")}


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("compass", [16, 32, 64, 5])
def test_thunder_scan_golden_shapes(dtype, compass):
    from esa.backends.thunder import thunder_scan
    for name, (A, B) in _shapes().items():
        Ad, Bd = A.to(dtype), B.to(dtype)
        ref = oracle.scan_fwd(Ad.double(), Bd.double())
        got = thunder_scan(Ad.to(DEV), Bd.to(DEV), compass=compass)
        assert got.dtype == dtype and got.shape == A.shape
        assert rel(got, ref) < TOL[dtype], (name, rel(got, ref))


def test_reference_lifecycle_case():
    """The reference's own chunked-vs-pulse case (test_v2_1_model_lifecycle.py:17-52)."""
    from esa.backends.pulse import pulse_scan
    from esa.backends.thunder import thunder_scan
    z = np.load(GOLDEN / "scan_lifecycle.npz")
    A, B = torch.from_numpy(z["A"]).to(DEV), torch.from_numpy(z["B"]).to(DEV)
    for got in (thunder_scan(A, B, compass=4), pulse_scan(A, B), thunder_scan(A, B, c=16)):
        torch.testing.assert_close(got.cpu(), torch.from_numpy(z["pulse_f32"]), atol=1e-5, rtol=1e-5)
        assert rel(got, z["pulse_f64"]) < 1e-6


@pytest.mark.parametrize("dtype", DTYPES)
def test_scan_backward_matches_oracle(dtype):
    from esa.backends.thunder import thunder_scan
    g = torch.Generator().manual_seed(3)
    for shp in [(2, 21, 3, 8), (1, 70, 2, 16), (3, 257, 4, 64), (2, 64, 1, 1024), (1, 1, 2, 8)]:
        A = torch.sigmoid(2 * torch.randn(shp, generator=g) + 2).to(dtype)
        B = torch.randn(shp, generator=g).to(dtype)
        dE = torch.randn(shp, generator=g).to(dtype)
        Ad = A.to(DEV).requires_grad_(True)
        Bd = B.to(DEV).requires_grad_(True)
        E = thunder_scan(Ad, Bd)
        E.backward(dE.to(DEV))
        # the reverse scan consumes the stored (rounded) E, as autograd would
        dA_ref, dB_ref, _ = oracle.scan_rev(A.double(), E.detach().double().cpu(), dE.double())
        assert rel(Bd.grad, dB_ref) < TOL[dtype], shp
        assert rel(Ad.grad, dA_ref) < TOL[dtype], shp


def test_scan_backward_golden_autograd():
    from esa.backends.thunder import thunder_scan
    z = np.load(GOLDEN / "scan_grad.npz")
    for n in ("g1", "g2"):
        A = torch.from_numpy(z[f"{n}_A"]).to(DEV).requires_grad_(True)
        B = torch.from_numpy(z[f"{n}_B"]).to(DEV).requires_grad_(True)
        thunder_scan(A, B).backward(torch.from_numpy(z[f"{n}_dE"]).to(DEV))
        assert rel(A.grad, z[f"{n}_dA"]) < 1e-12
        assert rel(B.grad, z[f"{n}_dB"]) < 1e-12


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_initial_state_and_final_state(dtype):
    from esa import ops
    g = torch.Generator().manual_seed(4)
    A = torch.sigmoid(torch.randn(3, 300, 2, 128, generator=g) + 3).to(dtype)
    B = torch.randn(3, 300, 2, 128, generator=g).to(dtype)
    e0 = torch.randn(3, 256, generator=g).to(dtype)
    E, e_last = ops.scan(A.to(DEV), B.to(DEV), e0.to(DEV), 16)
    ref = oracle.scan_fwd(A.double(), B.double(), e0=e0.double())
    assert rel(E, ref) < TOL[dtype]
    assert rel(e_last, ref[:, -1].reshape(3, 256)) < TOL[dtype]
    # gradient w.r.t. the initial state
    Ad = A.to(DEV).requires_grad_(True)
    Bd = B.to(DEV).requires_grad_(True)
    e0d = e0.to(DEV).requires_grad_(True)
    dE = torch.randn(A.shape, generator=g).to(dtype)
    E2, _ = ops.scan(Ad, Bd, e0d, 32)
    E2.backward(dE.to(DEV))
    dA_ref, dB_ref, de0_ref = oracle.scan_rev(A.double(), ref, dE.double(), e0=e0.double())
    assert rel(e0d.grad, de0_ref) < TOL[dtype]
    assert rel(Ad.grad, dA_ref) < TOL[dtype]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(16, 300, 8, 128), (16, 129, 8, 125)])
def test_scan_backward_narrow_strips(dtype, shape):
    """16-bit reverse scans on 128-channel strips of four-channel lanes (taken
    when those strips fill the GPU; here 128 of them): a ragged last tile
    (T = 300, 129), a last strip with 104 of 128 channels (hd = 1000), and
    the gradient w.r.t. an initial state."""
    from esa import _lib, ops
    g = torch.Generator().manual_seed(shape[1])
    nb, T, H, D = shape
    A = torch.sigmoid(torch.randn(shape, generator=g) + 3).to(dtype)
    B = torch.randn(shape, generator=g).to(dtype)
    e0 = torch.randn(nb, H * D, generator=g).to(dtype)
    dE = torch.randn(shape, generator=g).to(dtype)
    Ad = A.to(DEV).requires_grad_(True)
    Bd = B.to(DEV).requires_grad_(True)
    e0d = e0.to(DEV).requires_grad_(True)
    E, _ = ops.scan(Ad, Bd, e0d, 16)
    E.backward(dE.to(DEV))
    assert _lib.last_scan_path() in ("strip", "lane")  # lane: ESA_SCAN_PATH=lane
    dA_ref, dB_ref, de0_ref = oracle.scan_rev(A.double(), E.detach().double().cpu(), dE.double(),
                                              e0=e0.double())
    assert rel(Bd.grad, dB_ref) < TOL[dtype]
    assert rel(Ad.grad, dA_ref) < TOL[dtype]
    assert rel(e0d.grad, de0_ref.reshape(nb, H * D)) < TOL[dtype]


@pytest.mark.parametrize("raw_dtype,scan_dtype", [
    (torch.float32, torch.float32), (torch.float32, torch.float16), (torch.float16, torch.float16),
    (torch.bfloat16, torch.bfloat16), (torch.float16, torch.float32), (torch.float64, torch.float64),
    (torch.float32, torch.bfloat16)])
def test_gated_scan_fwd_bwd_strided(raw_dtype, scan_dtype):
    """Gate prologue + scan + gate epilogue on qgv slices (row stride 3C)."""
    from esa import ops
    g = torch.Generator().manual_seed(5)
    Bsz, T, C = 2, 131, 256
    qgv = torch.randn(Bsz, T, 3 * C, generator=g).to(raw_dtype)
    gr, vr = qgv[..., C:2 * C], qgv[..., 2 * C:]
    qd = qgv.to(DEV)
    grd, vrd = qd[..., C:2 * C], qd[..., 2 * C:]
    E, e_last = ops.gated_scan(grd, vrd, None, 0.8, 0.995, 16, scan_dtype)
    assert E.dtype == scan_dtype and E.shape == (Bsz, T, C)
    # oracle on the same rounded inputs: A, B rounded to the scan dtype (A.to(scan_dtype))
    A64, B64 = oracle.gate(gr, vr)
    Ar = torch.from_numpy(A64).to(scan_dtype).double()
    Br = torch.from_numpy(B64).to(scan_dtype).double()
    ref = oracle.scan_fwd(Ar.reshape(Bsz, T, 1, C), Br.reshape(Bsz, T, 1, C)).reshape(Bsz, T, C)
    tol = max(TOL[scan_dtype], TOL[raw_dtype] if raw_dtype != torch.float64 else 1e-12)
    assert rel(E, ref) < tol
    # backward
    dE = torch.randn(Bsz, T, C, generator=g).to(scan_dtype)
    dg, dv, _ = ops.gated_scan_backward(grd, vrd, E, dE.to(DEV), None, 0.8, 0.995, 16)
    assert dg.dtype == raw_dtype
    dA, dB, _ = oracle.scan_rev(Ar.reshape(Bsz, T, 1, C), E.double().cpu().reshape(Bsz, T, 1, C),
                                dE.double().reshape(Bsz, T, 1, C))
    dg_ref, dv_ref = oracle.gate_bwd(gr, vr, dA.reshape(Bsz, T, C), dB.reshape(Bsz, T, C))
    assert rel(dg, dg_ref) < tol * 2
    assert rel(dv, dv_ref) < tol * 2


def test_gated_scan_training_layer_shape():
    """The ESAModel training layer [16, 2048, 768] fp16 (12 heads of 64, qgv
    row stride 3C): forward and backward on the GPU, checked against the
    oracle on three batch rows (the kernels run all 16)."""
    from esa import ops
    g = torch.Generator().manual_seed(9)
    Bsz, T, C = 16, 2048, 768
    qgv = torch.randn(Bsz, T, 3 * C, generator=g).half()
    qd = qgv.to(DEV)
    grd, vrd = qd[..., C:2 * C], qd[..., 2 * C:]
    E, e_last = ops.gated_scan(grd, vrd, None, 0.8, 0.995, 16, torch.float16)
    dE = torch.randn(Bsz, T, C, generator=g).half()
    dg, dv, _ = ops.gated_scan_backward(grd, vrd, E, dE.to(DEV), None, 0.8, 0.995, 16)
    rows = [0, 7, 15]
    gr, vr = qgv[rows, :, C:2 * C], qgv[rows, :, 2 * C:]
    A64, B64 = oracle.gate(gr, vr)
    Ar = torch.from_numpy(A64).half().double().reshape(3, T, 1, C)
    Br = torch.from_numpy(B64).half().double().reshape(3, T, 1, C)
    ref = oracle.scan_fwd(Ar, Br).reshape(3, T, C)
    assert rel(E[rows], ref) < 2e-3
    assert rel(e_last[rows], ref[:, -1]) < 2e-3
    dA, dB, _ = oracle.scan_rev(Ar, E[rows].double().cpu().reshape(3, T, 1, C),
                                dE[rows].double().reshape(3, T, 1, C))
    dg_ref, dv_ref = oracle.gate_bwd(gr, vr, dA.reshape(3, T, C), dB.reshape(3, T, C))
    assert rel(dg[rows], dg_ref) < 4e-3
    assert rel(dv[rows], dv_ref) < 4e-3


@pytest.mark.parametrize("raw_dtype,scan_dtype", [
    (torch.float16, torch.float16), (torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32),
    (torch.float32, torch.float16), (torch.float32, torch.bfloat16), (torch.float16, torch.float32),
    (torch.bfloat16, torch.float32)])
@pytest.mark.parametrize("nb,T,C", [(4, 300, 2048), (8, 777, 1000)])
def test_gated_narrow_strip_scan(raw_dtype, scan_dtype, nb, T, C):
    """The narrow strip form (64-channel strips of 32 two-channel lanes),
    which the gated scans take whenever their 64-channel strips fill the GPU
    (here 128 strips): ragged last tiles (T = 300, 777), a last strip with 40
    of 64 channels (C = 1000), an initial state, the final state and its
    gradient -- against the oracle on the same rounded A, B."""
    from esa import _lib, ops
    g = torch.Generator().manual_seed(T + C)
    qgv = torch.randn(nb, T, 3 * C, generator=g).to(raw_dtype)
    gr, vr = qgv[..., C:2 * C], qgv[..., 2 * C:]
    qd = qgv.to(DEV)
    grd, vrd = qd[..., C:2 * C], qd[..., 2 * C:]
    e0 = torch.randn(nb, C, generator=g)
    E, e_last = ops.gated_scan(grd, vrd, e0.to(DEV), 0.8, 0.995, 16, scan_dtype)
    assert _lib.last_scan_path() in ("strip", "lane")  # lane: ESA_SCAN_PATH=lane
    A64, B64 = oracle.gate(gr, vr)
    Ar = torch.from_numpy(A64).to(scan_dtype).double().reshape(nb, T, 1, C)
    Br = torch.from_numpy(B64).to(scan_dtype).double().reshape(nb, T, 1, C)
    ref = oracle.scan_fwd(Ar, Br, e0=e0.double()).reshape(nb, T, C)
    tol = max(TOL[scan_dtype], TOL[raw_dtype])
    assert rel(E, ref) < tol
    assert rel(e_last, ref[:, -1]) < tol
    dE = torch.randn(nb, T, C, generator=g).to(scan_dtype)
    dg, dv, de0 = ops.gated_scan_backward(grd, vrd, E, dE.to(DEV), e0.to(DEV), 0.8, 0.995, 16)
    dA, dB, de0_ref = oracle.scan_rev(Ar, E.double().cpu().reshape(nb, T, 1, C), dE.double().reshape(nb, T, 1, C),
                                      e0=e0.double())
    dg_ref, dv_ref = oracle.gate_bwd(gr, vr, dA.reshape(nb, T, C), dB.reshape(nb, T, C))
    assert rel(dg, dg_ref) < tol * 2
    assert rel(dv, dv_ref) < tol * 2
    assert rel(de0, de0_ref.reshape(nb, C)) < tol


def test_gated_autograd_through_layer_slices():
    """torch autograd through the gated op equals autograd through the
    materialised gate + thunder_scan (both on the GPU, fp64)."""
    from esa import ops
    from esa.backends.thunder import thunder_scan
    g = torch.Generator().manual_seed(6)
    qgv = torch.randn(2, 77, 3 * 64, generator=g, dtype=torch.float64).to(DEV).requires_grad_(True)
    q, gr, vr = qgv.split(64, dim=-1)
    E, _ = ops.gated_scan(gr, vr, None, 0.8, 0.995, 16, torch.float64)
    w = torch.randn(2, 77, 64, generator=g, dtype=torch.float64).to(DEV)
    (E * w).sum().backward()
    g1 = qgv.grad.clone()
    qgv.grad = None
    q, gr, vr = qgv.split(64, dim=-1)
    A = 0.8 + (0.995 - 0.8) * torch.sigmoid(gr)
    Bw = (1 - A) * torch.tanh(vr)
    E2 = thunder_scan(A.reshape(2, 77, 4, 16).contiguous(), Bw.reshape(2, 77, 4, 16).contiguous())
    (E2.reshape(2, 77, 64) * w).sum().backward()
    assert rel(E, E2.reshape(2, 77, 64)) < 1e-13
    assert rel(g1, qgv.grad) < 1e-12


def test_fallback_path_unaligned_rows():
    """Rows that the bulk-copy path cannot stage (HD=15, odd pointer offsets)
    take the sequential kernel; results are the same."""
    from esa.backends.thunder import thunder_scan
    z = np.load(GOLDEN / "scan_shapes.npz")
    A = torch.from_numpy(z["t33_hd15_A"]).float().to(DEV)
    B = torch.from_numpy(z["t33_hd15_B"]).float().to(DEV)
    assert rel(thunder_scan(A, B), z["t33_hd15_pulse_f64"]) < 1e-5
    # misaligned base pointer: a view starting one element in
    buf = torch.randn(1 + 2 * 40 * 2 * 16, device=DEV)
    Bm = buf[1:].view(2, 40, 2, 16)
    Am = torch.sigmoid(Bm + 2)
    assert rel(thunder_scan(Am, Bm), oracle.scan_fwd(Am.cpu(), Bm.cpu())) < 1e-5


def test_empty_and_degenerate_shapes():
    from esa.backends.thunder import thunder_scan
    for shp in [(0, 5, 2, 8), (2, 0, 2, 8), (2, 5, 0, 8)]:
        E = thunder_scan(torch.ones(shp, device=DEV), torch.ones(shp, device=DEV))
        assert E.shape == shp
    A = torch.rand(4, 1, 3, 8, device=DEV)
    B = torch.randn(4, 1, 3, 8, device=DEV)
    torch.testing.assert_close(thunder_scan(A, B), B)


def test_argument_errors_match_reference():
    from esa.backends.thunder import thunder_scan
    a = torch.ones(2, 3, 4, 5, device=DEV)
    with pytest.raises(ValueError, match="same shape"):
        thunder_scan(a, torch.ones(2, 3, 4, 6, device=DEV))
    with pytest.raises(ValueError, match=r"\[B,T,H,D\]"):
        thunder_scan(a[0], a[0])
    with pytest.raises(ValueError, match="positive integer"):
        thunder_scan(a, a, compass=0)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_microbenchmark_size_properties(dtype):
    """Full microbenchmark size [32,4096,16,64]: sampled channels against the
    oracle, plus linearity in B (size-independent properties)."""
    from esa.backends.thunder import thunder_scan
    torch.manual_seed(0)
    shp = (32, 4096, 16, 64)
    A = torch.sigmoid(torch.randn(shp, device=DEV, dtype=torch.float32) * 2 + 2).to(dtype)
    B = torch.randn(shp, device=DEV, dtype=torch.float32).to(dtype)
    for compass in (16, 32, 64):
        E = thunder_scan(A, B, compass=compass)
        # channels sampled across heads, the first and last batch rows
        idx_b = torch.tensor([0, 13, 31])
        sub = (slice(None), slice(None), torch.tensor([0, 7, 15]))
        As = A[idx_b][:, :, [0, 7, 15]].cpu()
        Bs = B[idx_b][:, :, [0, 7, 15]].cpu()
        ref = oracle.scan_fwd(As.double(), Bs.double())
        assert rel(E[idx_b][:, :, [0, 7, 15]], ref) < TOL[dtype], compass
        del sub
    if dtype == torch.float32:
        B2 = torch.randn(shp, device=DEV)
        lhs = thunder_scan(A, B + B2)
        rhs = thunder_scan(A, B) + thunder_scan(A, B2)
        assert rel(lhs, rhs) < 1e-5


@pytest.mark.parametrize("shape,dtype,pinned", [
    ((6, 300, 4, 64), torch.float32, True),       # whole rows, several rows per chunk
    ((2, 9000, 4, 128), torch.float32, True),     # 18 MB rows: time pieces chained by e_last
    ((3, 40000, 2, 64), torch.bfloat16, True),    # bf16 time pieces with a ragged last piece
    ((5, 77, 3, 16), torch.float64, False),       # pageable host memory
])
def test_host_pipelined_scan(shape, dtype, pinned):
    """thunder_scan_host: CPU tensors in, CPU tensor out, chunks streamed
    through the device; equals the oracle on the same inputs."""
    from esa.backends.thunder import thunder_scan_host
    g = torch.Generator().manual_seed(7)
    A = torch.sigmoid(torch.randn(shape, generator=g, dtype=torch.float64) + 2.5).to(dtype)
    B = (torch.randn(shape, generator=g, dtype=torch.float64) * 0.5).to(dtype)
    if pinned:
        A, B = A.pin_memory(), B.pin_memory()
    E = thunder_scan_host(A, B, compass=16)
    assert E.device.type == "cpu" and E.dtype == dtype and E.shape == A.shape
    ref = oracle.scan_fwd(A.double(), B.double())
    assert rel(E, ref) < TOL[dtype]
    # into a caller's buffer (pageable): same result within the bar (the
    # time-parallel kernel's association order may differ from call to call)
    out = torch.empty_like(E)
    assert thunder_scan_host(A, B, out=out) is out
    assert rel(out, ref) < TOL[dtype]
