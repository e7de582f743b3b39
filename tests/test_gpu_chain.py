"""Parity of the scan on few-channel, long-time-axis problems.

With few channels per batch row the strips cannot fill the GPU, so the time
axis is cut across CTAs: below 8192 steps by the time-parallel look-back scan
(per-tile aggregates, a decoupled look-back over earlier tiles, outputs from
the exact incoming state), from 8192 steps by the single-pass chained scan
(plain forward of 16- and 32-bit data: time pieces read once, chained by a
per-warp look-back, re-read from L2 for the outputs) or the split scan (every
other kind: time pieces as strip rows, summary pass, composition of the
pieces' incoming states, output pass).  These shapes (a few strips' worth of channels, thousands of steps)
exercise both in every kind, with initial and final states, and the host
pipeline's time pieces.
Same bar as the other scan tests: relative Frobenius error against the fp64
oracle on the same rounded inputs -- 1e-5 fp32, 2e-3 fp16/bf16, 1e-12 fp64.
"""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 2e-3, torch.float64: 1e-12}
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


def _inputs(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    A = torch.sigmoid(torch.randn(shape, generator=g, dtype=torch.float64) + 3).to(dtype)
    B = (torch.randn(shape, generator=g, dtype=torch.float64) * 0.5).to(dtype)
    return A, B, g


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16, torch.float64])
@pytest.mark.parametrize("shape", [(2, 8192, 2, 64), (1, 12345, 3, 32), (3, 5000, 1, 256)])
def test_chained_forward_with_states(dtype, shape):
    from esa import ops
    A, B, g = _inputs(shape, dtype, 11)
    nb, T, H, D = shape
    e0 = torch.randn(nb, H * D, generator=g, dtype=torch.float64)
    acc = torch.float64 if dtype == torch.float64 else torch.float32
    E, e_last = ops.scan(A.to(DEV), B.to(DEV), e0.to(acc).to(DEV), 16)
    ref = oracle.scan_fwd(A.double(), B.double(), e0=e0.to(acc).double())
    assert rel(E, ref) < TOL[dtype]
    assert rel(e_last, ref[:, -1].reshape(nb, H * D)) < TOL[dtype]
    # zero initial state, every chunking of the call gives the same E
    E0, _ = ops.scan(A.to(DEV), B.to(DEV), None, 64)
    assert rel(E0, oracle.scan_fwd(A.double(), B.double())) < TOL[dtype]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(2, 8192, 2, 64), (1, 12345, 3, 32), (2, 9000, 3, 64), (3, 20000, 1, 8)])
def test_single_pass_chained_scan(dtype, shape):
    """The plain forward of few channels over >= 8192 steps runs the
    single-pass chained kernel: with an initial state, a ragged last piece and
    last tile (T = 12345, 9000, 20000), a partial last strip (96 and 192
    channels against 128-channel strips, 8 against 64) and several batch rows."""
    from esa import _lib, ops
    A, B, g = _inputs(shape, dtype, 21)
    nb, T, H, D = shape
    e0 = torch.randn(nb, H * D, generator=g, dtype=torch.float64).float()
    E, e_last = ops.scan(A.to(DEV), B.to(DEV), e0.to(DEV), 16)
    assert _lib.last_scan_path() == "chain"
    ref = oracle.scan_fwd(A.double(), B.double(), e0=e0.double())
    assert rel(E, ref) < TOL[dtype]
    assert rel(e_last, ref[:, -1].reshape(nb, H * D)) < TOL[dtype]
    # a second call (tickets and flags reset per launch) agrees to rounding:
    # how many predecessor aggregates a look-back composes before it meets an
    # inclusive prefix depends on timing, so the last bits may differ
    E2, _ = ops.scan(A.to(DEV), B.to(DEV), e0.to(DEV), 16)
    assert rel(E2, E.double().cpu().numpy()) < TOL[dtype] / 10


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float64])
def test_chained_reverse_with_states(dtype):
    from esa import ops
    shape = (2, 6000, 2, 64)
    A, B, g = _inputs(shape, dtype, 12)
    nb, T, H, D = shape
    acc = torch.float64 if dtype == torch.float64 else torch.float32
    e0 = torch.randn(nb, H * D, generator=g, dtype=torch.float64).to(acc)
    Ad = A.to(DEV).requires_grad_(True)
    Bd = B.to(DEV).requires_grad_(True)
    e0d = e0.to(DEV).requires_grad_(True)
    E, _ = ops.scan(Ad, Bd, e0d, 16)
    dE = torch.randn(shape, generator=g, dtype=torch.float64).to(dtype)
    E.backward(dE.to(DEV))
    dA_ref, dB_ref, de0_ref = oracle.scan_rev(A.double(), E.detach().double().cpu(), dE.double(),
                                              e0=e0.double())
    assert rel(Bd.grad, dB_ref) < TOL[dtype]
    assert rel(Ad.grad, dA_ref) < TOL[dtype]
    assert rel(e0d.grad, de0_ref) < TOL[dtype]


@pytest.mark.parametrize("raw_dtype,scan_dtype", [
    (torch.float32, torch.float32), (torch.float16, torch.float16), (torch.bfloat16, torch.float32)])
def test_chained_gated_fwd_bwd(raw_dtype, scan_dtype):
    from esa import ops
    g = torch.Generator().manual_seed(13)
    Bsz, T, C = 2, 7000, 128
    qgv = torch.randn(Bsz, T, 3 * C, generator=g).to(raw_dtype)
    gr, vr = qgv[..., C:2 * C], qgv[..., 2 * C:]
    qd = qgv.to(DEV)
    grd, vrd = qd[..., C:2 * C], qd[..., 2 * C:]
    E, _ = ops.gated_scan(grd, vrd, None, 0.8, 0.995, 16, scan_dtype)
    A64, B64 = oracle.gate(gr, vr)
    Ar = torch.from_numpy(A64).to(scan_dtype).double()
    Br = torch.from_numpy(B64).to(scan_dtype).double()
    ref = oracle.scan_fwd(Ar.reshape(Bsz, T, 1, C), Br.reshape(Bsz, T, 1, C)).reshape(Bsz, T, C)
    tol = max(TOL[scan_dtype], TOL[raw_dtype])
    assert rel(E, ref) < tol
    dE = torch.randn(Bsz, T, C, generator=g).to(scan_dtype)
    dg, dv, _ = ops.gated_scan_backward(grd, vrd, E, dE.to(DEV), None, 0.8, 0.995, 16)
    dA, dB, _ = oracle.scan_rev(Ar.reshape(Bsz, T, 1, C), E.double().cpu().reshape(Bsz, T, 1, C),
                                dE.double().reshape(Bsz, T, 1, C))
    dg_ref, dv_ref = oracle.gate_bwd(gr, vr, dA.reshape(Bsz, T, C), dB.reshape(Bsz, T, C))
    assert rel(dg, dg_ref) < tol * 2
    assert rel(dv, dv_ref) < tol * 2


def test_chained_long_sequence_properties():
    """Long-sequence size [4, 262144, 32, 64] bf16 (the single-pass chained
    kernel): sampled channels against the oracle (fp64 on the same rounded
    inputs) and the end state against the slice summary, which the split
    summary pass computes on its own (size-independent checks)."""
    from esa import _lib, ops
    torch.manual_seed(0)
    shp = (4, 262144, 32, 64)
    dev = torch.device(DEV)
    A = torch.sigmoid(torch.randn(shp, device=dev) + 3).to(torch.bfloat16)
    B = (torch.randn(shp, device=dev) * 0.5).to(torch.bfloat16)
    E, e_last = ops.scan(A, B, None, 16)
    assert _lib.last_scan_path() == "chain"
    # channels of two heads of rows 0 and 3, over the first and the last 4096 steps
    for rows in (slice(0, 1), slice(3, 4)):
        for ts in (slice(0, 4096), slice(shp[1] - 4096, shp[1])):
            As = A[rows, :, 5].double().cpu()
            Bs = B[rows, :, 5].double().cpu()
            ref = oracle.scan_fwd(As.unsqueeze(2).numpy(), Bs.unsqueeze(2).numpy())[:, ts, 0]
            assert rel(E[rows, ts, 5].double(), ref) < 2e-3
    # the end state equals the summary of the whole sequence
    e_end, prod = ops.scan_summary(A, B, None)
    assert rel(e_last, e_end) < 1e-4
    del prod


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_split_reverse_with_states(dtype):
    """T >= 8192 with few channels: the reverse scan runs split into time
    pieces (summary pass, composition in descending time, output pass)."""
    from esa import ops
    shape = (2, 10000, 2, 64)
    A, B, g = _inputs(shape, dtype, 14)
    nb, T, H, D = shape
    e0 = torch.randn(nb, H * D, generator=g, dtype=torch.float64).float()
    Ad = A.to(DEV).requires_grad_(True)
    Bd = B.to(DEV).requires_grad_(True)
    e0d = e0.to(DEV).requires_grad_(True)
    E, _ = ops.scan(Ad, Bd, e0d, 16)
    dE = torch.randn(shape, generator=g, dtype=torch.float64).to(dtype)
    E.backward(dE.to(DEV))
    dA_ref, dB_ref, de0_ref = oracle.scan_rev(A.double(), E.detach().double().cpu(), dE.double(),
                                              e0=e0.double())
    assert rel(Bd.grad, dB_ref) < TOL[dtype]
    assert rel(Ad.grad, dA_ref) < TOL[dtype]
    assert rel(e0d.grad, de0_ref) < TOL[dtype]


@pytest.mark.parametrize("raw_dtype,scan_dtype", [(torch.float32, torch.float32), (torch.float16, torch.float16)])
def test_split_gated_fwd_bwd(raw_dtype, scan_dtype):
    """Fused gated scans split into time pieces (T = 9000, 128 channels): the
    summary passes run the gate prologue, the reverse one in descending time."""
    from esa import ops
    g = torch.Generator().manual_seed(15)
    Bsz, T, C = 1, 9000, 128
    qgv = torch.randn(Bsz, T, 3 * C, generator=g).to(raw_dtype)
    gr, vr = qgv[..., C:2 * C], qgv[..., 2 * C:]
    qd = qgv.to(DEV)
    grd, vrd = qd[..., C:2 * C], qd[..., 2 * C:]
    e0 = torch.randn(Bsz, C, generator=g).to(DEV)
    E, e_last = ops.gated_scan(grd, vrd, e0, 0.8, 0.995, 16, scan_dtype)
    A64, B64 = oracle.gate(gr, vr)
    Ar = torch.from_numpy(A64).to(scan_dtype).double()
    Br = torch.from_numpy(B64).to(scan_dtype).double()
    ref = oracle.scan_fwd(Ar.reshape(Bsz, T, 1, C), Br.reshape(Bsz, T, 1, C),
                          e0=e0.double().cpu().reshape(Bsz, 1, C)).reshape(Bsz, T, C)
    tol = max(TOL[scan_dtype], TOL[raw_dtype])
    assert rel(E, ref) < tol
    assert rel(e_last, ref[:, -1]) < tol
    dE = torch.randn(Bsz, T, C, generator=g).to(scan_dtype)
    dg, dv, de0 = ops.gated_scan_backward(grd, vrd, E, dE.to(DEV), e0, 0.8, 0.995, 16)
    dA, dB, de0_ref = oracle.scan_rev(Ar.reshape(Bsz, T, 1, C), E.double().cpu().reshape(Bsz, T, 1, C),
                                      dE.double().reshape(Bsz, T, 1, C),
                                      e0=e0.double().cpu().reshape(Bsz, 1, C))
    dg_ref, dv_ref = oracle.gate_bwd(gr, vr, dA.reshape(Bsz, T, C), dB.reshape(Bsz, T, C))
    assert rel(dg, dg_ref) < tol * 2
    assert rel(dv, dv_ref) < tol * 2
    assert rel(de0, de0_ref.reshape(Bsz, C)) < tol * 2


def test_host_pipeline_time_pieces_with_split():
    """A 72 MB row: the host pipeline cuts it into time pieces chained through
    their end states, and each piece (65536 steps, 128 channels) is itself
    scanned split."""
    from esa.backends.thunder import thunder_scan_host
    A, B, _ = _inputs((1, 140000, 2, 64), torch.float32, 16)
    A, B = A.pin_memory(), B.pin_memory()
    E = thunder_scan_host(A, B)
    ref = oracle.scan_fwd(A.double(), B.double())
    assert rel(E, ref) < TOL[torch.float32]
