"""The ESA layer core entry points esa_layer_fwd / esa_layer_bwd (gated scan
then RMS readout; readout backward then reverse gated scan) with initial and
final states, through the C ABI and through the torch custom op.

Parity bar as everywhere: relative Frobenius error against the fp64 oracle on
the same rounded inputs -- 1e-5 fp32, 2e-3 for 16-bit outputs (4e-3 for the
gate gradients, products of two rounded quantities, as in test_gpu_scan.py).
The readout is checked on the kernel's own (rounded) E, the state it reads.
"""
import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
F16, BF16, F32 = torch.float16, torch.bfloat16, torch.float32
TOL = {F32: 1e-5, F16: 2e-3, BF16: 2e-3}
GMIN, GMAX, EPS = 0.8, 0.995, 1e-5

# (nb, T, C, qgv dtype, scan dtype, y dtype)
CASES = [
    (4, 2048, 768, F16, F16, F16),      # the ESAModel training layer's width
    (3, 1000, 768, BF16, BF16, BF16),   # ragged last tile
    (16, 1024, 128, F32, F32, F32),     # the single-layer workload
    (2, 777, 1024, F16, F16, F16),
    (5, 333, 192, F32, F16, F32),       # fp32 activations, 16-bit scan
    (1, 40, 64, F32, F32, F32),         # short single sequence
    (2, 300, 96, F32, F32, F32),        # C not a multiple of 64
    (8, 500, 2048, F16, F16, F16),      # 256 strips of 64 channels
]


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


def _case_id(c):
    nb, T, C, q, e, y = c
    n = {F16: "f16", BF16: "bf16", F32: "f32"}
    return f"{nb}x{T}x{C}-{n[q]}-{n[e]}-{n[y]}"


def _inputs(case, seed):
    nb, T, C, qdt, edt, ydt = case
    g = torch.Generator().manual_seed(seed)
    qgv = (torch.randn(nb, T, 3 * C, generator=g) * 1.5).to(qdt)
    e0 = torch.randn(nb, C, generator=g) * 0.5
    return qgv, e0


def _rounded_gate(qgv, C, edt):
    A64, B64 = oracle.gate(qgv[..., C:2 * C], qgv[..., 2 * C:], GMIN, GMAX)
    Ar = torch.from_numpy(A64).to(edt).double()
    Br = torch.from_numpy(B64).to(edt).double()
    return Ar, Br


def _fwd(case, qgv, e0):
    from esa import _lib, ops
    nb, T, C, qdt, edt, ydt = case
    L = _lib.lib()
    qd = qgv.to(DEV)
    E = torch.empty(nb, T, C, dtype=edt, device=DEV)
    y = torch.empty(nb, T, C, dtype=ydt, device=DEV)
    rstd = torch.empty(nb * T, dtype=torch.float32, device=DEV)
    e0d = e0.to(DEV)
    e_last = torch.empty(nb, C, device=DEV)
    ws = ops._layer_workspace(nb, T, C, qdt, edt, ydt, DEV)
    _lib.check(L.esa_layer_fwd(qd.data_ptr(), 3 * C, ops.dtype_code(qdt), E.data_ptr(), ops.dtype_code(edt),
                               y.data_ptr(), ops.dtype_code(ydt), rstd.data_ptr(), nb, T, C, GMIN, GMAX, EPS,
                               e0d.data_ptr(), e_last.data_ptr(), ws.data_ptr(), ws.numel(),
                               torch.cuda.current_stream().cuda_stream), "esa_layer_fwd")
    path = _lib.last_scan_path()
    torch.cuda.synchronize()
    return E, y, rstd, e_last, path


@pytest.mark.parametrize("case", CASES, ids=_case_id)
def test_layer_forward_matches_oracle(case):
    nb, T, C, qdt, edt, ydt = case
    qgv, e0 = _inputs(case, 1)
    E, y, rstd, e_last, path = _fwd(case, qgv, e0)
    assert path in ("strip", "lane", "lookback", "sequential")
    Ar, Br = _rounded_gate(qgv, C, edt)
    ref = oracle.scan_fwd(Ar.reshape(nb, T, 1, C), Br.reshape(nb, T, 1, C), e0.double()).reshape(nb, T, C)
    tol = TOL[edt]
    assert rel(E, ref) < tol
    assert rel(e_last, ref[:, -1]) < tol
    Ek = E.double().cpu()
    r_ref = 1.0 / np.sqrt((Ek.numpy() ** 2).mean(axis=-1) + EPS)
    assert rel(rstd.reshape(nb, T), r_ref) < 1e-5
    y_ref = oracle.readout(qgv[..., :C].double(), Ek, EPS)
    assert rel(y, y_ref) < max(TOL[ydt], 1e-5)


@pytest.mark.parametrize("case", CASES, ids=_case_id)
def test_layer_backward_matches_oracle(case):
    from esa import _lib, ops
    nb, T, C, qdt, edt, ydt = case
    qgv, e0 = _inputs(case, 2)
    E, y, rstd, _, _ = _fwd(case, qgv, e0)
    g = torch.Generator().manual_seed(3)
    dy = torch.randn(nb, T, C, generator=g).to(ydt)
    dqgv = torch.empty(nb, T, 3 * C, dtype=qdt, device=DEV)
    de0 = torch.empty(nb, C, device=DEV)
    L = _lib.lib()
    qd = qgv.to(DEV)
    dyd = dy.to(DEV)
    e0d = e0.to(DEV)
    ws = ops._layer_workspace(nb, T, C, qdt, edt, ydt, DEV)
    _lib.check(L.esa_layer_bwd(dyd.data_ptr(), ops.dtype_code(ydt), qd.data_ptr(), 3 * C, ops.dtype_code(qdt),
                               E.data_ptr(), ops.dtype_code(edt), rstd.data_ptr(), dqgv.data_ptr(), 3 * C, nb, T,
                               C, GMIN, GMAX, EPS, e0d.data_ptr(), de0.data_ptr(), ws.data_ptr(), ws.numel(),
                               torch.cuda.current_stream().cuda_stream), "esa_layer_bwd")
    torch.cuda.synchronize()
    Ek = E.double().cpu()
    dq_ref, dE_ref = oracle.readout_bwd(qgv[..., :C].double(), Ek, rstd.double().cpu().reshape(nb, T), dy.double())
    Ar, _ = _rounded_gate(qgv, C, edt)
    dA, dB, de0_ref = oracle.scan_rev(Ar.reshape(nb, T, 1, C), Ek.reshape(nb, T, 1, C),
                                      dE_ref.reshape(nb, T, 1, C), e0=e0.double())
    dg_ref, dv_ref = oracle.gate_bwd(qgv[..., C:2 * C], qgv[..., 2 * C:], dA.reshape(nb, T, C),
                                     dB.reshape(nb, T, C), GMIN, GMAX)
    tol = max(TOL[qdt], TOL[edt])
    assert rel(dqgv[..., :C], dq_ref) < tol
    assert rel(dqgv[..., C:2 * C], dg_ref) < 2 * tol
    assert rel(dqgv[..., 2 * C:], dv_ref) < 2 * tol
    assert rel(de0, de0_ref.reshape(nb, C)) < 2 * tol


def test_layer_core_autograd_training_shape():
    """The autocast training layer [16, 2048, 768] fp16 through the custom op
    and torch autograd: E, y and d qgv on three batch rows against the oracle."""
    from esa import ops
    nb, T, C = 16, 2048, 768
    g = torch.Generator().manual_seed(4)
    qgv = torch.randn(nb, T, 3 * C, generator=g).half()
    dy = torch.randn(nb, T, C, generator=g).half()
    qd = qgv.to(DEV).requires_grad_(True)
    y, E, rstd = ops.layer_core(qd, GMIN, GMAX, EPS, 16, F16, F16)
    y.backward(dy.to(DEV))
    rows = [0, 9, 15]
    q3 = qgv[rows]
    Ar, Br = _rounded_gate(q3, C, F16)
    ref = oracle.scan_fwd(Ar.reshape(3, T, 1, C), Br.reshape(3, T, 1, C)).reshape(3, T, C)
    assert rel(E[rows], ref) < 2e-3
    Ek = E[rows].double().cpu()
    assert rel(y[rows], oracle.readout(q3[..., :C].double(), Ek, EPS)) < 2e-3
    dq_ref, dE_ref = oracle.readout_bwd(q3[..., :C].double(), Ek, rstd.reshape(nb, T)[rows].double().cpu(),
                                        dy[rows].double())
    dA, dB, _ = oracle.scan_rev(Ar.reshape(3, T, 1, C), Ek.reshape(3, T, 1, C), dE_ref.reshape(3, T, 1, C))
    dg_ref, dv_ref = oracle.gate_bwd(q3[..., C:2 * C], q3[..., 2 * C:], dA.reshape(3, T, C), dB.reshape(3, T, C))
    gq = qd.grad[rows]
    assert rel(gq[..., :C], dq_ref) < 2e-3
    assert rel(gq[..., C:2 * C], dg_ref) < 4e-3
    assert rel(gq[..., 2 * C:], dv_ref) < 4e-3
