"""Parity of the fused readout kernels and of the fused layer core.

readout: y = sigmoid(q) * E * rsqrt(mean_C(E^2) + eps) (thunder.py:304-311).
The fused kernels compute in fp32 (fp64 for fp64 operands) with one rounding
per output; they are checked against the same math in fp64 torch on the same
rounded inputs, relative Frobenius error: 1e-6 fp32, 2e-3 fp16/bf16, 1e-12
fp64.  The layer core (gated scan + readout, fused backward into d qgv) is
checked against autograd through the unfused composition in fp64.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-6, torch.float16: 2e-3, torch.bfloat16: 2e-3, torch.float64: 1e-12}


def rel(got, ref) -> float:
    g = got.detach().double().cpu().numpy()
    r = ref.detach().double().cpu().numpy()
    assert g.shape == r.shape
    assert np.isfinite(g).all()
    return float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-300))


def _ref(q, E, eps):
    q, E = q.double(), E.double()
    r = torch.rsqrt(E.pow(2).mean(-1, keepdim=True) + eps)
    return torch.sigmoid(q) * E * r


@pytest.mark.parametrize("dt,C", [(torch.float32, 768), (torch.float16, 768), (torch.bfloat16, 256),
                                  (torch.float64, 64), (torch.float32, 100), (torch.float16, 36)])
def test_readout_forward_backward(dt, C):
    from esa import _lib, ops
    g = torch.Generator().manual_seed(21)
    nb, T, eps = 3, 50, 1e-5
    qgv = torch.randn(nb, T, 3 * C, generator=g, dtype=torch.float64).to(dt).cuda()
    q = qgv[..., :C]                                  # row stride 3C
    E = (torch.randn(nb, T, C, generator=g, dtype=torch.float64) * 0.3).to(dt).cuda()
    y = ops.readout(q, E, eps, dt)
    assert y.dtype == dt
    assert rel(y, _ref(q, E, eps)) < TOL[dt]
    # backward against autograd of the fp64 math
    qd = q.double().detach().requires_grad_(True)
    Ed = E.double().detach().requires_grad_(True)
    dy = torch.randn(nb, T, C, generator=g, dtype=torch.float64).to(dt).cuda()
    _ref(qd, Ed, eps).backward(dy.double())
    rows = nb * T
    rstd = torch.empty(rows, dtype=ops.acc_dtype(dt), device="cuda")
    y2 = torch.empty_like(E)
    L = _lib.lib()
    code = ops.dtype_code(dt)
    s = torch.cuda.current_stream().cuda_stream
    _lib.check(L.esa_readout_fwd(qgv.data_ptr(), 3 * C, code, E.data_ptr(), C, code, y2.data_ptr(), C, code,
                                 rstd.data_ptr(), rows, C, eps, s), "fwd")
    dqgv = torch.zeros_like(qgv)
    dE = torch.empty_like(E)
    _lib.check(L.esa_readout_bwd(dy.data_ptr(), C, code, qgv.data_ptr(), 3 * C, code, E.data_ptr(), C, code,
                                 rstd.data_ptr(), dqgv.data_ptr(), 3 * C, code, dE.data_ptr(), C, code,
                                 rows, C, eps, s), "bwd")
    torch.cuda.synchronize()
    assert torch.equal(y2, y)
    assert rel(dqgv[..., :C], qd.grad) < 2 * TOL[dt]
    assert rel(dE, Ed.grad) < 2 * TOL[dt]
    assert torch.count_nonzero(dqgv[..., C:]) == 0   # only the q third is written


@pytest.mark.parametrize("raw,scan", [(torch.float64, torch.float64), (torch.float32, torch.float32),
                                      (torch.float16, torch.float16), (torch.bfloat16, torch.float32)])
def test_layer_core_matches_unfused_autograd(raw, scan):
    """d qgv of the fused core against autograd through gated_scan + torch readout."""
    from esa import ops
    from esa.backends._layer import readout
    g = torch.Generator().manual_seed(22)
    nb, T, C, eps = 2, 300, 128, 1e-5
    base = torch.randn(nb, T, 3 * C, generator=g, dtype=torch.float64).to(raw).cuda()
    w = torch.randn(nb, T, C, generator=g, dtype=torch.float64).cuda()
    # fused
    qgv = base.clone().requires_grad_(True)
    y, _, _ = ops.layer_core(qgv, 0.8, 0.995, eps, 16, scan, raw)
    (y.double() * w).sum().backward()
    g_fused = qgv.grad.clone()
    # unfused
    qgv2 = base.clone().requires_grad_(True)
    q, gr, vr = qgv2.split(C, dim=-1)
    E, _ = ops.gated_scan(gr, vr, None, 0.8, 0.995, 16, scan)
    y2 = readout(q, E, eps, raw)
    (y2.double() * w).sum().backward()
    tol = {torch.float64: 1e-11, torch.float32: 1e-5}.get(raw, 5e-3)
    assert rel(y, y2) < tol
    assert rel(g_fused, qgv2.grad) < tol
