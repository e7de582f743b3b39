"""The CPU oracle against fixtures produced by running the reference package.

These pin the oracle: each fixture came from the reference's own functions
(tests/golden/make_golden.py), so agreement here means the oracle restates
the reference's algorithm.
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import oracle


def _load(name):
    return np.load(GOLDEN / name)


def _bf16(a):
    return torch.from_numpy(a).view(torch.bfloat16)


def test_scan_fwd_matches_reference_lifecycle_case():
    z = _load("scan_lifecycle.npz")
    E = oracle.scan_fwd(z["A"].astype(np.float64), z["B"].astype(np.float64))
    np.testing.assert_array_equal(E, z["pulse_f64"])
    np.testing.assert_allclose(E, z["pulse_f32"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(E, z["thunder_c4_f32"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", ["t1", "t9", "t33_hd15", "t130", "t64_hd1024"])
def test_scan_fwd_matches_reference_shapes(name):
    z = _load("scan_shapes.npz")
    E = oracle.scan_fwd(z[f"{name}_A"], z[f"{name}_B"])
    np.testing.assert_array_equal(E, z[f"{name}_pulse_f64"])
    ref32 = z[f"{name}_pulse_f32"].astype(np.float64)
    assert np.linalg.norm(E - ref32) / max(np.linalg.norm(E), 1e-30) < 1e-6


@pytest.mark.parametrize("name", ["t1", "t9", "t33_hd15", "t130", "t64_hd1024"])
def test_thunder_port_matches_reference_thunder(name):
    z = _load("scan_shapes.npz")
    A = torch.from_numpy(z[f"{name}_A"]).float()
    B = torch.from_numpy(z[f"{name}_B"]).float()
    got = oracle.thunder_scan_port(A, B, compass=16).numpy()
    np.testing.assert_allclose(got, z[f"{name}_thunder_c16_f32"], rtol=1e-6, atol=1e-6)
    # and the half-precision reference rounding is reproduced too
    got16 = oracle.thunder_scan_port(A.half(), B.half(), compass=16).float().numpy()
    np.testing.assert_allclose(got16, z[f"{name}_thunder_c16_f16"].astype(np.float32),
                               rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("name", ["g1", "g2"])
def test_scan_rev_matches_reference_autograd(name):
    z = _load("scan_grad.npz")
    E = oracle.scan_fwd(z[f"{name}_A"], z[f"{name}_B"])
    np.testing.assert_allclose(E, z[f"{name}_E"], rtol=0, atol=1e-13)
    dA, dB, _ = oracle.scan_rev(z[f"{name}_A"], E, z[f"{name}_dE"])
    np.testing.assert_allclose(dB, z[f"{name}_dB"], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dA, z[f"{name}_dA"], rtol=1e-12, atol=1e-12)


def test_scan_with_initial_state_is_composition():
    rng = np.random.default_rng(3)
    A = rng.uniform(0.8, 0.99, (2, 40, 3, 4))
    B = rng.normal(size=A.shape)
    full = oracle.scan_fwd(A, B)
    head = oracle.scan_fwd(A[:, :17], B[:, :17])
    tail = oracle.scan_fwd(A[:, 17:], B[:, 17:], e0=head[:, -1])
    np.testing.assert_allclose(np.concatenate([head, tail], 1), full, rtol=1e-13, atol=1e-13)
    # gradient w.r.t. the initial state equals the gradient flowing into E[:, 16]
    dE = rng.normal(size=A.shape)
    dA_full, dB_full, _ = oracle.scan_rev(A, full, dE)
    dA_t, dB_t, de0 = oracle.scan_rev(A[:, 17:], tail, dE[:, 17:], e0=head[:, -1])
    np.testing.assert_allclose(dA_t, dA_full[:, 17:], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(de0.reshape(2, 3, 4), dB_full[:, 16] - dE[:, 16],
                               rtol=1e-12, atol=1e-12)


def test_gate_bwd_matches_autograd():
    g = torch.randn(1000, dtype=torch.float64, requires_grad=True)
    v = torch.randn(1000, dtype=torch.float64, requires_grad=True)
    A = 0.8 + (0.995 - 0.8) * torch.sigmoid(g)
    Bw = (1 - A) * torch.tanh(v)
    dA, dB = torch.randn(1000, dtype=torch.float64), torch.randn(1000, dtype=torch.float64)
    torch.autograd.backward([A, Bw], [dA, dB])
    dg, dv = oracle.gate_bwd(g, v, dA, dB)
    np.testing.assert_allclose(dg, g.grad.numpy(), rtol=1e-12, atol=1e-14)
    np.testing.assert_allclose(dv, v.grad.numpy(), rtol=1e-12, atol=1e-14)
    A2, B2 = oracle.gate(g, v)
    np.testing.assert_allclose(A2, A.detach().numpy(), rtol=1e-15, atol=0)
    np.testing.assert_allclose(B2, Bw.detach().numpy(), rtol=1e-14, atol=1e-16)


def test_layer_restatement_matches_reference_pulse_fp64():
    z = _load("layer_pulse.npz")
    x = torch.from_numpy(z["x"]).double().requires_grad_(True)
    qw = torch.from_numpy(z["qgv_w"]).double().requires_grad_(True)
    ow = torch.from_numpy(z["out_w"]).double().requires_grad_(True)
    y = oracle.pulse_layer_forward(x, qw, ow, head=4)
    y.sum().backward()
    for got, key in ((y, "y"), (x.grad, "dx"), (qw.grad, "dqgv"), (ow.grad, "dout")):
        ref = z[f"pulse_fp64_{key}"]
        err = np.linalg.norm(got.detach().numpy() - ref) / np.linalg.norm(ref)
        assert err < 1e-12, (key, err)


def test_lightning_step_matches_reference_decode():
    z = _load("decode.npz")
    qw = z["qgv_w"].astype(np.float64)
    state = z["state_prefill"].astype(np.float64).reshape(3, 64)
    for i in range(5):
        qgv = z["x_steps"][i].astype(np.float64) @ qw.T
        state, zz = oracle.lightning_step(qgv, state)
        y = zz @ z["out_w"].astype(np.float64).T
        np.testing.assert_allclose(state.reshape(3, 4, 16), z["state_steps"][i], rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(y, z["y_steps"][i], rtol=1e-4, atol=1e-6)


def test_readout_matches_layer_formula():
    rng = np.random.default_rng(0)
    q, E = rng.normal(size=(5, 7, 32)), rng.normal(size=(5, 7, 32))
    z = oracle.readout(q, E)
    ref = (1 / (1 + np.exp(-q))) * E / np.sqrt((E ** 2).mean(-1, keepdims=True) + 1e-5)
    np.testing.assert_allclose(z, ref, rtol=1e-13)
