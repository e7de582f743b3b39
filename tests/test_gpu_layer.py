"""Layer, prefill, Lightning decode and ESAModel parity on the GPU.

Same rel-Frobenius bar as the scan tests (1e-5 fp32, 2e-3 fp16/bf16 against an
fp64 oracle); greedy token ids must be identical to the reference's in fp32.
"""
import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel(got, ref) -> float:
    got = np.asarray(got.detach().double().cpu() if torch.is_tensor(got) else got, dtype=np.float64)
    ref = np.asarray(ref.detach().double().cpu() if torch.is_tensor(ref) else ref, dtype=np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-300))


@pytest.fixture(autouse=True)
def _status_clean():
    yield
    from esa import ops
    torch.cuda.synchronize()
    ops.check_device_status()


def _layer_from_fixture(backend, precision, dtype):
    from esa import ESA
    z = np.load(GOLDEN / "layer_pulse.npz")
    lay = ESA(embd=128, head=4, backend=backend, precision=precision, device=DEV).to(dtype)
    lay.load_state_dict({"layer.qgv.weight": torch.from_numpy(z["qgv_w"]).to(dtype),
                         "layer.out_proj.weight": torch.from_numpy(z["out_w"]).to(dtype)})
    return lay, z


@pytest.mark.parametrize("backend", ["thunder", "pulse", "flare"])
@pytest.mark.parametrize("precision,dtype,tol", [("fp64", torch.float64, 1e-11),
                                                 ("fp32", torch.float32, 1e-5)])
def test_layer_forward_backward_vs_reference_pulse(backend, precision, dtype, tol):
    lay, z = _layer_from_fixture(backend, precision, dtype)
    x = torch.from_numpy(z["x"]).to(dtype).to(DEV).requires_grad_(True)
    y = lay(x)
    y.sum().backward()
    ref = "pulse_fp64"
    assert rel(y, z[f"{ref}_y"]) < tol
    assert rel(x.grad, z[f"{ref}_dx"]) < tol
    assert rel(lay.layer.qgv.weight.grad, z[f"{ref}_dqgv"]) < tol
    assert rel(lay.layer.out_proj.weight.grad, z[f"{ref}_dout"]) < tol
    if precision == "fp32":
        # the reference's own thunder fp32 forward on the same weights
        assert rel(y, z["thunder_fp32_y"]) < tol


@pytest.mark.parametrize("precision,scan_dtype", [("fp16", torch.float16), ("bf16", torch.bfloat16)])
def test_layer_half_precision_scan(precision, scan_dtype):
    """fp32 activations, 16-bit scan (the reference's default fp16 mode):
    E against the fp64 oracle on A, B rounded to the scan dtype."""
    lay, z = _layer_from_fixture("thunder", precision, torch.float32)
    x = torch.from_numpy(z["x"]).float().to(DEV)
    with torch.no_grad():
        qgv = lay.layer.qgv(x)
    from esa import ops
    E, _ = ops.gated_scan(qgv[..., 128:256], qgv[..., 256:], None, 0.8, 0.995, 16, scan_dtype)
    A64, B64 = oracle.gate(qgv[..., 128:256].cpu(), qgv[..., 256:].cpu())
    Ar = torch.from_numpy(A64).to(scan_dtype).double().reshape(2, 96, 1, 128)
    Br = torch.from_numpy(B64).to(scan_dtype).double().reshape(2, 96, 1, 128)
    ref = oracle.scan_fwd(Ar, Br).reshape(2, 96, 128)
    assert rel(E, ref) < 2e-3
    y = lay(x)
    y64 = oracle.pulse_layer_forward(torch.from_numpy(z["x"]).double(),
                                     torch.from_numpy(z["qgv_w"]).double(),
                                     torch.from_numpy(z["out_w"]).double(), head=4)
    assert rel(y, y64) < 2e-2  # includes the A/B rounding to 16 bits, as in the reference


def test_layer_config1_full_size_fp32():
    """ESA layer at embd=128, head=4, batch=16, block=1024, fp32: forward and
    backward of sum(y) against the fp64 oracle with identical weights."""
    from esa import ESA
    torch.manual_seed(1234)
    lay = ESA(embd=128, head=4, batch=16, block=1024, backend="thunder", precision="fp32",
              dropout=0.0, device=DEV)
    x = torch.randn(16, 1024, 128, generator=torch.Generator().manual_seed(1234))
    xd = x.to(DEV).requires_grad_(True)
    y = lay(xd)
    y.sum().backward()
    qw = lay.layer.qgv.weight.detach().cpu().double().requires_grad_(True)
    ow = lay.layer.out_proj.weight.detach().cpu().double().requires_grad_(True)
    x64 = x.double().requires_grad_(True)
    y64 = oracle.pulse_layer_forward(x64, qw, ow, head=4)
    y64.sum().backward()
    assert rel(y, y64) < 1e-5
    assert rel(xd.grad, x64.grad) < 1e-5
    assert rel(lay.layer.qgv.weight.grad, qw.grad) < 1e-5
    assert rel(lay.layer.out_proj.weight.grad, ow.grad) < 1e-5


def test_prefill_and_decode_vs_reference():
    from esa import ESA
    z = np.load(GOLDEN / "decode.npz")
    lay = ESA(embd=64, head=4, backend="pulse", precision="fp32", device=DEV)
    lay.load_state_dict({"layer.qgv.weight": torch.from_numpy(z["qgv_w"]),
                         "layer.out_proj.weight": torch.from_numpy(z["out_w"])})
    lay.eval()
    xp = torch.from_numpy(z["x_prompt"]).to(DEV)
    assert rel(lay(xp), z["y_forward"]) < 1e-5
    y_pre, state = lay.prefill(xp)
    assert rel(y_pre, z["y_prefill"]) < 1e-5
    assert rel(state, z["state_prefill"]) < 1e-5
    s = state
    for i in range(5):
        y1, s = lay.decode_step(torch.from_numpy(z["x_steps"][i]).to(DEV), s)
        assert y1.shape == (3, 64) and s.shape == (3, 4, 16)
        assert rel(y1, z["y_steps"][i]) < 1e-5
        assert rel(s, z["state_steps"][i]) < 1e-5
    # flat state layout and [B,1,C] input keep their shapes
    y3, s3 = lay.decode_step(torch.from_numpy(z["x_steps"][0]).to(DEV)[:, None], state.reshape(3, 64))
    assert y3.shape == (3, 1, 64) and s3.shape == (3, 64)


def test_prefill_engines_agree():
    """thunder_16 prefill state == exact-recurrence ('lightning') state
    (reference tests/test_optimized_defaults.py:54-80), and prefill with an
    explicit state continues a split prompt exactly."""
    from esa import ESAModel, ESAModelConfig
    torch.manual_seed(1)
    model = ESAModel(ESAModelConfig(vocab_size=32, block=32, n_layer=2, head=4, embd=32,
                                    dropout=0.0, precision="fp32"), device=DEV)
    ids = torch.randint(0, 32, (1, 9), device=DEV)
    _, s_thunder, _ = model.prefill(ids, engine="thunder_16")
    _, s_light, _ = model.prefill(ids, engine="lightning")
    torch.testing.assert_close(s_thunder, s_light)
    from esa import ESA
    lay = ESA(embd=64, head=4, precision="fp32", device=DEV)
    x = torch.randn(2, 40, 64, device=DEV)
    y_full, s_full = lay.prefill(x)
    y_a, s_a = lay.prefill(x[:, :17])
    y_b, s_b = lay.prefill(x[:, 17:], state=s_a)
    assert rel(torch.cat([y_a, y_b], 1), y_full) < 1e-5
    assert rel(s_b, s_full) < 1e-5


@pytest.mark.parametrize("prefill", ["thunder_16", "pulse"])
@pytest.mark.parametrize("decode_graph", [False, True])
def test_model_greedy_ids_bit_identical(prefill, decode_graph):
    """Greedy ids in fp32 equal the reference's on the same weights."""
    from esa import ESAModel, ESAModelConfig
    z = np.load(GOLDEN / "model_generate.npz")
    cfg = ESAModelConfig(vocab_size=64, block=32, n_layer=2, head=4, embd=32, dropout=0.0,
                         precision="fp32", backend="thunder")
    model = ESAModel(cfg, device=DEV)
    sd = {k[4:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("sd::")}
    model.load_state_dict(sd, strict=True)
    model.eval()
    ids = torch.from_numpy(z["ids"]).to(DEV)
    logits, _ = model(ids)
    assert rel(logits, z["logits"]) < 1e-5
    seq = model.generate(input_ids=ids, seek=12, prefill=prefill, compile=False, temperature=0.0,
                         decode_graph=decode_graph)
    assert torch.equal(seq.cpu(), torch.from_numpy(z[f"seq_{prefill}"]))


def test_model_training_step_runs_and_matches_eager():
    from esa import ESAModel, ESAModelConfig
    torch.manual_seed(0)
    cfg = ESAModelConfig(vocab_size=128, block=64, n_layer=2, head=4, embd=64, dropout=0.0,
                         precision="fp32", training_compile=False)
    model = ESAModel(cfg, device=DEV)
    ids = torch.randint(0, 128, (2, 64), device=DEV)
    logits, loss = model(ids, ids)
    loss.backward()
    grads = [p.grad for p in model.parameters() if p.requires_grad]
    assert all(g is not None and torch.isfinite(g).all() for g in grads)
