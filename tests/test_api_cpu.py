"""CPU-side checks: the drop-in API surface, argument validation, the C ABI
library (loads and exports every symbol include/esa_b200.h declares, without
calling compute), and that the product has no CPU fallback."""
import ctypes
import inspect
import re

import pytest
import torch

from conftest import ROOT

HEADER = ROOT / "include" / "esa_b200.h"


def _declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(esa_\w+)\s*\(", text, re.M)))


def test_header_declares_the_abi():
    syms = _declared_symbols()
    assert set(syms) == {
        "esa_abi_version", "esa_last_error", "esa_scan_last_path", "esa_device_status", "esa_scan_workspace_bytes",
        "esa_scan_fwd", "esa_scan_rev", "esa_gated_scan_fwd", "esa_gated_scan_bwd",
        "esa_lightning_step", "esa_scan_fwd_noalloc", "esa_scan_summary", "esa_scan_prod", "esa_scan_fixup",
        "esa_scan_host_staging_bytes", "esa_scan_fwd_host", "esa_scan_fwd_resume",
        "esa_wait_selftest", "esa_readout_fwd", "esa_readout_bwd", "esa_layer_norm_fwd",
        "esa_layer_norm_workspace_bytes", "esa_layer_norm_bwd", "esa_add_layer_norm_fwd",
        "esa_add_layer_norm_bwd", "esa_cross_entropy_fwd", "esa_cross_entropy_bwd",
        "esa_layer_workspace_bytes", "esa_layer_fwd", "esa_layer_bwd",
        "esa_decode_block_scratch_bytes", "esa_decode_block", "esa_decode_head"}


def test_decode_entry_points_reject_bad_arguments_without_device_work():
    """The fused decode kernels take 1..4 rows of fp16/bf16 data with C a
    multiple of 256; everything else is refused by the host checks."""
    from esa import _lib
    L = _lib.lib()
    assert L.esa_decode_block_scratch_bytes(1, 1024, _lib.DTYPE_F16) == 18 * 1024
    assert L.esa_decode_block_scratch_bytes(4, 1024, _lib.DTYPE_BF16) == 18 * 4 * 1024
    for nb, C, dt in ((0, 1024, _lib.DTYPE_F16), (5, 1024, _lib.DTYPE_F16), (1, 1000, _lib.DTYPE_F16),
                      (1, 1024, _lib.DTYPE_F32)):
        assert L.esa_decode_block_scratch_bytes(nb, C, dt) == 0
        rc = L.esa_decode_block(*([None] * 18), nb, C, dt, 0.8, 0.995, 1e-5, 1e-5, None, 0, None)
        assert rc != 0
        assert "decode" in _lib.last_error()
        rc = L.esa_decode_head(None, None, None, None, 1e-5, None, None, None, nb, C, 32000, dt, None)
        assert rc != 0
    # misaligned weight rows (the GEMVs read 16-byte vectors) are refused
    rc = L.esa_decode_head(16, None, 16, None, 1e-5, 18, None, 16, 1, 1024, 32000, _lib.DTYPE_F16, None)
    assert rc != 0 and "aligned" in _lib.last_error()
    # a valid shape without a scratch buffer is refused before any launch
    rc = L.esa_decode_block(*([None] * 18), 1, 1024, _lib.DTYPE_F16, 0.8, 0.995, 1e-5, 1e-5, None, 0, None)
    assert rc != 0 and "scratch" in _lib.last_error()
    # a successful call (zero rows) clears this thread's error message again
    assert L.esa_lightning_step(None, 3, 0, None, None, 0, None, 0, 0, 1, 0.8, 0.995, 1e-5, None) == 0
    assert _lib.last_error() == ""


def test_slice_prod_and_fixup_reject_bad_arguments_without_device_work():
    """esa_scan_prod / esa_scan_fixup: empty problems are no-ops, bad sizes,
    dtypes and null pointers are refused before any launch."""
    from esa import _lib
    L = _lib.lib()
    assert L.esa_scan_prod(None, None, 0, 100, 64, _lib.DTYPE_F16, None) == 0
    assert L.esa_scan_fixup(None, None, None, None, 4, 100, 0, _lib.DTYPE_BF16, None) == 0
    assert L.esa_scan_prod(None, None, -1, 100, 64, _lib.DTYPE_F16, None) != 0
    assert "negative" in _lib.last_error()
    assert L.esa_scan_prod(None, None, 1, 100, 64, 9, None) != 0
    assert "dtype" in _lib.last_error()
    assert L.esa_scan_prod(None, None, 1, 100, 64, _lib.DTYPE_F32, None) != 0
    assert "null" in _lib.last_error()
    assert L.esa_scan_fixup(16, 16, 16, None, 1, 100, 64, _lib.DTYPE_F32, None) != 0
    assert "null" in _lib.last_error()
    assert L.esa_scan_prod(None, None, 0, 0, 0, _lib.DTYPE_F32, None) == 0
    assert _lib.last_error() == ""


def test_library_loads_and_exports_every_declared_symbol():
    from esa import _lib
    L = _lib.lib()
    for name in _declared_symbols():
        assert hasattr(L, name), name
        assert name in _lib.SIGNATURES, name
    assert L.esa_abi_version() == _lib.ABI_VERSION
    assert _lib.last_error() == ""


def test_workspace_size_is_pure_host_arithmetic():
    from esa import _lib
    L = _lib.lib()
    n16 = L.esa_scan_workspace_bytes(32, 4096, 1024, _lib.DTYPE_F16, 16)
    n32 = L.esa_scan_workspace_bytes(32, 4096, 1024, _lib.DTYPE_F32, 16)
    assert n16 > 0 and n32 > 0
    assert L.esa_scan_workspace_bytes(32, 4096, 1024, 9, 16) == 0      # bad dtype
    assert L.esa_scan_workspace_bytes(32, 4096, 1024, _lib.DTYPE_F16, 0) == 0  # bad compass


def test_host_staging_is_bounded():
    from esa import _lib
    L = _lib.lib()
    small = L.esa_scan_host_staging_bytes(2, 64, 128, _lib.DTYPE_F16, 16)
    big = L.esa_scan_host_staging_bytes(32, 4096, 1024, _lib.DTYPE_F16, 16)
    huge = L.esa_scan_host_staging_bytes(4, 262144, 2048, _lib.DTYPE_BF16, 16)
    assert 0 < small <= big
    assert big < 512 << 20 and huge < 512 << 20
    assert L.esa_scan_host_staging_bytes(2, 64, 128, 9, 16) == 0
    rc = L.esa_scan_fwd_host(None, None, None, 1, 4, 8, _lib.DTYPE_F32, 16, None, 0, None)
    assert rc == -1 and "null host pointer" in _lib.last_error()


def test_abi_argument_errors_need_no_gpu():
    from esa import _lib
    L = _lib.lib()
    rc = L.esa_scan_fwd(None, None, None, 1, 4, 8, _lib.DTYPE_F32, 0, None, None, None, 0, None)
    assert rc == -1 and "compass" in _lib.last_error()
    rc = L.esa_scan_fwd(None, None, None, 1, 4, 8, 7, 16, None, None, None, 0, None)
    assert rc in (-1, -2)
    rc = L.esa_lightning_step(None, 3, _lib.DTYPE_F32, None, None, _lib.DTYPE_F32, None,
                              _lib.DTYPE_F32, 1, 4, 0.8, 0.995, 1e-5, None)
    assert rc == -1 and "stride" in _lib.last_error()


def test_cross_entropy_argument_errors_need_no_gpu():
    """The LM-head loss entry points reject bad shapes and dtypes before any
    device work; the Python op only takes 2-D CUDA logits."""
    import torch
    from esa import _lib, ops
    L = _lib.lib()
    rc = L.esa_cross_entropy_fwd(None, 10, _lib.DTYPE_F16, None, -1, None, None, 4, 0, None)
    assert rc == -1 and "V > 0" in _lib.last_error()
    rc = L.esa_cross_entropy_fwd(None, 5, _lib.DTYPE_F16, None, -1, None, None, 4, 10, None)
    assert rc == -1 and "row stride" in _lib.last_error()
    rc = L.esa_cross_entropy_fwd(None, 10, _lib.DTYPE_F64, None, -1, None, None, 4, 10, None)
    assert rc == -2
    rc = L.esa_cross_entropy_bwd(None, 10, _lib.DTYPE_F16, None, -1, None, None, None, 8, 4, 10, None)
    assert rc == -1 and "gradient row stride" in _lib.last_error()
    rc = L.esa_cross_entropy_fwd(None, 10, _lib.DTYPE_F32, None, -1, None, None, 4, 10, None)
    assert rc == -1 and "null" in _lib.last_error()
    z = torch.randn(4, 10)
    t = torch.zeros(4, dtype=torch.int64)
    assert not ops.cross_entropy_supported(z, t)          # CPU logits: the model keeps F.cross_entropy
    assert not ops.cross_entropy_supported(z[None], t)    # 3-D


def test_public_surface_matches_reference():
    import esa
    from esa import ESA
    from esa.backends import FlareESA, PulseESA, ThunderESA, flare_scan, pulse_scan, thunder_scan
    from esa.generation import (esa_prefill, lightning_decode_step, lightning_init_state,
                                lightning_prefill, parse_engine_spec, sample_next_token)
    assert esa.__version__ == "2.1.1"
    sig = inspect.signature(ESA)
    assert sig.parameters["backend"].default == "thunder"
    assert sig.parameters["precision"].default == "fp16"
    assert sig.parameters["eps"].default == 1e-5
    assert list(inspect.signature(thunder_scan).parameters) == ["A", "B_write", "compass", "c"]
    assert inspect.signature(thunder_scan).parameters["compass"].default == 16
    assert lightning_prefill is esa_prefill
    del FlareESA, PulseESA, ThunderESA, flare_scan, pulse_scan, lightning_decode_step
    del lightning_init_state, parse_engine_spec, sample_next_token


def test_layer_validation_matches_reference():
    from esa import ESA
    layer = ESA(embd=32, head=4, device=None)
    assert layer.compass == 16 and layer.backend == "thunder"
    assert ESA(embd=32, head=4, backend="pulse", device=None).compass is None
    with pytest.raises(ValueError, match="compass is only supported"):
        ESA(embd=32, head=4, backend="pulse", compass=16, device=None)
    with pytest.raises(ValueError, match="compass is only supported"):
        ESA(embd=32, head=4, backend="flare", compass=16, device=None)
    with pytest.raises(TypeError):
        ESA(n_embd=32, n_head=4)
    with pytest.raises(ValueError, match="Supported backends"):
        ESA(embd=32, head=4, backend="lightning", device=None)
    with pytest.raises(ValueError, match="divisible"):
        ESA(embd=30, head=4, device=None)
    with pytest.raises(ValueError, match="compass must be positive"):
        ESA(embd=32, head=4, compass=-1, device=None)


def test_state_dict_keys_match_reference_checkpoint():
    import numpy as np
    from conftest import GOLDEN
    from esa import ESAModel, ESAModelConfig
    z = np.load(GOLDEN / "model_generate.npz")
    ref_keys = {k[4:] for k in z.files if k.startswith("sd::")}
    cfg = ESAModelConfig(vocab_size=64, block=32, n_layer=2, head=4, embd=32, dropout=0.0,
                         precision="fp32", backend="thunder")
    model = ESAModel(cfg, device="cpu")
    assert set(model.state_dict().keys()) == ref_keys
    sd = {k[4:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("sd::")}
    model.load_state_dict(sd, strict=True)


def test_engine_parser_and_precision():
    from esa.generation import parse_engine_spec
    from esa.precision import resolve_scan_dtype
    s = parse_engine_spec("thunder_compiled_16")
    assert (s.backend, s.compiled, s.compass) == ("thunder", True, 16)
    assert parse_engine_spec("flare_compiled").compiled
    assert parse_engine_spec("lightning").backend == "lightning"
    assert parse_engine_spec("thunder").compass == 16
    with pytest.raises(ValueError):
        parse_engine_spec("pulse_16")
    with pytest.raises(ValueError):
        parse_engine_spec("warp")
    assert resolve_scan_dtype("fp16", "cuda") == torch.float16
    assert resolve_scan_dtype("fp16", "cpu") == torch.float32
    assert resolve_scan_dtype("bf16", "cpu") == torch.bfloat16
    assert resolve_scan_dtype("fp64", "cuda") == torch.float64
    with pytest.warns(RuntimeWarning):
        assert resolve_scan_dtype("fp8", "cuda") == torch.float16
    with pytest.raises(NotImplementedError):
        resolve_scan_dtype("fp8", "cuda", strict_precision=True)
    with pytest.raises(ValueError):
        resolve_scan_dtype("int8", "cuda")


def test_no_cpu_fallback():
    from esa import ESA
    from esa.backends.thunder import thunder_scan
    layer = ESA(embd=32, head=4, precision="fp32", device=None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        layer(torch.randn(2, 16, 32))
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        thunder_scan(torch.rand(1, 4, 2, 8), torch.rand(1, 4, 2, 8))


def test_scan_argument_errors_on_cpu_tensors():
    from esa.backends.thunder import thunder_scan
    a = torch.ones(2, 3, 4, 5)
    with pytest.raises(ValueError, match="same shape"):
        thunder_scan(a, torch.ones(2, 3, 4, 6))
    with pytest.raises(ValueError, match=r"\[B,T,H,D\]"):
        thunder_scan(a[0], a[0])
    with pytest.raises(ValueError, match="positive integer"):
        thunder_scan(a, a, compass=0)
    with pytest.raises(ValueError, match="positive integer"):
        thunder_scan(a, a, c=-3)


def test_fake_kernels_trace_without_gpu():
    """The custom ops have meta kernels: shapes/dtypes propagate on the meta device."""
    from esa import ops
    A = torch.empty(2, 10, 4, 8, device="meta", dtype=torch.float16)
    E, el = ops.scan(A, A, None, 16)
    assert E.shape == A.shape and E.dtype == torch.float16 and el.shape == (2, 32)
    assert el.dtype == torch.float32
    g = torch.empty(2, 10, 96, device="meta")[..., 32:64]
    E, el = ops.gated_scan(g, g, None, 0.8, 0.995, 16, torch.bfloat16)
    assert E.shape == (2, 10, 32) and E.dtype == torch.bfloat16
    ns, z = ops.lightning_step(torch.empty(3, 96, device="meta"),
                               torch.empty(3, 32, device="meta", dtype=torch.float16),
                               0.8, 0.995, 1e-5, torch.float32)
    assert ns.dtype == torch.float16 and z.dtype == torch.float32 and z.shape == (3, 32)
    z = torch.empty(6, 50, device="meta", dtype=torch.float16)
    t = torch.empty(6, device="meta", dtype=torch.int64)
    loss, lse = ops.cross_entropy_rows(z, t, -1)
    assert loss.shape == (6,) and lse.shape == (6,) and loss.dtype == torch.float32
    dz = ops.cross_entropy_rows_backward(z, t, lse, loss, -1)
    assert dz.shape == z.shape and dz.dtype == torch.float16


def test_library_symbols_via_ctypes_cdll():
    from esa import _lib
    cdll = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in _declared_symbols():
        getattr(cdll, name)


def test_seeded_weights_cover_the_model_fixtures():
    """The model-level fixtures carry no weights: both sides fill the model
    with tests/golden/seeded.py.  Its values are deterministic, the tied
    wte / lm_head weight is filled once, and this package's ESAModel has the
    parameter set the training-step fixture's gradients were taken over."""
    import sys

    import numpy as np
    from conftest import GOLDEN
    from esa import ESAModel, ESAModelConfig
    if str(GOLDEN) not in sys.path:
        sys.path.insert(0, str(GOLDEN))
    from seeded import fill_model
    cfg = ESAModelConfig(vocab_size=256, block=512, n_layer=2, head=4, embd=64, dropout=0.0,
                         precision="fp32", backend="thunder", training_compile=False)
    a, b = ESAModel(cfg, device="cpu"), ESAModel(cfg, device="cpu")
    fill_model(a, seed=7, n_layer=2)
    fill_model(b, seed=7, n_layer=2)
    for (n, p), (_, q) in zip(a.named_parameters(), b.named_parameters()):
        assert torch.equal(p, q), n
    assert a.lm_head.weight.data_ptr() == a.wte.weight.data_ptr()
    assert abs(float(a.blocks[0].ln1.weight.detach().mean()) - 1.0) < 0.05
    z = np.load(GOLDEN / "model_train_step.npz")
    grads = {k[6:]: z[k].shape for k in z.files if k.startswith("grad::")}
    assert {n: tuple(p.shape) for n, p in a.named_parameters()} == grads


def test_layer_core_entry_points_need_no_gpu_for_sizes_and_errors():
    """esa_layer_workspace_bytes is host arithmetic (the gated scan's
    workspace plus the dE buffer between the readout backward and the reverse
    scan); esa_layer_fwd / esa_layer_bwd reject bad arguments before any
    device work."""
    from esa import _lib
    L = _lib.lib()
    F16, F32 = _lib.DTYPE_F16, _lib.DTYPE_F32
    ws = L.esa_layer_workspace_bytes(16, 2048, 768, F16, F16, F16)
    scan = L.esa_scan_workspace_bytes(16, 2048, 768, F16, 16)
    de = 16 * 2048 * 768 * 2
    assert ws == de + scan
    two = L.esa_layer_workspace_bytes(2, 300, 96, F32, F32, F32)
    assert two >= 2 * 300 * 96 * 4                                # holds dE
    assert L.esa_layer_workspace_bytes(2, 300, 96, 9, F32, F32) == 0
    assert L.esa_layer_workspace_bytes(2, 300, 0, F32, F32, F32) == 0
    rc = L.esa_layer_fwd(None, 100, F16, None, F16, None, F16, None, 2, 8, 64, 0.8, 0.995, 1e-5,
                         None, None, None, 0, None)
    assert rc == -1 and "row stride" in _lib.last_error()
    rc = L.esa_layer_fwd(None, 192, F16, None, F16, None, F16, None, 2, 8, 64, 0.8, 0.995, 1e-5,
                         None, None, None, 0, None)
    assert rc == -1 and "null" in _lib.last_error()
    rc = L.esa_layer_bwd(None, F16, None, 192, 7, None, F16, None, None, 192, 2, 8, 64, 0.8, 0.995,
                         1e-5, None, None, None, 0, None)
    assert rc == -2
    assert L.esa_layer_fwd(None, 192, F16, None, F16, None, F16, None, 0, 8, 64, 0.8, 0.995, 1e-5,
                           None, None, None, 0, None) == 0  # empty problem
