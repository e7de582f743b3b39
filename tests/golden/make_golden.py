"""Generate the golden fixtures in this folder by running the reference ESA package.

The reference (maxzameer/Entangled-State-Attention_v2, v2.1.1) is pure Python on
PyTorch, so it can be imported on a CPU-only machine.  This script imports it from
the checkout named by ``ESA_REFERENCE_PATH`` (the directory holding ``esa/``),
runs the reference functions on seeded inputs and stores inputs plus outputs as
compressed ``.npz`` files.  The files are committed; the test suite and the GPU
box never read the reference itself.

Run from the repository root::

    ESA_REFERENCE_PATH=<reference checkout> python tests/golden/make_golden.py

Fixtures produced (all small enough for git):

* ``scan_lifecycle.npz``   -- the reference's own chunked-vs-pulse case
  (tests/test_v2_1_model_lifecycle.py:17-52): A = 0.8 + 0.19*U, B = 0.1*N,
  shape [2,17,4,8], seed 1; pulse_scan (fp32, fp64) and thunder_scan (compass 4, 16).
* ``scan_shapes.npz``      -- pulse_scan / thunder_scan on ragged and edge shapes
  (T = 1, 9, 33, 130; HD = 15, 24, 128, 1024) with the microbenchmark's value
  distribution A = sigmoid(2N+2), B = N(0,1), in fp64/fp32/fp16/bf16.
* ``scan_grad.npz``        -- autograd of sum(E * dE) through pulse_scan in fp64
  (the reverse-scan oracle) for two shapes.
* ``layer_pulse.npz``      -- ESA(embd=128, head=4, backend="pulse") forward and
  backward (x.grad, qgv.weight.grad, out_proj.weight.grad) in fp64 and fp32 at
  x [2,96,128]; and thunder fp32 forward on the same weights.
* ``decode.npz``           -- ESA(embd=64, head=4, backend="pulse", fp32):
  prefill over a prompt then five lightning decode steps.
* ``model_generate.npz``   -- a tiny ESAModel (2 layers, embd 32, head 4, vocab
  64, fp32, backend thunder) state_dict, a prompt, and greedy generate ids with
  prefill "thunder_16" and "pulse" (compile=False).
* ``model_decode_24l.npz`` -- the decode workload's model (24 layers, embd 1024,
  head 16, vocab 32000, block 1024, fp32, backend thunder) filled with the
  seeded weights of ``seeded.py`` (not stored: 1.3 GB); a 512-token uniform
  prompt and the 256 greedy ids of ``generate(prefill="thunder_16",
  runtime="lightning", temperature=0, compile=False)``, plus the smallest
  top-1/top-2 logit gap of a teacher-forced pass over the result (how far the
  greedy choices are from a tie).
* ``model_train_step.npz`` -- a small fp32 ESAModel (2 layers, embd 64, head 4,
  vocab 256, block 512, seeded weights) on a [12, 512] batch (6144 rows): the
  training loss, a slice of the logits and the gradient of every parameter
  after ``loss.backward()``.

Only some fixtures: ``python tests/golden/make_golden.py decode_24l train_step``.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def _np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        # numpy has no bfloat16: store the raw 16-bit pattern.
        return t.view(torch.int16).numpy()
    return t.numpy()


def main() -> None:
    ref = os.environ.get("ESA_REFERENCE_PATH")
    if not ref:
        raise SystemExit("set ESA_REFERENCE_PATH to the reference checkout (the directory holding esa/)")
    only = set(sys.argv[1:])
    sys.path.insert(0, ref)
    sys.path.insert(0, str(OUT))
    import esa  # noqa: F401  (the reference package)
    from esa import ESA, ESAModel, ESAModelConfig
    from esa.backends.pulse import pulse_scan
    from esa.backends.thunder import thunder_scan

    assert esa.__file__.startswith(os.path.abspath(ref)), esa.__file__
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    if only:
        unknown = only - set(MODEL_FIXTURES)
        if unknown:
            raise SystemExit(f"unknown fixtures {sorted(unknown)}; choose from {sorted(MODEL_FIXTURES)}")
        for name in sorted(only):
            MODEL_FIXTURES[name]()
        return

    # 1. The reference's own chunked-scan parity case.
    torch.manual_seed(1)
    A = 0.8 + 0.19 * torch.rand(2, 17, 4, 8)
    B = torch.randn_like(A) * 0.1
    np.savez_compressed(
        OUT / "scan_lifecycle.npz",
        A=_np(A), B=_np(B),
        pulse_f32=_np(pulse_scan(A, B)),
        pulse_f64=_np(pulse_scan(A.double(), B.double())),
        thunder_c4_f32=_np(thunder_scan(A, B, compass=4)),
        thunder_c16_f32=_np(thunder_scan(A, B, compass=16)),
    )

    # 2. Edge and ragged shapes, microbenchmark distribution.
    shapes = {
        "t1": (3, 1, 4, 8),
        "t9": (2, 9, 2, 12),         # T < compass
        "t33_hd15": (2, 33, 5, 3),   # HD not a multiple of any vector width
        "t130": (2, 130, 4, 32),
        "t64_hd1024": (1, 64, 16, 64),
    }
    arrays = {}
    g = torch.Generator().manual_seed(20261201)
    for name, shp in shapes.items():
        a = torch.sigmoid(torch.randn(shp, generator=g, dtype=torch.float64) * 2 + 2)
        b = torch.randn(shp, generator=g, dtype=torch.float64)
        arrays[f"{name}_A"] = _np(a)
        arrays[f"{name}_B"] = _np(b)
        arrays[f"{name}_pulse_f64"] = _np(pulse_scan(a, b))
        a32, b32 = a.float(), b.float()
        arrays[f"{name}_pulse_f32"] = _np(pulse_scan(a32, b32))
        arrays[f"{name}_thunder_c16_f32"] = _np(thunder_scan(a32, b32, compass=16))
        for dt, tag in ((torch.float16, "f16"), (torch.bfloat16, "bf16")):
            ad, bd = a.to(dt), b.to(dt)
            arrays[f"{name}_thunder_c16_{tag}"] = _np(thunder_scan(ad, bd, compass=16))
    np.savez_compressed(OUT / "scan_shapes.npz", **arrays)

    # 3. Reverse scan: autograd through pulse_scan in fp64.
    grads = {}
    for name, shp in {"g1": (2, 21, 3, 8), "g2": (1, 70, 2, 16)}.items():
        a = torch.sigmoid(torch.randn(shp, generator=g, dtype=torch.float64) * 2 + 2)
        b = torch.randn(shp, generator=g, dtype=torch.float64)
        de = torch.randn(shp, generator=g, dtype=torch.float64)
        a.requires_grad_(True)
        b.requires_grad_(True)
        e = pulse_scan(a, b)
        (e * de).sum().backward()
        grads.update({
            f"{name}_A": _np(a), f"{name}_B": _np(b), f"{name}_dE": _np(de),
            f"{name}_E": _np(e), f"{name}_dA": _np(a.grad), f"{name}_dB": _np(b.grad),
        })
    np.savez_compressed(OUT / "scan_grad.npz", **grads)

    # 4. Layer forward/backward, pulse fp64 + fp32 and thunder fp32 on same weights.
    torch.manual_seed(7)
    layer64 = ESA(embd=128, head=4, backend="pulse", precision="fp64", device=None)
    sd = {k: v.clone() for k, v in layer64.state_dict().items()}
    x = torch.randn(2, 96, 128, generator=g)
    out = {"x": _np(x), "qgv_w": _np(sd["layer.qgv.weight"]),
           "out_w": _np(sd["layer.out_proj.weight"])}
    for prec, dt in (("fp64", torch.float64), ("fp32", torch.float32)):
        lay = ESA(embd=128, head=4, backend="pulse", precision=prec, device=None).to(dt)
        lay.load_state_dict({k: v.to(dt) for k, v in sd.items()})
        xi = x.to(dt).clone().requires_grad_(True)
        y = lay(xi)
        y.sum().backward()
        out[f"pulse_{prec}_y"] = _np(y)
        out[f"pulse_{prec}_dx"] = _np(xi.grad)
        out[f"pulse_{prec}_dqgv"] = _np(lay.layer.qgv.weight.grad)
        out[f"pulse_{prec}_dout"] = _np(lay.layer.out_proj.weight.grad)
    th = ESA(embd=128, head=4, backend="thunder", precision="fp32", device=None)
    th.load_state_dict({k: v.float() for k, v in sd.items()})
    out["thunder_fp32_y"] = _np(th(x.float()))
    np.savez_compressed(OUT / "layer_pulse.npz", **out)

    # 5. Prefill + lightning decode steps.
    torch.manual_seed(11)
    dl = ESA(embd=64, head=4, backend="pulse", precision="fp32", device=None)
    dl.eval()
    xp = torch.randn(3, 12, 64, generator=g)
    y_fwd = dl(xp)
    y_pre, state = dl.prefill(xp)
    steps_x = torch.randn(5, 3, 64, generator=g)
    ys, sts = [], []
    s = state
    for i in range(5):
        y1, s = dl.decode_step(steps_x[i], s)
        ys.append(y1)
        sts.append(s)
    np.savez_compressed(
        OUT / "decode.npz",
        qgv_w=_np(dl.layer.qgv.weight), out_w=_np(dl.layer.out_proj.weight),
        x_prompt=_np(xp), y_forward=_np(y_fwd), y_prefill=_np(y_pre),
        state_prefill=_np(state), x_steps=_np(steps_x),
        y_steps=_np(torch.stack(ys)), state_steps=_np(torch.stack(sts)),
    )

    # 6. Tiny ESAModel greedy generation.
    torch.manual_seed(5)
    cfg = ESAModelConfig(vocab_size=64, block=32, n_layer=2, head=4, embd=32,
                         dropout=0.0, precision="fp32", backend="thunder")
    model = ESAModel(cfg, device="cpu")
    model.eval()
    ids = torch.randint(0, 64, (2, 10), generator=g)
    gen = {}
    for pf in ("thunder_16", "pulse"):
        seq = model.generate(input_ids=ids, seek=12, prefill=pf, compile=False,
                             temperature=0.0)
        gen[f"seq_{pf}"] = _np(seq)
    logits, _ = model(ids)
    sd = model.state_dict()
    np.savez_compressed(
        OUT / "model_generate.npz",
        ids=_np(ids), logits=_np(logits), **gen,
        **{f"sd::{k}": _np(v) for k, v in sd.items()},
    )
    for fn in MODEL_FIXTURES.values():
        fn()
    print("fixtures written to", OUT)


def decode_24l() -> None:
    """Greedy ids of the 24-layer decode model (fp32) on seeded weights."""
    from esa import ESAModel, ESAModelConfig
    from seeded import fill_model

    cfg = ESAModelConfig(vocab_size=32000, block=1024, n_layer=24, head=16, embd=1024,
                         dropout=0.0, precision="fp32", backend="thunder")
    model = ESAModel(cfg, device="cpu")
    fill_model(model, seed=24, n_layer=cfg.n_layer)
    model.eval()
    ids = torch.from_numpy(np.random.Generator(np.random.PCG64(512)).integers(0, 32000, size=(1, 512)))
    seq = model.generate(input_ids=ids, seek=256, prefill="thunder_16", runtime="lightning",
                         temperature=0.0, compile=False)
    with torch.no_grad():
        logits, _ = model(seq[:, :-1])
    top2 = torch.topk(logits[0, 511:], 2, dim=-1).values
    gap = (top2[:, 0] - top2[:, 1]).min()
    np.savez_compressed(OUT / "model_decode_24l.npz", prompt=_np(ids), seq=_np(seq),
                        min_top2_gap=np.float32(gap.item()), weight_seed=np.int64(24))
    print("decode_24l: min top-2 logit gap", float(gap))


def train_step() -> None:
    """Loss, logits and parameter gradients of one fp32 ESAModel training step."""
    from esa import ESAModel, ESAModelConfig
    from seeded import fill_model

    cfg = ESAModelConfig(vocab_size=256, block=512, n_layer=2, head=4, embd=64, dropout=0.0,
                         precision="fp32", backend="thunder", training_compile=False)
    model = ESAModel(cfg, device="cpu")
    fill_model(model, seed=7, n_layer=cfg.n_layer)
    model.train()
    ids = torch.from_numpy(np.random.Generator(np.random.PCG64(513)).integers(0, 256, size=(12, 513)))
    logits, loss = model(ids[:, :-1], ids[:, 1:])
    loss.backward()
    out = {"ids": _np(ids), "loss": _np(loss), "logits_rows_0_5_t_0_64": _np(logits[[0, 5], :64])}
    for name, p in model.named_parameters():
        out[f"grad::{name}"] = _np(p.grad)
    np.savez_compressed(OUT / "model_train_step.npz", **out)
    print("train_step: loss", float(loss.detach()))


MODEL_FIXTURES = {"decode_24l": decode_24l, "train_step": train_step}


if __name__ == "__main__":
    main()
