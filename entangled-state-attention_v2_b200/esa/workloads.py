"""Fixed kernel workloads for profiling (`python -m esa.workloads <name>`).

Each workload runs four iterations of one kernel family on seeded synthetic
inputs, so that a profiler can skip the first launches and capture one:

    rev        reverse scan, [32,4096,16,64] fp16 (the microbenchmark shape)
    gated      fused gated scan forward + backward, [16,2048,768] fp16 (an
               ESAModel training layer: 12 heads of 64)
    split      forward scan of a long sequence, [4,65536,32,64] bf16 (the
               split scan: summary pass, piece composition, output pass)
    readout    layer core forward + backward (readout kernels), [16,2048,768]
    layernorm  fused LayerNorm forward + backward, [16,2048,768] fp32 -> fp16
    train      the ESAModel training step (12 layers of 768, batch 16 x 2048,
               fp16 autocast, AdamW): four warm-up steps, then two steps under
               torch.profiler; prints the device time per step of the top
               kernels
"""

from __future__ import annotations

import sys

import torch

from . import ops

WORKLOADS = ("rev", "gated", "split", "readout", "layernorm", "train")


def train_profile(top: int = 30) -> None:
    from torch.profiler import ProfilerActivity, profile

    from .model import ESAModel, ESAModelConfig
    torch.manual_seed(1234)
    cfg = ESAModelConfig(vocab_size=32000, block=2048, n_layer=12, head=12, embd=768, backend="thunder",
                         precision="fp16", dropout=0.0, bias=True, tie_embeddings=True, training_compile=False)
    model = ESAModel(cfg, device="cuda")
    model.train()
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, fused=True)
    scaler = torch.amp.GradScaler("cuda")
    ids = torch.randint(0, 32000, (16, 2049), device="cuda")

    def step():
        with torch.autocast("cuda", dtype=torch.float16):
            _, loss = model(ids[:, :-1], ids[:, 1:])
        scaler.scale(loss).backward()
        scaler.step(opt)
        scaler.update()
        opt.zero_grad(set_to_none=True)

    for _ in range(4):
        step()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(2):
            step()
        torch.cuda.synchronize()
    rows = sorted(((k.device_time_total, k.count, k.key) for k in prof.key_averages()), reverse=True)
    total = sum(r[0] for r in rows)
    print(f"device time per step: {total / 2:.1f} us")
    for t, n, key in rows[:top]:
        print(f"{t / 2:10.1f} us {100 * t / total:5.1f} % {n // 2:4d} launches  {key[:100]}")


def run(name: str, iters: int = 4) -> None:
    if name not in WORKLOADS:
        raise ValueError(f"unknown workload {name!r}; one of {WORKLOADS}")
    if name == "train":
        train_profile()
        return
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape, dtype=torch.float16):
        return torch.randn(*shape, device=dev, generator=g).to(dtype)

    if name == "rev":
        A = torch.sigmoid(rnd(32, 4096, 16, 64, dtype=torch.float32) * 2 + 2).half()
        E, dE = rnd(32, 4096, 16, 64), rnd(32, 4096, 16, 64)
        for _ in range(iters):
            ops.scan_backward(A, E, dE, None, 16)
    elif name == "gated":
        C = 768
        qgv = rnd(16, 2048, 3 * C)
        gr, vr = qgv[..., C:2 * C], qgv[..., 2 * C:]
        for _ in range(iters):
            E, _ = ops.gated_scan(gr, vr, None, 0.8, 0.995, 16, torch.float16)
            ops.gated_scan_backward(gr, vr, E, E, None, 0.8, 0.995, 16)
    elif name == "split":
        A = torch.sigmoid(rnd(4, 65536, 32, 64, dtype=torch.float32) + 3).to(torch.bfloat16)
        B = (rnd(4, 65536, 32, 64, dtype=torch.float32) * 0.5).to(torch.bfloat16)
        for _ in range(iters):
            ops.scan(A, B, None, 16)
    elif name == "readout":
        C = 768
        qgv = rnd(16, 2048, 3 * C).requires_grad_(True)
        for _ in range(iters):
            y, _, _ = ops.layer_core(qgv, 0.8, 0.995, 1e-5, 16, torch.float16, torch.float16)
            y.backward(torch.ones_like(y))
    else:
        x = rnd(16, 2048, 768, dtype=torch.float32).requires_grad_(True)
        w = torch.ones(768, device=dev, requires_grad=True)
        b = torch.zeros(768, device=dev, requires_grad=True)
        for _ in range(iters):
            y, _, _ = ops.layer_norm(x, w, b, 1e-5, torch.float16)
            y.backward(torch.ones_like(y))
    torch.cuda.synchronize()
    ops.check_device_status()


if __name__ == "__main__":
    for n in sys.argv[1:] or WORKLOADS:
        run(n)
        print("ok", n)
