"""ESA hot-path benchmark: Thunder scan GB/s (fraction of the measured HBM
roofline) and ESAModel tokens/s, on 1 to 8 B200s of one node.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One run prints ONE JSON line (rank 0).  Its headline is the raw scan
microbenchmark: A, B of shape [B,T,H,D] = [32, 4096, 16, 64] (the reference
layout of [batch=32, heads=16, T=4096, d=64]), A = sigmoid(2 N(0,1) + 2),
B ~ N(0,1), E_0 = 0, fp16, compass 16; one step = one forward scan of the
whole tensor (kernel a).  Inputs (537 MB) and output (268 MB) exceed the
126 MB L2, so no flush is needed between steps.  At N > 1 (torchrun, one rank
per GPU) every rank scans its own [32,4096,16,64] shard (batch x head
sharding, no collective): weak scaling, value = all ranks' bytes /
max-over-ranks device time.

The same line carries the other workloads, each under its own key with its
own roofline and clock record:
  esamodel_train   ESAModel training step (12 layers, embd 768, head 12,
                   block 2048, vocab 32000, batch 16 x 2048 per GPU, fp16
                   autocast, GradScaler, AdamW), DDP over the N ranks;
  sp_scan          long-sequence scan [4, 262144, 32, 64] bf16 with T split
                   across the N ranks (slice summaries, one all-gather, scans
                   from the exact incoming states); the whole sequence on one
                   GPU at N = 1;
  decode           (N = 1) ESAModel 24 layers, embd 1024, head 16, vocab 32000,
                   512-token thunder_16 prefill + 256 greedy ESA-Lightning
                   tokens, batch 1 and 64 (prefill and decode tokens/s);
  layer            (N = 1) ESA(embd=128, head=4) fp32, x [16,1024,128],
                   forward + backward of sum(y), with the reference's CPU Pulse
                   layer timed beside it;
  gpu_comparators  (N = 1) the unmodified reference's own GPU paths on the
                   headline shape: Flare's Triton scan and Thunder eager and
                   under torch.compile (reference installed in baseline/_ref).
Random-init weights and seeded synthetic tokens / tensors throughout; no
dataset is involved.

Reference arm (--impl reference): the reference's CPU path for the headline
workload (its chunked Thunder scan restated in oracle/oracle.py, torch on all
host cores, fp32 -- the reference's CPU dtype for precision fp16) on a bounded
batch slice per step; rank 0 only.

Other entry points: --workload NAME prints one workload's own line;
--profile-workload NAME runs a fixed four-iteration kernel workload for ncu
(see profiles/).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
REF_INSTALL = ROOT / "baseline" / "_ref"
if "--gpu-comparators" not in sys.argv:
    # the reference's own package is also called `esa`: the comparator child
    # process imports it from baseline/_ref instead of this package
    sys.path.insert(0, str(ROOT / "entangled-state-attention_v2_b200"))
    sys.path.insert(0, str(ROOT))

SHAPE = (32, 4096, 16, 64)
METRIC = "thunder_scan_fwd_GBps"
UNIT = "GB/s"
WORKLOAD = "thunder_scan fwd [B,T,H,D]=[32,4096,16,64] fp16 compass=16"


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _bf16_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d.get("bf16_tflops_sustained", d.get("bf16_tflops"))), "measured sustained"
    return 1400.0, "fallback"


KERNEL_NAMES = {
    "lane": "lane_scan_kernel<FwdPlain, __half, __half, NW> (one lane per channel pair, steps in order)",
    "strip": "strip_scan_kernel<FwdPlain, __half, __half, LPR, SR> (strip width chosen per shape)",
}


def _traffic_summary():
    p = ROOT / "profiles" / "roofline_traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            return None
    return None


class ClockSampler:
    """nvidia-smi sampled every 100 ms while a timed region runs."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        sms, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                sms.append(float(parts[2]))
                mx = float(parts[3])
            except ValueError:
                continue
            for n, v in zip(names, parts[6:10]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sms)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class Ctx:
    """Rank, device and the collective helpers every leg shares."""

    def __init__(self, args):
        import torch
        import torch.distributed as dist

        self.args = args
        self.ws, self.rank, self.local = _dist()
        if args.gpus != self.ws and self.ws > 1:
            raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={self.ws}")
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.dist = dist
        if self.ws > 1:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=self.dev)

    def barrier(self):
        if self.ws > 1:
            self.dist.barrier()

    def max_over_ranks(self, x: float) -> float:
        import torch
        t = torch.tensor([x], device=self.dev, dtype=torch.float64)
        if self.ws > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.ws > 1:
            self.dist.destroy_process_group()


def _timed(ctx, fn, steps: int, stream=None) -> tuple[float, float, dict]:
    """Run fn() `steps` times back to back between two CUDA events on the
    launching stream (an event between steps would add its own gap to every
    step), barrier + synchronize on both sides, clocks sampled meanwhile.
    Returns (max-over-ranks total ms, this rank's mean ms per step, clocks)."""
    import torch
    stream = stream or torch.cuda.current_stream(ctx.dev)
    clocks = ClockSampler(ctx.local).start()
    time.sleep(0.3)
    fn()  # one more untimed step after the sampler's start-up pause (the GPU idled meanwhile)
    ctx.barrier()
    torch.cuda.synchronize(ctx.dev)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        fn()
    ev1.record(stream)
    torch.cuda.synchronize(ctx.dev)
    ctx.barrier()
    clk = clocks.stop()
    mine = ev0.elapsed_time(ev1)
    total = ctx.max_over_ranks(mine)
    return total, mine / steps, clk


# ---------------------------------------------------------------------------
# CPU baseline and the reference arm (the reference's CPU Thunder scan)
# ---------------------------------------------------------------------------
def cpu_baseline(target_s: float = 12.0, max_rows: int = 32) -> dict:
    """The reference's CPU Thunder scan (restated in the oracle), fp32, all
    host threads, on a batch slice of the workload; GB/s of algorithmic bytes."""
    import torch

    from oracle import oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    _, T, H, D = SHAPE
    rows = 1
    A = torch.sigmoid(torch.randn(rows, T, H, D, generator=g) * 2 + 2)
    B = torch.randn(rows, T, H, D, generator=g)
    oracle.thunder_scan_port(A, B, 16)  # warm-up
    t0 = time.perf_counter()
    oracle.thunder_scan_port(A, B, 16)
    one = time.perf_counter() - t0
    rows = int(max(1, min(max_rows, target_s / max(one, 1e-3) / 3)))
    A = torch.sigmoid(torch.randn(rows, T, H, D, generator=g) * 2 + 2)
    B = torch.randn(rows, T, H, D, generator=g)
    times = []
    for _ in range(3):
        t0 = time.perf_counter()
        oracle.thunder_scan_port(A, B, 16)
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    nbytes = 3 * A.numel() * 4
    return {"value": nbytes / t / 1e9, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"thunder_scan restatement (oracle.thunder_scan_port, torch eager CPU, fp32, "
                      f"compass 16) on a [{rows},{T},{H},{D}] batch slice, median of 3, "
                      f"{t:.2f} s each"}


def run_reference(args) -> None:
    ws, rank, _ = _dist()
    if rank != 0:
        return
    import torch

    from oracle import oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    _, T, H, D = SHAPE
    g = torch.Generator().manual_seed(0)
    # size each step's slice so that warmup + steps stay within ~2 minutes
    A1 = torch.sigmoid(torch.randn(1, T, H, D, generator=g) * 2 + 2)
    B1 = torch.randn(1, T, H, D, generator=g)
    oracle.thunder_scan_port(A1, B1, 16)
    t0 = time.perf_counter()
    oracle.thunder_scan_port(A1, B1, 16)
    one = max(time.perf_counter() - t0, 1e-4)
    budget = 120.0 / max(1, args.steps + args.warmup)
    Tn = T
    if one > budget:
        Tn = max(64, int(T * budget / one) // 64 * 64)
    A = A1[:, :Tn].contiguous()
    B = B1[:, :Tn].contiguous()
    for _ in range(args.warmup):
        oracle.thunder_scan_port(A, B, 16)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.thunder_scan_port(A, B, 16)
    el = time.perf_counter() - t0
    nbytes = 3 * A.numel() * 4
    val = nbytes * args.steps / el / 1e9
    sample = (f"thunder_scan restatement (torch eager CPU, fp32, compass 16) on a [1,{Tn},{H},{D}] "
              f"slice of the [32,4096,16,64] workload per step")
    line = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded)", "config": {"workload": WORKLOAD, "cpu_sample": sample},
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Headline: forward Thunder scan, config 2
# ---------------------------------------------------------------------------
def _gpu_numa_node(dev_index: int):
    try:
        import torch
        pr = torch.cuda.get_device_properties(dev_index)
        bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        return int(Path(f"/sys/bus/pci/devices/{bus}/numa_node").read_text().strip())
    except Exception:
        return None


def scan_leg(ctx) -> dict:
    import torch

    from esa import _lib, ops

    args = ctx.args
    dev, ws, rank = ctx.dev, ctx.ws, ctx.rank
    L = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    A = torch.sigmoid(torch.randn(SHAPE, device=dev, generator=gen) * 2 + 2).half()
    B = torch.randn(SHAPE, device=dev, generator=gen).half()
    E = torch.empty_like(A)
    nb, T, H, D = SHAPE
    hd = H * D
    N = A.numel()
    compass = 16
    wsb = L.esa_scan_workspace_bytes(nb, T, hd, _lib.DTYPE_F16, compass)
    wsp = torch.empty(wsb, dtype=torch.uint8, device=dev)
    sp = stream.cuda_stream

    def step():
        rc = L.esa_scan_fwd(A.data_ptr(), B.data_ptr(), E.data_ptr(), nb, T, hd, _lib.DTYPE_F16,
                            compass, None, None, wsp.data_ptr(), wsb, sp)
        if rc:
            raise RuntimeError(_lib.last_error())

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    path = _lib.last_scan_path()  # kernel family the timed launches use
    total_ms, mean_launch_ms, clk = _timed(ctx, step, args.steps, stream)
    alg_bytes = 3 * N * 2
    value = ws * alg_bytes * args.steps / (total_ms * 1e-3) / 1e9
    peak, peak_kind = _peaks()
    achieved = alg_bytes / (mean_launch_ms * 1e-3) / 1e9
    ops.check_device_status(dev)

    # correctness spot check of the timed output: 16 channels x the first 256
    # steps against a plain fp32 torch recurrence
    ref_a, ref_b = A[0, :256, 0, :16].float(), B[0, :256, 0, :16].float()
    s = torch.zeros(16, device=dev)
    outs = []
    for tt in range(256):
        s = ref_a[tt] * s + ref_b[tt]
        outs.append(s)
    ref = torch.stack(outs)
    errs = float((E[0, :256, 0, :16].float() - ref).norm() / ref.norm())

    # e2e through the public API with pinned host buffers: thunder_scan_host
    # streams A, B from host memory through the device and E back (the copies
    # in both directions overlap the scans of other chunks)
    from esa.backends.thunder import thunder_scan_host
    hA = A.cpu().pin_memory()
    hB = B.cpu().pin_memory()
    hE = torch.empty_like(hA).pin_memory()
    k2 = max(3, min(args.steps, 10))

    def e2e_step():
        thunder_scan_host(hA, hB, compass=16, out=hE)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    e2e_total, _, e2e_clk = _timed(ctx, e2e_step, k2, stream)
    ms = e2e_total / k2
    e2e_err = float((hE[0, :256, 0, :16].float() - ref.cpu()).norm() / ref.cpu().norm())
    host_bytes = 3 * N * 2
    e2e = {"value": ws * alg_bytes / (ms * 1e-3) / 1e9, "unit": UNIT,
           "h2d_bytes_per_step": 2 * N * 2, "d2h_bytes_per_step": N * 2,
           "ms_per_step": ms, "spot_check_rel_err": e2e_err,
           "api": "esa.backends.thunder.thunder_scan_host (C ABI esa_scan_fwd_host), "
                  "pinned host buffers, copies pipelined in 32 MB chunks",
           "limiter": {"host_link_GBps_per_rank": host_bytes / (ms * 1e-3) / 1e9,
                       "host_link_GBps_all_ranks": ws * host_bytes / (ms * 1e-3) / 1e9,
                       "gpu_numa_node": _gpu_numa_node(ctx.local),
                       "cpu_affinity_cores": len(os.sched_getaffinity(0)),
                       "note": "host->device and device->host copies over PCIe, every rank's "
                               "pinned buffers in host memory: bound by the PCIe links and, "
                               "when all GPUs sit on one NUMA node, that node's memory"},
           "clocks": e2e_clk}
    del hA, hB, hE, A, B, E, wsp

    extra = secondary(dev, stream, L) if (rank == 0 and not args.quick) else {}
    ctx.barrier()
    traffic = _traffic_summary()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded)",
        "config": {"workload": WORKLOAD, "shape_BTHD": list(SHAPE), "compass": compass,
                   "compass_note": "compass picks the time tile of the look-back kernel only; "
                                   "this shape runs the lane-serial kernel, which has no chunk "
                                   "size (secondary.fwd_f16_compass32/64 time the sweep)",
                   "parallelism": f"batch x head sharding, {ws} independent shards",
                   "l2": "inputs 537 MB + output 268 MB > 126 MB L2; no flush",
                   "spot_check_rel_err": errs},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "algorithmic_bytes_per_launch": alg_bytes,
                     "mean_launch_ms": mean_launch_ms,
                     "kernel": KERNEL_NAMES.get(path, path),
                     "traffic": (traffic or {}).get("bytes_per_launch"),
                     "traffic_source": (traffic or {}).get("source")},
        "cpu_baseline": None,
        "e2e": e2e,
        "gpu_launches": args.steps,
        "clocks": clk,
    }
    if extra:
        line["secondary"] = extra
    return line


def secondary(dev, stream, L) -> dict:
    """Kernel-only GB/s of the other scan kinds and dtypes (algorithmic bytes):
    forward fp32, bare reverse fp16/fp32, the headline at compass 32 and 64,
    the fused gated forward/backward of a [16, 2048, 768] fp16 layer, and a
    [74, 2048, 16, 64] fp16 forward whose 296 strips fill every SM evenly."""
    import torch

    from esa import _lib

    sp = stream.cuda_stream
    out = {}

    def timeit(fn, k=30):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(k):
            fn()
        b.record(stream)
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / k

    g = torch.Generator(device=dev).manual_seed(99)
    codes = {torch.float16: _lib.DTYPE_F16, torch.float32: _lib.DTYPE_F32}

    def scans(shape, dt, tag, compasses=(16,)):
        nb, T, H, D = shape
        hd = H * D
        N = nb * T * hd
        es = torch.empty((), dtype=dt).element_size()
        code = codes[dt]
        A = torch.sigmoid(torch.randn(shape, device=dev, generator=g) * 2 + 2).to(dt)
        B = torch.randn(shape, device=dev, generator=g).to(dt)
        E = torch.empty_like(A)
        for c in compasses:
            wsb = L.esa_scan_workspace_bytes(nb, T, hd, code, c)
            w = torch.empty(wsb, dtype=torch.uint8, device=dev)
            ms = timeit(lambda: L.esa_scan_fwd(A.data_ptr(), B.data_ptr(), E.data_ptr(), nb, T, hd, code, c,
                                               None, None, w.data_ptr(), wsb, sp))
            key = f"fwd_{tag}_GBps" if c == 16 else f"fwd_f16_compass{c}_GBps"
            out[key] = 3 * N * es / (ms * 1e-3) / 1e9
        if tag.endswith("32x4096x16x64"):
            wsb = L.esa_scan_workspace_bytes(nb, T, hd, code, 16)
            w = torch.empty(wsb, dtype=torch.uint8, device=dev)
            dE = torch.randn(shape, device=dev, generator=g).to(dt)
            dA = torch.empty_like(A)
            dB = torch.empty_like(A)
            ms = timeit(lambda: L.esa_scan_rev(A.data_ptr(), E.data_ptr(), dE.data_ptr(), dA.data_ptr(),
                                               dB.data_ptr(), nb, T, hd, code, 16, None, None,
                                               w.data_ptr(), wsb, sp))
            out[f"rev_{tag}_GBps"] = 5 * N * es / (ms * 1e-3) / 1e9

    scans(SHAPE, torch.float32, "f32_32x4096x16x64")
    scans(SHAPE, torch.float16, "f16_32x4096x16x64", compasses=(16, 32, 64))
    scans((74, 2048, 16, 64), torch.float16, "f16_74x2048x16x64")
    # fused gated scans of one ESA layer: qgv [16, 2048, 3*768] fp16
    nb, T, C = 16, 2048, 768
    qgv = torch.randn(nb, T, 3 * C, device=dev, generator=g).half()
    gr, vr = qgv[..., C:2 * C], qgv[..., 2 * C:]
    Eg = torch.empty(nb, T, C, device=dev, dtype=torch.float16)
    dE = torch.randn(nb, T, C, device=dev, generator=g).half()
    dg = torch.empty_like(Eg)
    dv = torch.empty_like(Eg)
    wsb = L.esa_scan_workspace_bytes(nb, T, C, _lib.DTYPE_F16, 16)
    w = torch.empty(wsb, dtype=torch.uint8, device=dev)
    N = nb * T * C
    ms = timeit(lambda: L.esa_gated_scan_fwd(gr.data_ptr(), vr.data_ptr(), 3 * C, _lib.DTYPE_F16,
                                             Eg.data_ptr(), _lib.DTYPE_F16, nb, T, C, 0.8, 0.995, 1, 16,
                                             None, None, w.data_ptr(), wsb, sp))
    out["gated_fwd_f16_16x2048x768_GBps"] = 3 * N * 2 / (ms * 1e-3) / 1e9
    ms = timeit(lambda: L.esa_gated_scan_bwd(gr.data_ptr(), vr.data_ptr(), 3 * C, _lib.DTYPE_F16,
                                             Eg.data_ptr(), dE.data_ptr(), _lib.DTYPE_F16, dg.data_ptr(),
                                             dv.data_ptr(), C, _lib.DTYPE_F16, nb, T, C, 0.8, 0.995, 1, 16,
                                             None, None, w.data_ptr(), wsb, sp))
    out["gated_bwd_f16_16x2048x768_GBps"] = 6 * N * 2 / (ms * 1e-3) / 1e9
    # the layer core (esa_layer_fwd: gated scan, then RMS readout; backward:
    # readout backward, then reverse gated scan), against the bytes a layer
    # must move: forward reads q, g, v and writes E, y (10 bytes an element);
    # backward reads dy, q, g, v, E and writes dq, dg, dv (16 bytes)
    y = torch.empty_like(Eg)
    rstd = torch.empty(nb * T, device=dev)
    dy = torch.randn(nb, T, C, device=dev, generator=g).half()
    dqgv = torch.empty_like(qgv)
    lwb = L.esa_layer_workspace_bytes(nb, T, C, _lib.DTYPE_F16, _lib.DTYPE_F16, _lib.DTYPE_F16)
    lw = torch.empty(lwb, dtype=torch.uint8, device=dev)
    ms = timeit(lambda: L.esa_layer_fwd(qgv.data_ptr(), 3 * C, _lib.DTYPE_F16, Eg.data_ptr(), _lib.DTYPE_F16,
                                        y.data_ptr(), _lib.DTYPE_F16, rstd.data_ptr(), nb, T, C, 0.8, 0.995, 1e-5,
                                        None, None, lw.data_ptr(), lwb, sp))
    out["layer_fwd_f16_16x2048x768_GBps"] = 10 * N * 2 / (ms * 1e-3) / 1e9
    out["layer_fwd_f16_16x2048x768_us"] = ms * 1e3
    ms = timeit(lambda: L.esa_layer_bwd(dy.data_ptr(), _lib.DTYPE_F16, qgv.data_ptr(), 3 * C, _lib.DTYPE_F16,
                                        Eg.data_ptr(), _lib.DTYPE_F16, rstd.data_ptr(), dqgv.data_ptr(), 3 * C, nb,
                                        T, C, 0.8, 0.995, 1e-5, None, None, lw.data_ptr(), lwb, sp))
    out["layer_bwd_f16_16x2048x768_GBps"] = 16 * N * 2 / (ms * 1e-3) / 1e9
    out["layer_bwd_f16_16x2048x768_us"] = ms * 1e3
    return out


# ---------------------------------------------------------------------------
# ESAModel training step (config 3), DDP over the ranks
# ---------------------------------------------------------------------------
def _in_situ_scan(step, dev, n_elem: int, n_layer: int) -> dict | None:
    """GB/s of the fused gated scans inside the training step: one extra step
    after the timed region under torch.profiler (CUDA activity), the device
    time of the forward and reverse scan kernels against their algorithmic
    bytes (forward reads g, v and writes E: 3 x 2 bytes an element; reverse
    reads g, v, E, dE and writes dg, dv: 6 x 2 bytes)."""
    import torch
    try:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step()
            torch.cuda.synchronize(dev)
        fwd = bwd = 0.0
        for k in prof.key_averages():
            name = k.key
            if "scan_kernel" not in name:
                continue
            if "Kind)1" in name:
                fwd += k.device_time_total
            elif "Kind)3" in name:
                bwd += k.device_time_total
        if fwd <= 0 or bwd <= 0:
            return None
        hbm, _ = _peaks()
        f = n_layer * 3 * n_elem * 2 / (fwd * 1e-6) / 1e9
        b = n_layer * 6 * n_elem * 2 / (bwd * 1e-6) / 1e9
        return {"fwd_GBps": f, "bwd_GBps": b, "fwd_frac": f / hbm, "bwd_frac": b / hbm, "unit": "GB/s",
                "source": "torch.profiler device time of one step after the timed region"}
    except Exception as exc:  # the extra figure never blocks the bench line
        return {"error": str(exc)}


def train_leg(ctx) -> dict:
    import torch

    from esa import ESAModel, ESAModelConfig, ops

    args = ctx.args
    dev, ws, rank, local = ctx.dev, ctx.ws, ctx.rank, ctx.local
    steps = max(3, min(args.steps, 10))
    warm = max(3, min(args.warmup, 5))
    torch.manual_seed(1234)
    cfg = ESAModelConfig(vocab_size=32000, block=2048, n_layer=12, head=12, embd=768,
                         backend="thunder", precision="fp16", dropout=0.0, bias=True,
                         tie_embeddings=True, training_compile=bool(args.compile))
    model = ESAModel(cfg, device=f"cuda:{local}")
    model.train()
    n_params = sum(p.numel() for p in model.parameters())
    net = model
    if ws > 1:
        net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local],
                                                        gradient_as_bucket_view=True)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, fused=True)
    scaler = torch.amp.GradScaler("cuda")
    B, T = 16, 2048
    g = torch.Generator().manual_seed(4321 + rank)
    host_ids = torch.randint(0, 32000, (B, T + 1), generator=g).pin_memory()
    ids = torch.empty_like(host_ids, device=dev)
    host_loss = torch.empty((), dtype=torch.float32).pin_memory()

    def step():
        ids.copy_(host_ids, non_blocking=True)
        with torch.autocast("cuda", dtype=torch.float16):
            _, loss = net(ids[:, :-1], ids[:, 1:])
        scaler.scale(loss).backward()
        scaler.step(opt)
        scaler.update()
        opt.zero_grad(set_to_none=True)
        host_loss.copy_(loss.detach().float(), non_blocking=True)

    for _ in range(warm):
        step()
    torch.cuda.synchronize(dev)
    total_ms, _, clk = _timed(ctx, step, steps)
    ops.check_device_status(dev)
    tok = ws * B * T * steps / (total_ms * 1e-3)
    peak, kind = _bf16_peak()
    scan = _in_situ_scan(step, dev, B * T * cfg.embd, cfg.n_layer)
    flops_per_token = 6 * n_params
    out = {
        "metric": "esamodel_train_tokens_per_s", "value": tok, "unit": "tokens/s", "n_gpus": ws,
        "steps": steps, "warmup": warm, "ms_per_step": total_ms / steps, "higher_is_better": True,
        "scaling": "weak", "dtype": "f16", "data": "synthetic tokens, random init",
        "config": {"workload": "ESAModel train step 12L/768/12h, vocab 32000, block 2048, batch 16 "
                               "per GPU, fp16 autocast, GradScaler, AdamW, " + ("DDP" if ws > 1 else "1 GPU"),
                   "compile": bool(args.compile), "params": n_params, "global_batch": B * ws,
                   "seq_len": T, "parallelism": f"dp{ws}", "final_loss": float(host_loss)},
        "roofline": {"bound": "tensor", "achieved": tok * flops_per_token / 1e12 / ws, "peak": peak,
                     "unit": "TFLOP/s", "frac": tok * flops_per_token / 1e12 / ws / peak,
                     "peak_kind": kind, "flops_per_token": flops_per_token, "note": "per GPU (MFU)"},
        "in_situ_scan": scan,
        "e2e": {"value": tok, "unit": "tokens/s", "h2d_bytes_per_step": host_ids.numel() * 8,
                "d2h_bytes_per_step": 4},
        "clocks": clk,
    }
    if ws > 1:
        # what DDP adds: one all-reduce of every gradient (fp32, bucketed and
        # overlapped with the backward by DDP); timed here on its own
        flat = torch.zeros(n_params, dtype=torch.float32, device=dev)
        for _ in range(3):
            ctx.dist.all_reduce(flat)
        ar_ms, _, _ = _timed(ctx, lambda: ctx.dist.all_reduce(flat), 5)
        ar_ms /= 5
        busbw = 2 * (ws - 1) / ws * n_params * 4 / (ar_ms * 1e-3) / 1e9
        out["ddp_allreduce"] = {"bytes": n_params * 4, "ms": ar_ms, "bus_GBps": busbw,
                                "share_of_step": ar_ms / (total_ms / steps),
                                "note": "a standalone NCCL all-reduce of all gradients (fp32); DDP "
                                        "splits it into 25 MB buckets overlapped with the backward"}
        del flat
    del model, net, opt
    torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# Long-sequence scan, T split across the ranks (config 5)
# ---------------------------------------------------------------------------
def sp_leg(ctx) -> dict:
    import torch

    from esa import ops
    from esa.parallel import sequence_parallel_scan

    args = ctx.args
    dev, ws, rank = ctx.dev, ctx.ws, ctx.rank
    steps = max(3, min(args.steps, 10))
    nb, T, H, D = 4, 262144, 32, 64
    Tr = T // ws
    g = torch.Generator(device=dev).manual_seed(9000 + rank)
    A = torch.sigmoid(torch.randn(nb, Tr, H, D, device=dev, generator=g) + 3).to(torch.bfloat16)
    B = (torch.randn(nb, Tr, H, D, device=dev, generator=g) * 0.5).to(torch.bfloat16)
    out_box = {}

    def step(form="single_pass"):
        if ws > 1:
            out_box["E"] = sequence_parallel_scan(A, B, form=form)
        else:
            out_box["E"] = ops.scan(A, B, None, 16)[0]

    # the two-pass form first, for comparison (same inputs, same ranks)
    two_pass_ms = None
    if ws > 1:
        for _ in range(3):
            step("two_pass")
        torch.cuda.synchronize(dev)
        two_total, _, _ = _timed(ctx, lambda: step("two_pass"), steps)
        two_pass_ms = two_total / steps
    for _ in range(3):
        step()
    torch.cuda.synchronize(dev)
    total_ms, _, clk = _timed(ctx, step, steps)
    ms = total_ms / steps
    ops.check_device_status(dev)
    out_box.clear()
    del A, B
    torch.cuda.empty_cache()
    peak, pk = _peaks()
    alg = 3 * nb * T * H * D * 2
    val = alg / (ms * 1e-3) / 1e9
    return {
        "metric": "sp_scan_GBps", "value": val, "unit": "GB/s", "n_gpus": ws, "steps": steps,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
        "data": "synthetic (seeded per rank)",
        "config": {"workload": "long-sequence scan [4,262144,32,64] bf16, T split across ranks",
                   "form": "plain scan of the whole sequence" if ws == 1 else
                   "single pass: slice scan from zero + product of A (stops where it is zero) + NCCL "
                   "all_gather of [2,4,2048] fp32 + rescan of the slice head from the exact incoming state",
                   "parallelism": f"sp{ws}"},
        "two_pass": None if two_pass_ms is None else {
            "ms_per_step": two_pass_ms, "value": alg / (two_pass_ms * 1e-3) / 1e9,
            "form": "slice summary + all_gather + scan from the exact incoming state (5 bytes-per-element "
                    "passes)"},
        "roofline": {"bound": "hbm", "achieved": val / ws, "peak": peak, "unit": "GB/s",
                     "frac": val / ws / peak, "peak_kind": pk, "note": "per GPU, algorithmic 3N bytes"},
        "clocks": clk,
    }


# ---------------------------------------------------------------------------
# Decode (config 4) and the single layer (config 1): N = 1
# ---------------------------------------------------------------------------
def decode_leg(ctx, prec: str = "fp16") -> dict:
    import torch

    from esa import ESAModel, ESAModelConfig, ops

    args = ctx.args
    dev, local = ctx.dev, ctx.local
    torch.manual_seed(1234)
    cfg = ESAModelConfig(vocab_size=32000, n_layer=24, embd=1024, head=16, block=1024, dropout=0.0,
                         precision=prec)
    model = ESAModel(cfg, device=f"cuda:{local}").eval()
    if prec == "fp16":
        model = model.half()
    n_params = sum(p.numel() for p in model.parameters())
    wbytes = sum(p.numel() * p.element_size() for p in model.parameters())
    results = {}
    clocks = ClockSampler(local).start()
    for batch in (1, 64):
        g = torch.Generator().manual_seed(77 + batch)
        ids = torch.randint(0, 32000, (batch, 512), generator=g).to(dev)
        for _ in range(max(1, min(args.warmup, 3))):
            model.generate(input_ids=ids, seek=16, prefill="thunder_16", temperature=0.0,
                           compile=False, decode_graph=True)
        res = model.generate(input_ids=ids, seek=256, prefill="thunder_16", temperature=0.0,
                             compile=False, decode_graph=True, stats=True)
        st = res.stats
        results[f"batch{batch}"] = {
            "prefill_tok_s": batch * st.prefill_tokens / st.prefill_seconds,
            "decode_tok_s": batch * st.decode_tok_s,
            "decode_ms_per_token": 1e3 * st.decode_seconds / max(1, st.decode_steps),
            "weight_GBps": wbytes * st.decode_tok_s / 1e9,
        }
    clk = clocks.stop()
    ops.check_device_status(dev)
    del model
    torch.cuda.empty_cache()
    peak, pk = _peaks()
    b1 = results["batch1"]
    return {
        "metric": "esamodel_decode_tokens_per_s", "value": b1["decode_tok_s"], "unit": "tokens/s",
        "n_gpus": 1, "steps": 256, "ms_per_step": b1["decode_ms_per_token"], "higher_is_better": True,
        "scaling": "replicas", "dtype": "f16" if prec == "fp16" else "f32",
        "data": "synthetic prompt, random init",
        "config": {"workload": "ESAModel 24L/1024/16h vocab 32000: 512-token thunder_16 prefill + "
                               "256 greedy ESA-Lightning tokens (CUDA-graph decode)",
                   "precision": prec, "params": n_params, "weight_bytes": wbytes, **results},
        "roofline": {"bound": "hbm", "achieved": b1["weight_GBps"], "peak": peak, "unit": "GB/s",
                     "frac": b1["weight_GBps"] / peak, "peak_kind": pk,
                     "note": "batch-1 decode reads every weight once per token"},
        "clocks": clk,
        "timing": "GenerationStats (host perf_counter around device-synchronised prefill and decode)",
    }


def layer_leg(ctx, with_cpu: bool = True) -> dict:
    import torch

    from esa import ESA, ops

    args = ctx.args
    dev = ctx.dev
    torch.manual_seed(1234)
    lay = ESA(embd=128, head=4, batch=16, block=1024, backend="thunder", precision="fp32", dropout=0.0,
              device=dev)
    x = torch.randn(16, 1024, 128, generator=torch.Generator().manual_seed(1234)).to(dev)

    def step():
        xi = x.detach().requires_grad_(True)
        lay(xi).sum().backward()

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    steps = max(10, min(args.steps, 50))
    total_ms, _, clk = _timed(ctx, step, steps)
    ms = total_ms / steps
    ops.check_device_status(dev)
    line = {"metric": "esa_layer_fwd_bwd_ms", "value": ms, "unit": "ms", "n_gpus": 1,
            "steps": steps, "ms_per_step": ms, "higher_is_better": False,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": "ESA(embd=128, head=4, thunder, fp32) forward + backward of sum(y), "
                                   "x [16,1024,128]"},
            "clocks": clk}
    if with_cpu:
        from oracle import oracle
        torch.set_num_threads(os.cpu_count() or 1)
        xc = x.cpu().requires_grad_(True)
        qw = lay.layer.qgv.weight.detach().cpu().requires_grad_(True)
        ow = lay.layer.out_proj.weight.detach().cpu().requires_grad_(True)
        times = []
        for _ in range(3):
            t0 = time.perf_counter()
            oracle.pulse_layer_port(xc, qw, ow, head=4).sum().backward()
            times.append(time.perf_counter() - t0)
        line["cpu_baseline"] = {"value": statistics.median(times) * 1e3, "unit": "ms",
                                "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": "the reference's Pulse layer restated in torch (oracle."
                                          "pulse_layer_port: fp32, sequential scan, autograd), forward + "
                                          "backward of sum(y) on the same x and weights, median of 3"}
    return line


# ---------------------------------------------------------------------------
# The unmodified reference's own GPU paths (Flare Triton scan, Thunder eager
# and under torch.compile), run in a child process that imports the reference
# package from baseline/_ref
# ---------------------------------------------------------------------------
def gpu_comparators_child() -> None:
    import torch

    sys.path.insert(0, str(REF_INSTALL))
    import esa  # the reference package
    from esa.backends.flare import flare_scan
    from esa.backends.thunder import thunder_scan
    assert str(REF_INSTALL) in esa.__file__, esa.__file__
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1234)
    A = torch.sigmoid(torch.randn(SHAPE, device=dev, generator=g) * 2 + 2).half()
    B = torch.randn(SHAPE, device=dev, generator=g).half()
    nbytes = 3 * A.numel() * 2
    out = {"shape_BTHD": list(SHAPE), "dtype": "f16", "source": str(REF_INSTALL.relative_to(ROOT))}

    def timeit(fn, k):
        fn()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(k):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / k

    def record(name, fn, k):
        try:
            t0 = time.perf_counter()
            fn()  # first call: Triton / Inductor compilation
            torch.cuda.synchronize()
            first = time.perf_counter() - t0
            ms = timeit(fn, k)
            out[name] = {"ms": ms, "GBps": nbytes / (ms * 1e-3) / 1e9, "first_call_s": first}
        except Exception as exc:
            out[name] = {"error": f"{type(exc).__name__}: {exc}"[:300]}

    with torch.no_grad():
        record("flare_triton_scan", lambda: flare_scan(A, B), 10)
        record("thunder_eager_c16", lambda: thunder_scan(A, B, compass=16), 5)
        compiled = torch.compile(thunder_scan)
        record("thunder_torch_compile_c16", lambda: compiled(A, B, compass=16), 10)
    print(json.dumps(out), flush=True)


def comparators_leg(timeout_s: int = 420) -> dict:
    if not (REF_INSTALL / "esa").exists():
        return {"unavailable": "reference not installed in baseline/_ref"}
    env = dict(os.environ)
    env.pop("PYTHONPATH", None)
    try:
        r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--gpu-comparators"], env=env,
                           capture_output=True, text=True, timeout=timeout_s, cwd=str(ROOT))
    except subprocess.TimeoutExpired:
        return {"unavailable": f"comparator run exceeded {timeout_s} s"}
    for line in reversed(r.stdout.strip().splitlines()):
        if line.startswith("{"):
            d = json.loads(line)
            hbm, _ = _peaks()
            for v in d.values():
                if isinstance(v, dict) and "GBps" in v:
                    v["frac_of_measured_hbm"] = v["GBps"] / hbm
            return d
    return {"unavailable": f"comparator run rc={r.returncode}: {(r.stderr or '')[-300:]}"}


# ---------------------------------------------------------------------------
# Fixed kernel workloads for ncu (python bench.py --profile-workload NAME):
# four iterations of one kernel family, so a profiler can skip the first
# launches and capture one
# ---------------------------------------------------------------------------
PROFILE_WORKLOADS = ("rev", "gated", "long", "readout", "layer", "layernorm", "train", "decode")


def profile_workload(name: str, iters: int = 4) -> None:
    import torch

    from esa import ops

    if name not in PROFILE_WORKLOADS:
        raise SystemExit(f"unknown workload {name!r}; one of {PROFILE_WORKLOADS}")
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape, dtype=torch.float16):
        return torch.randn(*shape, device=dev, generator=g).to(dtype)

    if name == "train":
        from torch.profiler import ProfilerActivity, profile

        from esa import ESAModel, ESAModelConfig
        torch.manual_seed(1234)
        cfg = ESAModelConfig(vocab_size=32000, block=2048, n_layer=12, head=12, embd=768, backend="thunder",
                             precision="fp16", dropout=0.0, bias=True, tie_embeddings=True,
                             training_compile=False)
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
        for t, n, key in rows[:30]:
            print(f"{t / 2:10.1f} us {100 * t / total:5.1f} % {n // 2:4d} launches  {key[:100]}")
        return
    if name == "decode":
        # eager batch-1 decode steps of the 24-layer / 1024-wide fp16 model
        from esa import ESAModel, ESAModelConfig
        torch.manual_seed(1234)
        cfg = ESAModelConfig(vocab_size=32000, n_layer=24, embd=1024, head=16, block=1024, dropout=0.0,
                             precision="fp16")
        model = ESAModel(cfg, device="cuda").eval().half()
        token = torch.zeros(1, dtype=torch.long, device=dev)
        states = torch.zeros(24, 1, 16, 64, dtype=torch.float16, device=dev)
        pos = torch.tensor(3, device=dev)
        with torch.inference_mode():
            for _ in range(iters):
                logits, states = model.lightning_step(token, states, pos)
                token = torch.argmax(logits, dim=-1)
        torch.cuda.synchronize()
        ops.check_device_status()
        print("ok", name)
        return
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
    elif name == "long":
        # a quarter of the long-sequence shape: the single-pass chained scan
        A = torch.sigmoid(rnd(4, 65536, 32, 64, dtype=torch.float32) + 3).to(torch.bfloat16)
        B = (rnd(4, 65536, 32, 64, dtype=torch.float32) * 0.5).to(torch.bfloat16)
        for _ in range(iters):
            ops.scan(A, B, None, 16)
    elif name in ("readout", "layer"):
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
    print("ok", name)


# ---------------------------------------------------------------------------
def run_ours(args) -> None:
    import torch

    ctx = Ctx(args)
    wl = args.workload
    try:
        if wl == "train":
            line = train_leg(ctx)
        elif wl == "sp":
            line = sp_leg(ctx)
        elif wl == "decode":
            line = decode_leg(ctx, args.precision)
        elif wl == "layer":
            line = layer_leg(ctx, with_cpu=not args.no_cpu)
        else:
            line = scan_leg(ctx)
            torch.cuda.empty_cache()
            if wl == "all":
                line["esamodel_train"] = train_leg(ctx)
                line["sp_scan"] = sp_leg(ctx)
                if ctx.ws == 1:
                    for key, fn in (("decode", lambda: decode_leg(ctx)),
                                    ("layer", lambda: layer_leg(ctx, with_cpu=not args.no_cpu)),
                                    ("gpu_comparators", comparators_leg)):
                        try:  # rank-local legs: an error is reported, not fatal
                            line[key] = fn()
                        except Exception as exc:
                            line[key] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
            if ctx.ws == 1 and not args.no_cpu and ctx.rank == 0:
                try:
                    line["cpu_baseline"] = cpu_baseline()
                except Exception as exc:  # the CPU baseline never blocks the GPU line
                    line["cpu_baseline"] = {"error": str(exc)}
        if ctx.rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        ctx.close()


def main() -> None:
    if "--gpu-comparators" in sys.argv:
        gpu_comparators_child()
        return
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["all", "scan", "train", "decode", "layer", "sp"], default="all",
                    help="all (default: the headline plus every workload) or one workload's own line")
    ap.add_argument("--compile", action="store_true", help="train: torch.compile the forward")
    ap.add_argument("--precision", default="fp16", choices=["fp16", "fp32"], help="decode precision")
    ap.add_argument("--quick", action="store_true", help="skip the secondary figures")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline legs")
    ap.add_argument("--profile-workload", choices=PROFILE_WORKLOADS, default=None,
                    help="run one fixed kernel workload for a profiler and exit")
    args = ap.parse_args()
    if args.profile_workload:
        profile_workload(args.profile_workload)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
