"""CPU oracle for the ESA recurrence -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this module, always as the checker or as the timed CPU
baseline, never as part of the product path (the ``esa`` package never imports
it and has no CPU fallback).

Contents
--------
* ctypes bindings to ``liboracle_esa.so`` (``esa_oracle.c``): fp64 forward scan,
  reverse scan, gate prologue / epilogue, RMS readout and one Lightning decode
  step, each a sequential restatement of the reference (file:line cited in the C
  source).
* ``OracleScan`` -- a torch autograd Function over the fp64 C scan, so that
  layer-level gradients come from torch autograd around an exact scan.
* ``pulse_layer_forward`` -- fp64 restatement of ``PulseESA.forward``
  (esa/backends/pulse.py:69-98, identical math to ThunderESA.forward,
  esa/backends/thunder.py:264-316).
* ``thunder_scan_port`` -- a torch restatement of the reference's chunked
  Thunder scan (esa/backends/thunder.py:70-159): pad T to a multiple of the
  chunk, run the local recurrence of every chunk in parallel, scan the chunk
  summaries by recursive doubling (thunder.py:13-67), then combine.  It is the
  timed CPU baseline ("port") because it has the reference's cost structure.

Parity pin: tests/test_oracle.py checks all of these against fixtures that
tests/golden/make_golden.py produced by running the reference package.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np
import torch

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "liboracle_esa.so"
_lib = None

_dp = ctypes.POINTER(ctypes.c_double)
_fp = ctypes.POINTER(ctypes.c_float)
_i64 = ctypes.c_int64


def build() -> Path:
    """Compile liboracle_esa.so with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(_LIB_PATH))
        L.esa_oracle_scan_fwd.argtypes = [_dp, _dp, _dp, _i64, _i64, _i64, _dp]
        L.esa_oracle_scan_rev.argtypes = [_dp, _dp, _dp, _dp, _dp, _i64, _i64, _i64, _dp, _dp]
        L.esa_oracle_gate.argtypes = [_dp, _dp, _dp, _dp, _i64, ctypes.c_double, ctypes.c_double]
        L.esa_oracle_gate_bwd.argtypes = [_dp, _dp, _dp, _dp, _dp, _dp, _i64,
                                          ctypes.c_double, ctypes.c_double]
        L.esa_oracle_lightning_step.argtypes = [_dp, _dp, _dp, _dp, _i64, _i64,
                                                ctypes.c_double, ctypes.c_double, ctypes.c_double]
        L.esa_oracle_readout.argtypes = [_dp, _dp, _dp, _i64, _i64, ctypes.c_double]
        L.esa_oracle_scan_fwd_f32.argtypes = [_fp, _fp, _fp, _i64, _i64, _i64]
        for f in ("esa_oracle_scan_fwd", "esa_oracle_scan_rev", "esa_oracle_gate",
                  "esa_oracle_gate_bwd", "esa_oracle_lightning_step", "esa_oracle_readout",
                  "esa_oracle_scan_fwd_f32"):
            getattr(L, f).restype = None
        _lib = L
    return _lib


def _f64(x) -> np.ndarray:
    if isinstance(x, torch.Tensor):
        x = x.detach().cpu()
        if x.dtype != torch.float64:
            x = x.to(torch.float64)
        x = x.numpy()
    return np.ascontiguousarray(x, dtype=np.float64)


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(_dp)


def _dims(shape) -> tuple[int, int, int]:
    if len(shape) != 4:
        raise ValueError(f"expected [B,T,H,D], got {tuple(shape)}")
    b, t, h, d = shape
    return b, t, h * d


def scan_fwd(A, B, e0=None) -> np.ndarray:
    """fp64 E_t = A_t E_{t-1} + B_t over [B,T,H,D] (pulse.py:25-31)."""
    A, B = _f64(A), _f64(B)
    if A.shape != B.shape:
        raise ValueError("A and B must have the same shape")
    nb, T, hd = _dims(A.shape)
    E = np.empty_like(A)
    e0a = None if e0 is None else _f64(e0).reshape(nb * hd)
    lib().esa_oracle_scan_fwd(_ptr(A), _ptr(B), _ptr(E), nb, T, hd, _ptr(e0a))
    return E


def scan_rev(A, E, dE, e0=None):
    """fp64 reverse scan: returns (dA, dB, de0) (flare.py:66-78 math)."""
    A, E, dE = _f64(A), _f64(E), _f64(dE)
    nb, T, hd = _dims(A.shape)
    dA, dB = np.empty_like(A), np.empty_like(A)
    de0 = np.empty((nb, hd), dtype=np.float64)
    e0a = None if e0 is None else _f64(e0).reshape(nb * hd)
    lib().esa_oracle_scan_rev(_ptr(A), _ptr(E), _ptr(dE), _ptr(dA), _ptr(dB),
                              nb, T, hd, _ptr(e0a), _ptr(de0))
    return dA, dB, de0


def gate(g, v, gmin=0.80, gmax=0.995):
    g, v = _f64(g), _f64(v)
    A, Bw = np.empty_like(g), np.empty_like(g)
    lib().esa_oracle_gate(_ptr(g), _ptr(v), _ptr(A), _ptr(Bw), g.size, gmin, gmax)
    return A, Bw


def gate_bwd(g, v, dA, dB, gmin=0.80, gmax=0.995):
    g, v, dA, dB = _f64(g), _f64(v), _f64(dA), _f64(dB)
    dg, dv = np.empty_like(g), np.empty_like(g)
    lib().esa_oracle_gate_bwd(_ptr(g), _ptr(v), _ptr(dA), _ptr(dB), _ptr(dg), _ptr(dv),
                              g.size, gmin, gmax)
    return dg, dv


def lightning_step(qgv, state, gmin=0.80, gmax=0.995, eps=1e-5):
    """One decode step: returns (new_state [B,C], z [B,C]) with z the out_proj input."""
    qgv = _f64(qgv)
    nb, c3 = qgv.shape
    C = c3 // 3
    st = _f64(state).reshape(nb, C)
    ns, z = np.empty_like(st), np.empty_like(st)
    lib().esa_oracle_lightning_step(_ptr(qgv), _ptr(st), _ptr(ns), _ptr(z), nb, C,
                                    gmin, gmax, eps)
    return ns, z


def readout(q, E, eps=1e-5):
    q, E = _f64(q), _f64(E)
    C = E.shape[-1]
    z = np.empty_like(E)
    lib().esa_oracle_readout(_ptr(q), _ptr(E), _ptr(z), E.size // C, C, eps)
    return z


def readout_bwd(q, E, rstd, dy):
    """fp64 gradient of the readout y = sigmoid(q) * E * r, r = rsqrt(mean_C(E^2)
    + eps) given per row as `rstd` (thunder.py:304-311, differentiated through
    r as autograd does): dq = dy n s (1 - s), dE = r (dy s - n mean_C(dy s n))
    with s = sigmoid(q), n = E r.  Returns (dq, dE)."""
    q, E, dy = _f64(q), _f64(E), _f64(dy)
    r = _f64(rstd).reshape(E.shape[:-1] + (1,))
    s = 1.0 / (1.0 + np.exp(-q))
    n = E * r
    t1 = dy * s
    dq = t1 * n * (1.0 - s)
    dE = r * (t1 - n * np.mean(t1 * n, axis=-1, keepdims=True))
    return dq, dE


def scan_fwd_f32_scalar(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """Single-threaded fp32 scalar scan (a timed CPU baseline)."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    nb, T, hd = _dims(A.shape)
    E = np.empty_like(A)
    lib().esa_oracle_scan_fwd_f32(A.ctypes.data_as(_fp), B.ctypes.data_as(_fp),
                                  E.ctypes.data_as(_fp), nb, T, hd)
    return E


class OracleScan(torch.autograd.Function):
    """Exact fp64 scan with its exact reverse-scan gradient (CPU tensors)."""

    @staticmethod
    def forward(ctx, A, B):
        E = torch.from_numpy(scan_fwd(A, B))
        ctx.save_for_backward(A.detach(), E)
        return E

    @staticmethod
    def backward(ctx, dE):
        A, E = ctx.saved_tensors
        dA, dB, _ = scan_rev(A, E, dE)
        return torch.from_numpy(dA), torch.from_numpy(dB)


def pulse_layer_forward(x, qgv_w, out_w, head, *, gmin=0.80, gmax=0.995, eps=1e-5):
    """fp64 restatement of PulseESA/ThunderESA forward (pulse.py:69-98,
    thunder.py:264-316) with an exact scan; differentiable via torch autograd."""
    Bsz, T, C = x.shape
    D = C // head
    qgv = x @ qgv_w.t()
    q, g, v = qgv.split(C, dim=-1)
    A = gmin + (gmax - gmin) * torch.sigmoid(g)
    Bw = (1.0 - A) * torch.tanh(v)
    E = OracleScan.apply(A.reshape(Bsz, T, head, D).contiguous(),
                         Bw.reshape(Bsz, T, head, D).contiguous())
    E = E.reshape(Bsz, T, C)
    E = E * torch.rsqrt(E.pow(2).mean(dim=-1, keepdim=True) + eps)
    y = torch.sigmoid(q) * E
    return y @ out_w.t()


def thunder_scan_port(A: torch.Tensor, B: torch.Tensor, compass: int = 16) -> torch.Tensor:
    """Torch restatement of the reference chunked scan (thunder.py:70-159).

    Steps: pad T up to a multiple of ``compass`` with identity steps (A=1, B=0);
    run the local recurrence of all chunks at once, keeping each step's local
    state and running product of A; scan the per-chunk (product, end state)
    pairs by recursive doubling with (a2, b2) o (a1, b1) = (a2 a1, a2 b1 + b2);
    shift to get each chunk's incoming state and combine
    E = local_state + running_product * incoming.
    """
    nb, T, H, D = A.shape
    pad = (-T) % compass
    if pad:
        A = torch.cat([A, A.new_ones(nb, pad, H, D)], dim=1)
        B = torch.cat([B, B.new_zeros(nb, pad, H, D)], dim=1)
    G = A.shape[1] // compass
    a5 = A.view(nb, G, compass, H, D)
    b5 = B.view(nb, G, compass, H, D)
    loc = torch.empty_like(b5)
    prod = torch.empty_like(a5)
    s = b5[:, :, 0]
    p = a5[:, :, 0]
    loc[:, :, 0] = s
    prod[:, :, 0] = p
    for i in range(1, compass):
        s = a5[:, :, i] * s + b5[:, :, i]
        p = a5[:, :, i] * p
        loc[:, :, i] = s
        prod[:, :, i] = p
    ca = prod[:, :, -1].clone()
    cb = loc[:, :, -1].clone()
    step = 1
    while step < G:
        na = ca.clone()
        nbv = cb.clone()
        na[:, step:] = ca[:, step:] * ca[:, :-step]
        nbv[:, step:] = ca[:, step:] * cb[:, :-step] + cb[:, step:]
        ca, cb = na, nbv
        step *= 2
    incoming = torch.zeros_like(cb)
    incoming[:, 1:] = cb[:, :-1]
    E = (loc + prod * incoming.unsqueeze(2)).reshape(nb, G * compass, H, D)
    return E[:, :T]


def pulse_scan_port(A: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """Torch restatement of the reference's sequential scan (pulse.py:12-31):
    one state update per step in the input dtype, the steps stacked along T.
    Differentiable through torch autograd, as the reference's is."""
    state = torch.zeros_like(A[:, 0])
    outs = []
    for t in range(A.shape[1]):
        state = A[:, t] * state + B[:, t]
        outs.append(state)
    return torch.stack(outs, dim=1)


def pulse_layer_port(x, qgv_w, out_w, head, *, gmin=0.80, gmax=0.995, eps=1e-5):
    """Torch restatement of PulseESA.forward (pulse.py:69-98) in the input
    dtype with the sequential scan of ``pulse_scan_port``: the reference's CPU
    layer (the timed CPU baseline of the layer workload)."""
    Bsz, T, C = x.shape
    D = C // head
    qgv = x @ qgv_w.t()
    q, g, v = qgv.split(C, dim=-1)
    A = gmin + (gmax - gmin) * torch.sigmoid(g)
    Bw = (1.0 - A) * torch.tanh(v)
    E = pulse_scan_port(A.reshape(Bsz, T, head, D), Bw.reshape(Bsz, T, head, D)).reshape(Bsz, T, C)
    E = E * torch.rsqrt(E.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (torch.sigmoid(q) * E) @ out_w.t()
