"""PyTorch operators over the C-ABI library (``libesa_b200.so``).

Each operator is a ``torch.library.custom_op`` with a fake (meta) kernel and,
where the reference path is differentiable, an autograd formula, so that it is
opaque to ``torch.compile`` (no graph break inside) and capturable in CUDA
graphs (fixed workspace, no host synchronisation).  Work is enqueued on the
current CUDA stream.  CPU tensors raise: there is no CPU fallback.

Operators
---------
``esa_b200::scan``                 E, e_last = scan(A, B, e0)         (kernel a)
``esa_b200::scan_backward``        dA, dB, de0                        (kernel b, bare)
``esa_b200::gated_scan``           E, e_last from gate/value logits   (kernel a + gate prologue)
``esa_b200::gated_scan_backward``  d gate, d value, de0               (kernel b + gate epilogue)
``esa_b200::lightning_step``       new state, out_proj input          (kernel c)
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from . import _lib

_CODES = {
    torch.float16: _lib.DTYPE_F16,
    torch.bfloat16: _lib.DTYPE_BF16,
    torch.float32: _lib.DTYPE_F32,
    torch.float64: _lib.DTYPE_F64,
}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _CODES[dt]
    except KeyError:
        raise TypeError(f"ESA kernels support float16/bfloat16/float32/float64, got {dt}") from None


def acc_dtype(*dts: torch.dtype) -> torch.dtype:
    return torch.float64 if torch.float64 in dts else torch.float32


def _widest(*dts: torch.dtype) -> torch.dtype:
    return max(dts, key=lambda d: (torch.empty((), dtype=d).element_size(), d == torch.float64))


def _require_cuda(who: str, *ts: Optional[Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                f"{who}: the ESA B200 kernels need CUDA tensors (there is no CPU fallback); "
                f"got a tensor on {t.device}"
            )


def _stream(t: Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t: Optional[Tensor]):
    return None if t is None else t.data_ptr()


def _workspace(nb: int, T: int, hd: int, dt: torch.dtype, compass: int, device) -> Tensor:
    n = _lib.lib().esa_scan_workspace_bytes(nb, T, hd, dtype_code(dt), int(compass))
    if n == 0 and nb * T * hd > 0:
        raise ValueError("invalid scan problem")
    return torch.empty(max(int(n), 256), dtype=torch.uint8, device=device)


def _rows(t: Tensor) -> tuple[Tensor, int]:
    """A [B, T, C] view with unit channel stride and uniformly spaced (b, t)
    rows, and its row stride in elements (copies the tensor if it is not)."""
    B, T, C = t.shape
    s0, s1, s2 = t.stride()
    if s2 == 1 and (B <= 1 or s0 == T * s1) and s1 >= C:
        return t, (s1 if T > 1 else (s0 if B > 1 else C))
    t = t.contiguous()
    return t, C


def _state_arg(e0: Optional[Tensor], nb: int, hd: int, acc: torch.dtype) -> Optional[Tensor]:
    if e0 is None:
        return None
    return e0.reshape(nb, hd).to(acc).contiguous()


# --------------------------------------------------------------------------
# Forward / reverse scan over materialised A, B  (thunder_scan, pulse_scan)
# --------------------------------------------------------------------------
@torch.library.custom_op("esa_b200::scan", mutates_args=())
def scan(A: Tensor, B: Tensor, e0: Optional[Tensor], compass: int) -> tuple[Tensor, Tensor]:
    """E_t = A_t E_{t-1} + B_t over [B,T,H,D]; returns (E, E_{T-1} in the acc dtype)."""
    _require_cuda("esa scan", A, B, e0)
    nb, T, H, D = A.shape
    hd = H * D
    A = A.contiguous()
    B = B.contiguous()
    acc = acc_dtype(A.dtype)
    E = torch.empty_like(A)
    e0c = _state_arg(e0, nb, hd, acc)
    if T == 0 or nb * hd == 0:
        e_last = e0c.clone() if e0c is not None else A.new_zeros(nb, hd, dtype=acc)
        return E, e_last
    e_last = torch.empty(nb, hd, dtype=acc, device=A.device)
    ws = _workspace(nb, T, hd, A.dtype, compass, A.device)
    rc = _lib.lib().esa_scan_fwd(A.data_ptr(), B.data_ptr(), E.data_ptr(), nb, T, hd,
                                 dtype_code(A.dtype), int(compass), _ptr(e0c), e_last.data_ptr(),
                                 ws.data_ptr(), ws.numel(), _stream(A))
    _lib.check(rc, "esa_scan_fwd")
    return E, e_last


@scan.register_fake
def _(A, B, e0, compass):
    nb, T, H, D = A.shape
    return torch.empty_like(A, memory_format=torch.contiguous_format), \
        A.new_empty(nb, H * D, dtype=acc_dtype(A.dtype))


@torch.library.custom_op("esa_b200::scan_backward", mutates_args=())
def scan_backward(A: Tensor, E: Tensor, dE: Tensor, e0: Optional[Tensor],
                  compass: int) -> tuple[Tensor, Tensor, Tensor]:
    """Reverse scan: (dA, dB, de0) for upstream gradient dE (kernel b, bare)."""
    _require_cuda("esa scan backward", A, E, dE, e0)
    nb, T, H, D = A.shape
    hd = H * D
    A, E, dE = A.contiguous(), E.contiguous(), dE.to(A.dtype).contiguous()
    acc = acc_dtype(A.dtype)
    dA = torch.empty_like(A)
    dB = torch.empty_like(A)
    de0 = torch.zeros(nb, hd, dtype=acc, device=A.device)
    if T == 0 or nb * hd == 0:
        return dA, dB, de0
    e0c = _state_arg(e0, nb, hd, acc)
    ws = _workspace(nb, T, hd, A.dtype, compass, A.device)
    rc = _lib.lib().esa_scan_rev(A.data_ptr(), E.data_ptr(), dE.data_ptr(), dA.data_ptr(),
                                 dB.data_ptr(), nb, T, hd, dtype_code(A.dtype), int(compass),
                                 _ptr(e0c), de0.data_ptr(), ws.data_ptr(), ws.numel(), _stream(A))
    _lib.check(rc, "esa_scan_rev")
    return dA, dB, de0


@scan_backward.register_fake
def _(A, E, dE, e0, compass):
    nb, T, H, D = A.shape
    c = torch.contiguous_format
    return (torch.empty_like(A, memory_format=c), torch.empty_like(A, memory_format=c),
            A.new_empty(nb, H * D, dtype=acc_dtype(A.dtype)))


def _scan_setup(ctx, inputs, output):
    A, B, e0, compass = inputs
    E, _ = output
    ctx.save_for_backward(A, E, e0)
    ctx.compass = compass
    ctx.has_e0 = e0 is not None
    ctx.e0_dtype = None if e0 is None else e0.dtype
    ctx.b_dtype = B.dtype


def _scan_bwd(ctx, dE, de_last):
    A, E, e0 = ctx.saved_tensors
    if dE is None:
        dE = torch.zeros_like(E)
    if de_last is not None:
        dE = dE.clone()
        dE[:, -1] += de_last.reshape(dE[:, -1].shape).to(dE.dtype)
    dA, dB, de0 = scan_backward(A, E, dE, e0, ctx.compass)
    return (dA, dB.to(ctx.b_dtype),
            de0.reshape(e0.shape).to(ctx.e0_dtype) if ctx.has_e0 else None, None)


torch.library.register_autograd("esa_b200::scan", _scan_bwd, setup_context=_scan_setup)


@torch.library.custom_op("esa_b200::scan_summary", mutates_args=())
def scan_summary(A: Tensor, B: Tensor, e0: Optional[Tensor]) -> tuple[Tensor, Tensor]:
    """Per-channel (E_{T-1}, prod_t A_t) of a time slice, [B, H*D] in the acc
    dtype; reads A and B once and writes no per-step output."""
    _require_cuda("esa scan summary", A, B, e0)
    nb, T, H, D = A.shape
    hd = H * D
    A = A.contiguous()
    B = B.to(A.dtype).contiguous()
    acc = acc_dtype(A.dtype)
    e0c = _state_arg(e0, nb, hd, acc)
    if T == 0 or nb * hd == 0:
        e_last = e0c.clone() if e0c is not None else A.new_zeros(nb, hd, dtype=acc)
        return e_last, A.new_ones(nb, hd, dtype=acc)
    e_last = torch.empty(nb, hd, dtype=acc, device=A.device)
    prod = torch.empty(nb, hd, dtype=acc, device=A.device)
    ws = _workspace(nb, T, hd, A.dtype, 16, A.device)
    rc = _lib.lib().esa_scan_summary(A.data_ptr(), B.data_ptr(), nb, T, hd, dtype_code(A.dtype),
                                     _ptr(e0c), e_last.data_ptr(), prod.data_ptr(), ws.data_ptr(),
                                     ws.numel(), _stream(A))
    _lib.check(rc, "esa_scan_summary")
    return e_last, prod


@scan_summary.register_fake
def _(A, B, e0):
    nb, T, H, D = A.shape
    acc = acc_dtype(A.dtype)
    return A.new_empty(nb, H * D, dtype=acc), A.new_empty(nb, H * D, dtype=acc)


# --------------------------------------------------------------------------
# Gated scan: gate prologue fused into the forward, gate epilogue fused into
# the reverse scan (ThunderESA.forward, esa_prefill)
# --------------------------------------------------------------------------
@torch.library.custom_op("esa_b200::gated_scan", mutates_args=())
def gated_scan(gate_raw: Tensor, value_raw: Tensor, e0: Optional[Tensor], gate_min: float,
               gate_max: float, compass: int, scan_dtype: torch.dtype) -> tuple[Tensor, Tensor]:
    """E [B,T,C] in scan_dtype from gate/value logits [B,T,C] (row-strided views
    allowed); returns (E, E_{T-1} in the acc dtype)."""
    _require_cuda("esa gated scan", gate_raw, value_raw, e0)
    if gate_raw.shape != value_raw.shape or gate_raw.dim() != 3:
        raise ValueError(f"gate/value logits must be the same [B,T,C], got {tuple(gate_raw.shape)} "
                         f"and {tuple(value_raw.shape)}")
    if gate_raw.dtype != value_raw.dtype:
        raise TypeError("gate/value logits must share a dtype")
    nb, T, C = gate_raw.shape
    g, rs_g = _rows(gate_raw)
    v, rs_v = _rows(value_raw)
    if rs_g != rs_v:
        g, v = g.contiguous(), v.contiguous()
        rs_g = rs_v = C
    # the kernels accumulate in fp64 when any operand is fp64
    acc = acc_dtype(scan_dtype, g.dtype)
    E = torch.empty(nb, T, C, dtype=scan_dtype, device=gate_raw.device)
    e0c = _state_arg(e0, nb, C, acc)
    if T == 0 or nb * C == 0:
        e_last = e0c.clone() if e0c is not None else E.new_zeros(nb, C, dtype=acc)
        return E, e_last
    e_last = torch.empty(nb, C, dtype=acc, device=E.device)
    ws = _workspace(nb, T, C, _widest(g.dtype, scan_dtype), compass, E.device)
    rc = _lib.lib().esa_gated_scan_fwd(g.data_ptr(), v.data_ptr(), rs_g, dtype_code(g.dtype),
                                       E.data_ptr(), dtype_code(scan_dtype), nb, T, C,
                                       float(gate_min), float(gate_max), 1, int(compass), _ptr(e0c),
                                       e_last.data_ptr(), ws.data_ptr(), ws.numel(), _stream(E))
    _lib.check(rc, "esa_gated_scan_fwd")
    return E, e_last


@gated_scan.register_fake
def _(gate_raw, value_raw, e0, gate_min, gate_max, compass, scan_dtype):
    nb, T, C = gate_raw.shape
    return (gate_raw.new_empty(nb, T, C, dtype=scan_dtype),
            gate_raw.new_empty(nb, C, dtype=acc_dtype(scan_dtype, gate_raw.dtype)))


@torch.library.custom_op("esa_b200::gated_scan_backward", mutates_args=())
def gated_scan_backward(gate_raw: Tensor, value_raw: Tensor, E: Tensor, dE: Tensor,
                        e0: Optional[Tensor], gate_min: float, gate_max: float,
                        compass: int) -> tuple[Tensor, Tensor, Tensor]:
    """(d gate_raw, d value_raw, de0) -- reverse scan with the gate chain rule fused."""
    _require_cuda("esa gated scan backward", gate_raw, value_raw, E, dE, e0)
    nb, T, C = gate_raw.shape
    g, rs_g = _rows(gate_raw)
    v, rs_v = _rows(value_raw)
    if rs_g != rs_v:
        g, v = g.contiguous(), v.contiguous()
        rs_g = C
    E = E.contiguous()
    dE = dE.to(E.dtype).contiguous()
    acc = acc_dtype(E.dtype, g.dtype)
    dg = torch.empty(nb, T, C, dtype=g.dtype, device=g.device)
    dv = torch.empty(nb, T, C, dtype=g.dtype, device=g.device)
    de0 = torch.zeros(nb, C, dtype=acc, device=g.device)
    if T == 0 or nb * C == 0:
        return dg, dv, de0
    e0c = _state_arg(e0, nb, C, acc)
    ws = _workspace(nb, T, C, _widest(g.dtype, E.dtype), compass, g.device)
    rc = _lib.lib().esa_gated_scan_bwd(g.data_ptr(), v.data_ptr(), rs_g, dtype_code(g.dtype),
                                       E.data_ptr(), dE.data_ptr(), dtype_code(E.dtype),
                                       dg.data_ptr(), dv.data_ptr(), C, dtype_code(g.dtype),
                                       nb, T, C, float(gate_min), float(gate_max), 1, int(compass),
                                       _ptr(e0c), de0.data_ptr(), ws.data_ptr(), ws.numel(),
                                       _stream(g))
    _lib.check(rc, "esa_gated_scan_bwd")
    return dg, dv, de0


@gated_scan_backward.register_fake
def _(gate_raw, value_raw, E, dE, e0, gate_min, gate_max, compass):
    nb, T, C = gate_raw.shape
    return (gate_raw.new_empty(nb, T, C), gate_raw.new_empty(nb, T, C),
            gate_raw.new_empty(nb, C, dtype=acc_dtype(E.dtype, gate_raw.dtype)))


def _gated_setup(ctx, inputs, output):
    g, v, e0, gmin, gmax, compass, scan_dtype = inputs
    E, _ = output
    ctx.save_for_backward(g, v, E, e0)
    ctx.args = (gmin, gmax, compass)
    ctx.has_e0 = e0 is not None
    ctx.e0_dtype = None if e0 is None else e0.dtype


def _gated_bwd(ctx, dE, de_last):
    g, v, E, e0 = ctx.saved_tensors
    if dE is None:
        dE = torch.zeros_like(E)
    if de_last is not None:
        dE = dE.clone()
        dE[:, -1] += de_last.to(dE.dtype)
    dg, dv, de0 = gated_scan_backward(g, v, E, dE, e0, *ctx.args)
    return (dg, dv, de0.reshape(e0.shape).to(ctx.e0_dtype) if ctx.has_e0 else None,
            None, None, None, None)


torch.library.register_autograd("esa_b200::gated_scan", _gated_bwd, setup_context=_gated_setup)


# --------------------------------------------------------------------------
# ESA-Lightning one-token step (kernel c)
# --------------------------------------------------------------------------
@torch.library.custom_op("esa_b200::lightning_step", mutates_args=())
def lightning_step(qgv: Tensor, state: Tensor, gate_min: float, gate_max: float, eps: float,
                   z_dtype: torch.dtype) -> tuple[Tensor, Tensor]:
    """qgv [B, 3C], state [B, C] -> (new_state [B, C] in state's dtype,
    z = sigmoid(q) * S' * rsqrt(mean(S'^2) + eps) [B, C] in z_dtype)."""
    _require_cuda("esa lightning step", qgv, state)
    nb, c3 = qgv.shape
    C = c3 // 3
    if qgv.stride(1) != 1:
        qgv = qgv.contiguous()
    state = state.reshape(nb, C).contiguous()
    new_state = torch.empty_like(state)
    z = torch.empty(nb, C, dtype=z_dtype, device=qgv.device)
    if nb == 0:
        return new_state, z
    rc = _lib.lib().esa_lightning_step(qgv.data_ptr(), qgv.stride(0) if nb > 1 else c3,
                                       dtype_code(qgv.dtype), state.data_ptr(),
                                       new_state.data_ptr(), dtype_code(state.dtype), z.data_ptr(),
                                       dtype_code(z_dtype), nb, C, float(gate_min),
                                       float(gate_max), float(eps), _stream(qgv))
    _lib.check(rc, "esa_lightning_step")
    return new_state, z


@lightning_step.register_fake
def _(qgv, state, gate_min, gate_max, eps, z_dtype):
    nb, c3 = qgv.shape
    return (state.new_empty(nb, c3 // 3), qgv.new_empty(nb, c3 // 3, dtype=z_dtype))


DECODE_MAX_ROWS = 4


def _ptr_or_none(t):
    return None if t is None else t.data_ptr()


def decode_block_supported(x: Tensor, block) -> bool:
    """The fused decode kernels apply: 1..4 rows of an fp16 or bf16 model
    (every weight, the stream and the state in that dtype), C a multiple of
    256, no gradient and no active dropout."""
    if not x.is_cuda or x.dtype not in (torch.float16, torch.bfloat16) or torch.is_grad_enabled():
        return False
    if x.ndim != 2 or not (1 <= x.shape[0] <= DECODE_MAX_ROWS) or x.shape[1] % 256 != 0:
        return False
    if block.training:
        return False
    return all(p.dtype == x.dtype and p.is_contiguous() and p.data_ptr() % 16 == 0 for p in block.parameters())


def decode_head_supported(x: Tensor, ln_f, head) -> bool:
    """esa_decode_head applies to these rows (see decode_block_supported)."""
    if not x.is_cuda or x.dtype not in (torch.float16, torch.bfloat16) or torch.is_grad_enabled():
        return False
    if x.ndim != 2 or not (1 <= x.shape[0] <= DECODE_MAX_ROWS) or x.shape[1] % 256 != 0:
        return False
    return all(p.dtype == x.dtype and p.is_contiguous() and p.data_ptr() % 16 == 0
               for p in (*ln_f.parameters(), *head.parameters()))


def decode_block(x: Tensor, pending: Optional[Tensor], state: Tensor, block, gate_min: float,
                 gate_max: float, eps: float, qgv_lin, out_lin) -> tuple[Tensor, Tensor, Tensor]:
    """One ESAModel block's decode step in four launches (C ABI
    esa_decode_block): returns (x', pending', new state)."""
    nb, C = x.shape
    x = x.contiguous()
    pending = None if pending is None else pending.contiguous()
    st = state.reshape(nb, C).contiguous()
    x_out = torch.empty_like(x)
    p_out = torch.empty_like(x)
    new_state = torch.empty_like(st)
    code = dtype_code(x.dtype)
    L = _lib.lib()
    nbytes = L.esa_decode_block_scratch_bytes(nb, C, code)
    scratch = torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=x.device)
    ln1, ln2, fc, proj = block.ln1, block.ln2, block.mlp.fc, block.mlp.proj
    rc = L.esa_decode_block(x.data_ptr(), _ptr_or_none(pending), x_out.data_ptr(), p_out.data_ptr(),
                            st.data_ptr(), new_state.data_ptr(), ln1.weight.data_ptr(), _ptr_or_none(ln1.bias),
                            qgv_lin.weight.data_ptr(), _ptr_or_none(qgv_lin.bias), out_lin.weight.data_ptr(),
                            _ptr_or_none(out_lin.bias), ln2.weight.data_ptr(), _ptr_or_none(ln2.bias),
                            fc.weight.data_ptr(), _ptr_or_none(fc.bias), proj.weight.data_ptr(),
                            _ptr_or_none(proj.bias), nb, C, code, float(gate_min), float(gate_max), float(eps),
                            1e-5, scratch.data_ptr(), scratch.numel(), _stream(x))
    _lib.check(rc, "esa_decode_block")
    return x_out, p_out, new_state.reshape(state.shape)


def decode_head(x: Tensor, pending: Optional[Tensor], ln_f, head) -> Tensor:
    """logits = head(ln_f(x + pending)) for the rows of a decode step (C ABI
    esa_decode_head)."""
    nb, C = x.shape
    V = head.weight.shape[0]
    logits = torch.empty(nb, V, dtype=x.dtype, device=x.device)
    rc = _lib.lib().esa_decode_head(x.contiguous().data_ptr(),
                                    _ptr_or_none(None if pending is None else pending.contiguous()),
                                    ln_f.weight.data_ptr(), _ptr_or_none(ln_f.bias), 1e-5,
                                    head.weight.data_ptr(), _ptr_or_none(head.bias), logits.data_ptr(), nb, C, V,
                                    dtype_code(x.dtype), _stream(x))
    _lib.check(rc, "esa_decode_head")
    return logits


def check_device_status(device=None) -> None:
    """Raise if a kernel on `device` reported a bounded wait that ran out."""
    if device is None:
        device = torch.cuda.current_device()
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    st = _lib.device_status(idx, clear=True)
    if st:
        names = []
        if st & _lib.STATUS_LOOKBACK_TIMEOUT:
            names.append("lookback wait ran out")
        if st & _lib.STATUS_COPY_TIMEOUT:
            names.append("bulk copy wait ran out")
        raise RuntimeError(f"ESA kernel on cuda:{idx} reported: {', '.join(names)} "
                           f"(status {st:#x}); results of the affected launch are invalid")


# --------------------------------------------------------------------------
# Layer core: qgv -> y (gated scan + fused readout) and its backward, which
# writes the whole qgv gradient in place (ThunderESA.forward between the qgv
# projection and out_proj, esa/backends/thunder.py:282-311)
# --------------------------------------------------------------------------
def _core_views(qgv: Tensor) -> tuple[Tensor, int, int, int]:
    if qgv.dim() != 3 or qgv.shape[-1] % 3 != 0:
        raise ValueError(f"qgv must be [B,T,3C], got {tuple(qgv.shape)}")
    nb, T, C3 = qgv.shape
    return qgv.contiguous(), nb, T, C3 // 3


@torch.library.custom_op("esa_b200::layer_core", mutates_args=())
def layer_core(qgv: Tensor, gate_min: float, gate_max: float, eps: float, compass: int,
               scan_dtype: torch.dtype, out_dtype: torch.dtype) -> tuple[Tensor, Tensor, Tensor]:
    """(y, E, rstd): E = gated scan of the g, v slices of qgv [B,T,3C] in
    scan_dtype, y = sigmoid(q) * E * rsqrt(mean_C(E^2) + eps) in out_dtype,
    rstd the per-row rsqrt (kept for the backward)."""
    _require_cuda("esa layer core", qgv)
    qgv, nb, T, C = _core_views(qgv)
    L = _lib.lib()
    rdt = dtype_code(qgv.dtype)
    acc = acc_dtype(scan_dtype, qgv.dtype, out_dtype)
    E = torch.empty(nb, T, C, dtype=scan_dtype, device=qgv.device)
    y = torch.empty(nb, T, C, dtype=out_dtype, device=qgv.device)
    rstd = torch.empty(nb * T, dtype=acc, device=qgv.device)
    if nb * T * C == 0:
        return y, E, rstd
    ws = _layer_workspace(nb, T, C, qgv.dtype, scan_dtype, out_dtype, qgv.device)
    _lib.check(L.esa_layer_fwd(qgv.data_ptr(), 3 * C, rdt, E.data_ptr(), dtype_code(scan_dtype), y.data_ptr(),
                               dtype_code(out_dtype), rstd.data_ptr(), nb, T, C, float(gate_min), float(gate_max),
                               float(eps), None, None, ws.data_ptr(), ws.numel(), _stream(qgv)), "esa_layer_fwd")
    return y, E, rstd


def _layer_workspace(nb: int, T: int, C: int, qdt: torch.dtype, edt: torch.dtype, ydt: torch.dtype,
                     device) -> Tensor:
    n = _lib.lib().esa_layer_workspace_bytes(nb, T, C, dtype_code(qdt), dtype_code(edt), dtype_code(ydt))
    if n == 0:
        raise ValueError("invalid layer problem")
    return torch.empty(int(n), dtype=torch.uint8, device=device)


@layer_core.register_fake
def _(qgv, gate_min, gate_max, eps, compass, scan_dtype, out_dtype):
    nb, T, C3 = qgv.shape
    C = C3 // 3
    return (qgv.new_empty(nb, T, C, dtype=out_dtype), qgv.new_empty(nb, T, C, dtype=scan_dtype),
            qgv.new_empty(nb * T, dtype=acc_dtype(scan_dtype, qgv.dtype, out_dtype)))


@torch.library.custom_op("esa_b200::layer_core_backward", mutates_args=())
def layer_core_backward(dy: Tensor, qgv: Tensor, E: Tensor, rstd: Tensor, gate_min: float,
                        gate_max: float, eps: float, compass: int) -> Tensor:
    """d qgv [B,T,3C] (qgv's dtype): dq from the readout backward, d gate and
    d value from the gated reverse scan (one fused kernel where the shape and
    dtypes allow)."""
    _require_cuda("esa layer core backward", dy, qgv, E, rstd)
    qgv, nb, T, C = _core_views(qgv)
    dy = dy.contiguous()
    E = E.contiguous()
    L = _lib.lib()
    rdt = dtype_code(qgv.dtype)
    dqgv = torch.empty_like(qgv)
    if nb * T * C == 0:
        return dqgv.zero_()
    ws = _layer_workspace(nb, T, C, qgv.dtype, E.dtype, dy.dtype, qgv.device)
    _lib.check(L.esa_layer_bwd(dy.data_ptr(), dtype_code(dy.dtype), qgv.data_ptr(), 3 * C, rdt, E.data_ptr(),
                               dtype_code(E.dtype), rstd.data_ptr(), dqgv.data_ptr(), 3 * C, nb, T, C,
                               float(gate_min), float(gate_max), float(eps), None, None, ws.data_ptr(), ws.numel(),
                               _stream(qgv)), "esa_layer_bwd")
    return dqgv


@layer_core_backward.register_fake
def _(dy, qgv, E, rstd, gate_min, gate_max, eps, compass):
    return torch.empty_like(qgv)


def _core_setup(ctx, inputs, output):
    qgv, gmin, gmax, eps, compass, scan_dtype, out_dtype = inputs
    _, E, rstd = output
    ctx.save_for_backward(qgv, E, rstd)
    ctx.args = (gmin, gmax, eps, compass)


def _core_bwd(ctx, dy, dE_unused, drstd_unused):
    qgv, E, rstd = ctx.saved_tensors
    gmin, gmax, eps, compass = ctx.args
    if dy is None:
        return None, None, None, None, None, None, None
    dqgv = layer_core_backward(dy, qgv, E, rstd, gmin, gmax, eps, compass)
    return dqgv, None, None, None, None, None, None


torch.library.register_autograd("esa_b200::layer_core", _core_bwd, setup_context=_core_setup)


def readout(q: Tensor, E: Tensor, eps: float, out_dtype: torch.dtype) -> Tensor:
    """Fused readout sigmoid(q) * E * rsqrt(mean_C(E^2) + eps), [B,T,C] (q may
    be a row-strided slice), no autograd (inference: prefill)."""
    _require_cuda("esa readout", q, E)
    nb, T, C = E.shape
    E = E.contiguous()
    qr, rs_q = _rows(q)
    y = torch.empty(nb, T, C, dtype=out_dtype, device=E.device)
    if nb * T * C == 0:
        return y
    rstd = torch.empty(nb * T, dtype=acc_dtype(q.dtype, E.dtype, out_dtype), device=E.device)
    _lib.check(_lib.lib().esa_readout_fwd(qr.data_ptr(), rs_q, dtype_code(qr.dtype), E.data_ptr(), C,
                                          dtype_code(E.dtype), y.data_ptr(), C, dtype_code(out_dtype),
                                          rstd.data_ptr(), nb * T, C, float(eps), _stream(E)),
               "esa_readout_fwd")
    return y


# --------------------------------------------------------------------------
# LayerNorm of the ESAModel residual stream, written in its consumer's dtype
# (the blocks' F.layer_norm, esa/model.py)
# --------------------------------------------------------------------------
# Below this many rows the fused LayerNorm measured 1-1.5 us slower per call
# than PyTorch's (4.3 vs 3.2 us at one row inside a CUDA graph: decode), above
# it faster (49 vs 90 us at 32768 x 768 fp32).
LAYER_NORM_MIN_ROWS = 4096


def layer_norm_supported(x: Tensor, weight: Tensor, bias: Optional[Tensor]) -> bool:
    C = x.shape[-1]
    ok_dt = (torch.float16, torch.bfloat16, torch.float32)
    return (x.is_cuda and bias is not None and weight.is_cuda and C % 8 == 0 and 0 < C <= 2048
            and x.numel() >= LAYER_NORM_MIN_ROWS * C
            and x.dtype in ok_dt and weight.dtype in ok_dt and bias.dtype == weight.dtype)


@torch.library.custom_op("esa_b200::layer_norm", mutates_args=())
def layer_norm(x: Tensor, weight: Tensor, bias: Tensor, eps: float,
               out_dtype: torch.dtype) -> tuple[Tensor, Tensor, Tensor]:
    """(y, mean, rstd): y = (x - mean) rstd w + b over the last axis in
    out_dtype (fp32 arithmetic); mean, rstd per row (fp32) for the backward."""
    _require_cuda("esa layer norm", x, weight, bias)
    C = x.shape[-1]
    xc = x.contiguous()
    rows = xc.numel() // C if C else 0
    y = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    mean = torch.empty(rows, dtype=torch.float32, device=x.device)
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
    if rows == 0:
        return y, mean, rstd
    _lib.check(_lib.lib().esa_layer_norm_fwd(xc.data_ptr(), dtype_code(xc.dtype), weight.contiguous().data_ptr(),
                                             bias.contiguous().data_ptr(), dtype_code(weight.dtype), y.data_ptr(),
                                             dtype_code(out_dtype), mean.data_ptr(), rstd.data_ptr(), rows, C,
                                             float(eps), _stream(x)), "esa_layer_norm_fwd")
    return y, mean, rstd


@layer_norm.register_fake
def _(x, weight, bias, eps, out_dtype):
    rows = x.numel() // x.shape[-1] if x.shape[-1] else 0
    return (x.new_empty(x.shape, dtype=out_dtype), x.new_empty(rows, dtype=torch.float32),
            x.new_empty(rows, dtype=torch.float32))


@torch.library.custom_op("esa_b200::layer_norm_backward", mutates_args=())
def layer_norm_backward(dy: Tensor, x: Tensor, weight: Tensor, mean: Tensor,
                        rstd: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """(dx, dw, db) of esa_b200::layer_norm (dw, db reduced in a fixed order)."""
    _require_cuda("esa layer norm backward", dy, x, weight, mean, rstd)
    C = x.shape[-1]
    xc = x.contiguous()
    dyc = dy.contiguous()
    rows = xc.numel() // C if C else 0
    dx = torch.empty_like(xc)
    dw = torch.empty_like(weight)
    db = torch.empty_like(weight)
    L = _lib.lib()
    n = int(L.esa_layer_norm_workspace_bytes(rows, C))
    ws = torch.empty(max(n // 4, 1), dtype=torch.float32, device=x.device)
    _lib.check(L.esa_layer_norm_bwd(dyc.data_ptr(), dtype_code(dyc.dtype), xc.data_ptr(), dtype_code(xc.dtype),
                                    weight.contiguous().data_ptr(), dtype_code(weight.dtype), mean.data_ptr(),
                                    rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(), db.data_ptr(), ws.data_ptr(),
                                    ws.numel() * 4, rows, C, _stream(x)), "esa_layer_norm_bwd")
    return dx, dw, db


@layer_norm_backward.register_fake
def _(dy, x, weight, mean, rstd):
    return torch.empty_like(x), torch.empty_like(weight), torch.empty_like(weight)


def _ln_setup(ctx, inputs, output):
    x, weight, bias, eps, out_dtype = inputs
    _, mean, rstd = output
    ctx.save_for_backward(x, weight, mean, rstd)


def _ln_bwd(ctx, dy, dmean_unused, drstd_unused):
    x, weight, mean, rstd = ctx.saved_tensors
    if dy is None:
        return None, None, None, None, None
    dx, dw, db = layer_norm_backward(dy, x, weight, mean, rstd)
    return dx, dw, db, None, None


torch.library.register_autograd("esa_b200::layer_norm", _ln_bwd, setup_context=_ln_setup)


@torch.library.custom_op("esa_b200::add_layer_norm", mutates_args=())
def add_layer_norm(x: Tensor, res: Tensor, weight: Tensor, bias: Tensor, eps: float,
                   out_dtype: torch.dtype) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """(xsum, y, mean, rstd): xsum = x + res in x's dtype (the residual add),
    y = LayerNorm(xsum) in out_dtype -- one pass instead of an add and a norm."""
    _require_cuda("esa add layer norm", x, res, weight, bias)
    if res.shape != x.shape:
        raise ValueError(f"res must have x's shape {tuple(x.shape)}, got {tuple(res.shape)}")
    C = x.shape[-1]
    xc, rc = x.contiguous(), res.contiguous()
    rows = xc.numel() // C if C else 0
    xsum = torch.empty_like(xc)
    y = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    mean = torch.empty(rows, dtype=torch.float32, device=x.device)
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
    if rows == 0:
        return xsum, y, mean, rstd
    _lib.check(_lib.lib().esa_add_layer_norm_fwd(
        xc.data_ptr(), dtype_code(xc.dtype), rc.data_ptr(), dtype_code(rc.dtype), xsum.data_ptr(),
        weight.contiguous().data_ptr(), bias.contiguous().data_ptr(), dtype_code(weight.dtype), y.data_ptr(),
        dtype_code(out_dtype), mean.data_ptr(), rstd.data_ptr(), rows, C, float(eps), _stream(x)),
        "esa_add_layer_norm_fwd")
    return xsum, y, mean, rstd


@add_layer_norm.register_fake
def _(x, res, weight, bias, eps, out_dtype):
    rows = x.numel() // x.shape[-1] if x.shape[-1] else 0
    return (torch.empty_like(x), x.new_empty(x.shape, dtype=out_dtype),
            x.new_empty(rows, dtype=torch.float32), x.new_empty(rows, dtype=torch.float32))


@torch.library.custom_op("esa_b200::add_layer_norm_backward", mutates_args=())
def add_layer_norm_backward(dy: Tensor, dsum: Optional[Tensor], xsum: Tensor, weight: Tensor, mean: Tensor,
                            rstd: Tensor, res_dtype: torch.dtype) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """(dx, dres, dw, db) of esa_b200::add_layer_norm."""
    _require_cuda("esa add layer norm backward", dy, dsum, xsum, weight, mean, rstd)
    C = xsum.shape[-1]
    xc = xsum.contiguous()
    dyc = dy.contiguous()
    dsc = None if dsum is None else dsum.contiguous()
    rows = xc.numel() // C if C else 0
    dx = torch.empty_like(xc)
    dres = torch.empty(xc.shape, dtype=res_dtype, device=xc.device)
    dw = torch.empty_like(weight)
    db = torch.empty_like(weight)
    L = _lib.lib()
    n = int(L.esa_layer_norm_workspace_bytes(rows, C))
    ws = torch.empty(max(n // 4, 1), dtype=torch.float32, device=xc.device)
    _lib.check(L.esa_add_layer_norm_bwd(
        dyc.data_ptr(), dtype_code(dyc.dtype), _ptr(dsc), dtype_code(dsc.dtype) if dsc is not None else 0,
        xc.data_ptr(), dtype_code(xc.dtype), weight.contiguous().data_ptr(), dtype_code(weight.dtype),
        mean.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dres.data_ptr(), dtype_code(res_dtype), dw.data_ptr(),
        db.data_ptr(), ws.data_ptr(), ws.numel() * 4, rows, C, _stream(xc)), "esa_add_layer_norm_bwd")
    return dx, dres, dw, db


@add_layer_norm_backward.register_fake
def _(dy, dsum, xsum, weight, mean, rstd, res_dtype):
    return (torch.empty_like(xsum), xsum.new_empty(xsum.shape, dtype=res_dtype), torch.empty_like(weight),
            torch.empty_like(weight))


def _add_ln_setup(ctx, inputs, output):
    x, res, weight, bias, eps, out_dtype = inputs
    xsum, _, mean, rstd = output
    ctx.save_for_backward(xsum, weight, mean, rstd)
    ctx.res_dtype = res.dtype


def _add_ln_bwd(ctx, dsum, dy, dmean_unused, drstd_unused):
    xsum, weight, mean, rstd = ctx.saved_tensors
    if dy is None:
        if dsum is None:
            return None, None, None, None, None, None
        return dsum, dsum.to(ctx.res_dtype), None, None, None, None
    dx, dres, dw, db = add_layer_norm_backward(dy, dsum, xsum, weight, mean, rstd, ctx.res_dtype)
    return dx, dres, dw, db, None, None


torch.library.register_autograd("esa_b200::add_layer_norm", _add_ln_bwd, setup_context=_add_ln_setup)


# ---------------------------------------------------------------------------
# Cross-entropy of the LM head (the ESAModel training loss)
# ---------------------------------------------------------------------------
def cross_entropy_supported(logits: Tensor, targets: Tensor) -> bool:
    """The fused loss takes 2-D CUDA logits (f16, bf16, f32) and int64 targets."""
    return (logits.is_cuda and logits.dim() == 2 and logits.dtype in (torch.float16, torch.bfloat16, torch.float32)
            and targets.dtype == torch.int64 and targets.dim() == 1 and targets.shape[0] == logits.shape[0]
            and logits.stride(1) == 1)


@torch.library.custom_op("esa_b200::cross_entropy_rows", mutates_args=())
def cross_entropy_rows(logits: Tensor, targets: Tensor, ignore_index: int) -> tuple[Tensor, Tensor]:
    """(loss, lse) per row of logits [rows, V]: lse = logsumexp, loss = lse -
    logits[target] (0 on ignored rows), both fp32; one read of the logits."""
    _require_cuda("esa cross entropy", logits, targets)
    rows, V = logits.shape
    tc = targets.contiguous()
    loss = torch.empty(rows, dtype=torch.float32, device=logits.device)
    lse = torch.empty(rows, dtype=torch.float32, device=logits.device)
    if rows == 0:
        return loss, lse
    _lib.check(_lib.lib().esa_cross_entropy_fwd(logits.data_ptr(), logits.stride(0), dtype_code(logits.dtype),
                                                tc.data_ptr(), int(ignore_index), lse.data_ptr(), loss.data_ptr(),
                                                rows, V, _stream(logits)), "esa_cross_entropy_fwd")
    return loss, lse


@cross_entropy_rows.register_fake
def _(logits, targets, ignore_index):
    rows = logits.shape[0]
    return logits.new_empty(rows, dtype=torch.float32), logits.new_empty(rows, dtype=torch.float32)


@torch.library.custom_op("esa_b200::cross_entropy_rows_backward", mutates_args=())
def cross_entropy_rows_backward(logits: Tensor, targets: Tensor, lse: Tensor, grad_rows: Tensor,
                                ignore_index: int) -> Tensor:
    """d logits (logits' dtype) = grad_rows[i] (softmax(logits[i]) - onehot(target[i])), 0 on ignored rows."""
    _require_cuda("esa cross entropy backward", logits, targets, lse, grad_rows)
    rows, V = logits.shape
    dz = torch.empty((rows, V), dtype=logits.dtype, device=logits.device)
    if rows == 0:
        return dz
    g = grad_rows.to(torch.float32).contiguous()
    _lib.check(_lib.lib().esa_cross_entropy_bwd(logits.data_ptr(), logits.stride(0), dtype_code(logits.dtype),
                                                targets.contiguous().data_ptr(), int(ignore_index), lse.data_ptr(),
                                                g.data_ptr(), dz.data_ptr(), V, rows, V, _stream(logits)),
               "esa_cross_entropy_bwd")
    return dz


@cross_entropy_rows_backward.register_fake
def _(logits, targets, lse, grad_rows, ignore_index):
    return torch.empty_like(logits)


def _xent_setup(ctx, inputs, output):
    logits, targets, ignore_index = inputs
    _, lse = output
    ctx.ignore_index = ignore_index
    ctx.save_for_backward(logits, targets, lse)


def _xent_bwd(ctx, dloss, dlse_unused):
    logits, targets, lse = ctx.saved_tensors
    if dloss is None:
        return None, None, None
    return cross_entropy_rows_backward(logits, targets, lse, dloss, ctx.ignore_index), None, None


torch.library.register_autograd("esa_b200::cross_entropy_rows", _xent_bwd, setup_context=_xent_setup)


def cross_entropy(logits: Tensor, targets: Tensor, ignore_index: int = -100) -> Tensor:
    """Mean cross-entropy over the rows whose target is not ignore_index, as
    `F.cross_entropy(logits, targets, ignore_index=...)` computes it (fp32
    arithmetic whatever the logits' dtype; NaN when every row is ignored)."""
    loss_rows, _ = cross_entropy_rows(logits, targets, ignore_index)
    count = (targets != ignore_index).sum()
    return loss_rows.sum() / count
