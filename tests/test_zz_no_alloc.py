"""esa_scan_fwd_noalloc, the forward scan that allocates nothing.

Some callers of the C ABI have no device allocator to hand: a plain C host
program or a foreign-language binding that is given its input and output
buffers, or code whose device memory plan is fixed before it starts.  For them
the library offers esa_scan_fwd_noalloc, which runs the time-parallel scan
kernel with its scratch taken from a fixed array inside the library instead of
a caller workspace.  These tests call it through the C ABI (ctypes) and check
its output against the regular entry point, esa_scan_fwd, on two calls in a
row -- the second call must not be disturbed by what the first one left in the
shared scratch.  This file is named so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 2e-3, torch.float64: 1e-12}


def _rel(got: torch.Tensor, ref: torch.Tensor) -> float:
    g = got.double().cpu().numpy()
    r = ref.double().cpu().numpy()
    assert np.isfinite(g).all()
    return float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-300))


def _inputs(shape, dtype, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.sigmoid(torch.randn(shape, device="cuda", generator=g) * 2 + 2).to(dtype)
    B = torch.randn(shape, device="cuda", generator=g).to(dtype)
    return A, B


def _noalloc(L, A, B, compass=16, e_last=None, e0=None):
    from esa import _lib, ops
    nb, T, H, D = A.shape
    E = torch.empty_like(A)
    rc = L.esa_scan_fwd_noalloc(A.data_ptr(), B.data_ptr(), E.data_ptr(), nb, T, H * D,
                                ops.dtype_code(A.dtype), compass, None if e0 is None else e0.data_ptr(),
                                None if e_last is None else e_last.data_ptr(),
                                torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    return E


def _with_workspace(L, A, B, compass=16, e0=None):
    from esa import _lib, ops
    nb, T, H, D = A.shape
    E = torch.empty_like(A)
    code = ops.dtype_code(A.dtype)
    n = L.esa_scan_workspace_bytes(nb, T, H * D, code, compass)
    ws = torch.empty(max(n, 256), dtype=torch.uint8, device="cuda")
    rc = L.esa_scan_fwd(A.data_ptr(), B.data_ptr(), E.data_ptr(), nb, T, H * D, code, compass,
                        None if e0 is None else e0.data_ptr(), None, ws.data_ptr(), ws.numel(),
                        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    return E


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_noalloc_matches_workspace_entry_point_two_calls(dtype):
    from esa import _lib
    L = _lib.lib()
    # two calls in a row with different shapes and data on the shared scratch
    for shape, seed, compass in (((4, 777, 2, 64), 1, 16), ((2, 1500, 4, 32), 2, 32)):
        A, B = _inputs(shape, dtype, seed)
        e_last = torch.empty(shape[0], shape[2] * shape[3], dtype=torch.float32, device="cuda")
        got = _noalloc(L, A, B, compass, e_last)
        ref = _with_workspace(L, A, B, compass)
        torch.cuda.synchronize()
        assert _rel(got, ref) < TOL[dtype], (shape, _rel(got, ref))
        assert _rel(e_last, ref[:, -1].reshape(shape[0], -1)) < TOL[dtype]
    assert _lib.device_status(torch.cuda.current_device()) == 0


def test_noalloc_with_initial_state_and_unaligned_rows():
    """Prefill with a state (a non-null fp32 e0) and rows whose byte length is
    not a multiple of 16 (fp16 with hd = 6, which takes the one-thread-per-
    channel kernel): the same results as esa_scan_fwd, again two calls in a
    row."""
    from esa import _lib
    L = _lib.lib()
    cases = (((3, 500, 2, 64), torch.float32, True), ((2, 300, 2, 3), torch.float16, False))
    for shape, dtype, with_e0 in cases:
        A, B = _inputs(shape, dtype, 7)
        nb, _, H, D = shape
        e0 = torch.randn(nb, H * D, device="cuda") if with_e0 else None
        got = _noalloc(L, A, B, 16, None, e0)
        ref = _with_workspace(L, A, B, 16, e0)
        torch.cuda.synchronize()
        assert _rel(got, ref) < TOL[dtype], (shape, _rel(got, ref))
    assert _lib.device_status(torch.cuda.current_device()) == 0


def test_noalloc_rejects_problems_beyond_its_scratch():
    from esa import _lib
    L = _lib.lib()
    # [64, 65536, 1024] fp32 would need far more than the fixed scratch
    rc = L.esa_scan_fwd_noalloc(ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16),
                                64, 65536, 1024, _lib.DTYPE_F32, 16, None, None, None)
    assert rc == -3
    msg = _lib.last_error()
    assert "scratch" in msg and str(16 << 20) in msg
