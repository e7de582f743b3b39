"""The bounded waits: a wait that runs out reports and returns.

Every spin-wait in the kernels gives up after a one-second budget, raises a
bit in the device status word and lets the kernel return.  esa_wait_selftest
runs the strip kernels' own mbarrier wait on a barrier that nothing arrives
on; the test checks that the wait gave up after about the budget, that the
status bit is set (and cleared on request), and that the context is still
usable for a scan afterwards.  No fault, trap or hang is involved.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_runs_out_reports_and_returns():
    from esa import _lib, ops
    L = _lib.lib()
    torch.cuda.synchronize()
    ops.check_device_status()  # starts clean
    done = ctypes.c_uint(7)
    waited = ctypes.c_uint(0)
    rc = L.esa_wait_selftest(ctypes.byref(done), ctypes.byref(waited),
                             torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    assert done.value == 0                    # the barrier never completed
    assert 900 <= waited.value <= 10000       # gave up after the ~1 s budget
    st = _lib.device_status(torch.cuda.current_device(), clear=True)
    assert st & _lib.STATUS_COPY_TIMEOUT
    assert _lib.device_status(torch.cuda.current_device(), clear=False) == 0
    # the context still works: a scan runs and is right
    A = torch.full((2, 64, 2, 32), 0.5, device="cuda")
    B = torch.ones_like(A)
    E, _ = ops.scan(A, B, None, 16)
    expect = 2 * (1 - 0.5 ** torch.arange(1, 65, device="cuda", dtype=torch.float32))
    torch.testing.assert_close(E[0, :, 0, 0], expect)
    ops.check_device_status()
