"""Sequence-parallel scan: the carry exchange and composition.

CPU part (gloo, world size 2 and 3): every rank summarises its time slice
with the fp64 oracle, the summaries are all-gathered over gloo, and each rank
composes its incoming state with esa.parallel.compose_carries; the states
must equal the oracle's full-sequence state at the slice boundaries.
GPU part: the same slices on one GPU through esa_scan_summary + the seeded
scan, and (with two or more GPUs) the real NCCL path.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _slices(world, T=120, shape=(2, 3, 8), seed=0):
    rng = np.random.default_rng(seed)
    nb, H, D = shape
    A = 1 / (1 + np.exp(-(rng.normal(size=(nb, T, H, D)) + 3)))
    B = rng.normal(scale=0.5, size=(nb, T, H, D))
    cuts = np.linspace(0, T, world + 1).astype(int)
    return A, B, cuts


def _gloo_worker(rank, world, port, result_q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "entangled-state-attention_v2_b200"))
    sys.path.insert(0, str(root))
    from esa.parallel import compose_carries
    from oracle import oracle as orc
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        A, B, cuts = _slices(world)
        a, b = A[:, cuts[rank]:cuts[rank + 1]], B[:, cuts[rank]:cuts[rank + 1]]
        nb, _, H, D = a.shape
        E = orc.scan_fwd(a, b)
        e_end = torch.from_numpy(E[:, -1].reshape(nb, H * D))
        prod = torch.from_numpy(np.prod(a, axis=1).reshape(nb, H * D))
        mine = torch.stack([e_end, prod])
        gathered = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(gathered, mine)
        carry = compose_carries(gathered, rank)
        result_q.put((rank, carry.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_carry_exchange_over_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    A, B, cuts = _slices(world)
    full = oracle.scan_fwd(A, B)
    nb, T, H, D = A.shape
    for r in range(world):
        expect = np.zeros((nb, H * D)) if r == 0 else full[:, cuts[r] - 1].reshape(nb, H * D)
        np.testing.assert_allclose(got[r], expect, rtol=1e-12, atol=1e-12)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-3)])
def test_summary_and_sliced_scan_on_one_gpu(dtype, tol):
    from esa import ops
    from esa.parallel import compose_carries
    torch.manual_seed(0)
    nb, T, H, D = 4, 4096, 32, 64
    A = torch.sigmoid(torch.randn(nb, T, H, D, device="cuda") + 3).to(dtype)
    B = (torch.randn(nb, T, H, D, device="cuda") * 0.5).to(dtype)
    world = 4
    cuts = [i * T // world for i in range(world + 1)]
    summaries = []
    for r in range(world):
        e_end, prod = ops.scan_summary(A[:, cuts[r]:cuts[r + 1]], B[:, cuts[r]:cuts[r + 1]], None)
        summaries.append(torch.stack([e_end, prod]))
    # summary of a slice against the oracle
    a0 = A[:, :cuts[1]].double().cpu()
    b0 = B[:, :cuts[1]].double().cpu()
    ref0 = oracle.scan_fwd(a0, b0)
    e_ref = ref0[:, -1].reshape(nb, H * D)
    p_ref = np.prod(a0.numpy(), axis=1).reshape(nb, H * D)
    np.testing.assert_allclose(summaries[0][0].double().cpu().numpy(), e_ref, rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(summaries[0][1].double().cpu().numpy(), p_ref, rtol=1e-4, atol=1e-30)
    parts = []
    for r in range(world):
        carry = compose_carries(summaries, r)
        E, _ = ops.scan(A[:, cuts[r]:cuts[r + 1]], B[:, cuts[r]:cuts[r + 1]], carry, 16)
        parts.append(E)
    got = torch.cat(parts, dim=1).double().cpu().numpy()
    ref = oracle.scan_fwd(A.double().cpu(), B.double().cpu())
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert err < tol, err


def _nccl_worker(rank, world, port, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "entangled-state-attention_v2_b200"))
    import datetime
    from esa.parallel import sequence_parallel_scan
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        g = torch.Generator().manual_seed(1)
        nb, T, H, D = 2, 2048, 8, 64
        A = torch.sigmoid(torch.randn(nb, T, H, D, generator=g) + 3)
        B = torch.randn(nb, T, H, D, generator=g) * 0.5
        cuts = [i * T // world for i in range(world + 1)]
        sl = slice(cuts[rank], cuts[rank + 1])
        E = sequence_parallel_scan(A[:, sl].cuda(), B[:, sl].cuda())
        E2 = sequence_parallel_scan(A[:, sl].cuda(), B[:, sl].cuda(), form="two_pass")
        torch.cuda.synchronize()
        q.put((rank, (E.cpu().numpy(), E2.cpu().numpy())))
    finally:
        dist.destroy_process_group()


def _one_gpu_worker(rank, world, port, backend, form, q):
    """Rank of a sequence-parallel scan whose ranks all share GPU 0 (the
    kernels of different ranks never wait on one another: the only exchange is
    the all-gather between the summary and the scan)."""
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root / "entangled-state-attention_v2_b200"))
    import datetime
    from esa import ops
    from esa.parallel import sequence_parallel_scan
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(0)
    kw = {"device_id": torch.device("cuda", 0)} if backend == "nccl" else {}
    dist.init_process_group(backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), **kw)
    try:
        A, B, e0 = _sp_inputs()
        T = A.shape[1]
        cuts = [i * T // world for i in range(world + 1)]
        sl = slice(cuts[rank], cuts[rank + 1])
        E = sequence_parallel_scan(A[:, sl].cuda(), B[:, sl].cuda(), e0=e0.cuda(), form=form)
        torch.cuda.synchronize()
        ops.check_device_status()
        q.put((rank, E.cpu().numpy()))
    finally:
        dist.destroy_process_group()


def _sp_inputs():
    g = torch.Generator().manual_seed(3)
    nb, T, H, D = 2, 24576, 4, 64
    A = torch.sigmoid(torch.randn(nb, T, H, D, generator=g) + 3)
    B = torch.randn(nb, T, H, D, generator=g) * 0.5
    e0 = torch.randn(nb, H * D, generator=g)
    return A, B, e0


@pytest.mark.gpu
@pytest.mark.parametrize("form", ["single_pass", "two_pass"])
@pytest.mark.parametrize("backend,world", [("nccl", 1), ("gloo", 2), ("gloo", 3)])
def test_sequence_parallel_scan_on_one_gpu(backend, world, form):
    """esa.parallel.sequence_parallel_scan end to end with every rank on
    GPU 0: NCCL at world size 1, gloo at 2 and 3 (slices of 8192 steps or
    more).  single_pass: scan from zero + product, all-gather, carry
    composition, fix-up of the slice head; two_pass: split summary,
    all-gather, resumed scan.  The joined slices against the fp64 oracle of
    the whole sequence from the same initial state."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_one_gpu_worker, args=(r, world, port, backend, form, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    A, B, e0 = _sp_inputs()
    nb, T, H, D = A.shape
    ref = oracle.scan_fwd(A.double(), B.double(), e0.double().reshape(nb, H, D))
    full = np.concatenate([got[r] for r in range(world)], axis=1)
    assert np.linalg.norm(full - ref) / np.linalg.norm(ref) < 1e-5


@pytest.mark.gpu
def test_sequence_parallel_scan_nccl():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    g = torch.Generator().manual_seed(1)
    nb, T, H, D = 2, 2048, 8, 64
    A = torch.sigmoid(torch.randn(nb, T, H, D, generator=g) + 3)
    B = torch.randn(nb, T, H, D, generator=g) * 0.5
    ref = oracle.scan_fwd(A.double(), B.double())
    for form in range(2):
        full = np.concatenate([got[r][form] for r in range(world)], axis=1)
        assert np.linalg.norm(full - ref) / np.linalg.norm(ref) < 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(4, 16384, 32, 64), (2, 300, 4, 64)])
def test_summary_then_resume_equals_full_scan(shape):
    """esa_scan_fwd_resume after esa_scan_summary on the same workspace agrees
    with esa_scan_fwd (split slices reuse the piece summaries; short slices
    are scanned in full)."""
    from esa import _lib, ops
    torch.manual_seed(2)
    A = torch.sigmoid(torch.randn(shape, device="cuda") + 3).to(torch.bfloat16)
    B = (torch.randn(shape, device="cuda") * 0.5).to(torch.bfloat16)
    nb, T, H, D = shape
    hd = H * D
    e0 = torch.randn(nb, hd, device="cuda")
    ref, ref_last = ops.scan(A, B, e0, 16)
    L = _lib.lib()
    code = ops.dtype_code(A.dtype)
    ws = ops._workspace(nb, T, hd, A.dtype, 16, A.device)
    s = torch.cuda.current_stream().cuda_stream
    e_end = torch.empty(nb, hd, device="cuda")
    prod = torch.empty(nb, hd, device="cuda")
    _lib.check(L.esa_scan_summary(A.data_ptr(), B.data_ptr(), nb, T, hd, code, None, e_end.data_ptr(),
                                  prod.data_ptr(), ws.data_ptr(), ws.numel(), s), "summary")
    E = torch.empty_like(A)
    e_last = torch.empty(nb, hd, device="cuda")
    _lib.check(L.esa_scan_fwd_resume(A.data_ptr(), B.data_ptr(), E.data_ptr(), nb, T, hd, code, 16,
                                     e0.data_ptr(), e_last.data_ptr(), ws.data_ptr(), ws.numel(), s),
               "resume")
    torch.cuda.synchronize()
    # esa_scan_fwd takes a time-parallel kernel (the single-pass chained scan
    # from 8192 steps, the look-back scan below) whose association order
    # differs from the split passes': equal to rounding
    torch.testing.assert_close(E.float(), ref.float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(e_last, ref_last, rtol=1e-5, atol=1e-5)
    # the slice summary composes with e0 into the end state
    torch.testing.assert_close(prod * e0 + e_end, e_last, rtol=1e-4, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,tol", [(torch.float16, 2e-3), (torch.bfloat16, 2e-3), (torch.float32, 1e-5),
                                       (torch.float64, 1e-12)])
@pytest.mark.parametrize("shape,gates", [((2, 5000, 4, 64), "sigmoid"), ((3, 700, 1, 77), "sigmoid"),
                                         ((2, 3000, 2, 64), "ones"), ((1, 1, 2, 1024), "sigmoid")])
def test_slice_prod_and_fixup_against_oracle(dtype, tol, shape, gates):
    """esa_scan_prod (product of A over the slice, stopping where it is zero)
    and esa_scan_fixup (the head of a slice scanned from zero, rescanned from
    its incoming state) against the fp64 oracle: the result equals the scan
    from e0 = carry.  Covers
    16-bit channel pairs (even hd) and single channels (hd = 77), gates of one
    everywhere (the product never reaches zero: both kernels walk the whole
    slice) and a one-step slice (2048 channels: the 16-bit bar is a relative
    Frobenius norm, meaningful over many elements)."""
    from esa import _lib, ops
    g = torch.Generator().manual_seed(21)
    nb, T, H, D = shape
    hd = H * D
    if gates == "ones":
        A = torch.ones(shape, dtype=torch.float64)
    else:
        A = torch.sigmoid(torch.randn(shape, generator=g, dtype=torch.float64) + 3)
    A = A.to(dtype)
    B = (torch.randn(shape, generator=g, dtype=torch.float64) * 0.5).to(dtype)
    carry = torch.randn(nb, hd, generator=g, dtype=torch.float64)
    acc = ops.acc_dtype(dtype)
    Ad, Bd = A.cuda(), B.cuda()
    E0, _ = ops.scan(Ad, Bd, None, 16)
    L = _lib.lib()
    s = torch.cuda.current_stream().cuda_stream
    code = ops.dtype_code(dtype)
    prod = torch.empty(nb, hd, dtype=acc, device="cuda")
    _lib.check(L.esa_scan_prod(Ad.data_ptr(), prod.data_ptr(), nb, T, hd, code, s), "esa_scan_prod")
    cd = carry.to(acc).cuda()
    E = E0.clone()
    _lib.check(L.esa_scan_fixup(Ad.data_ptr(), Bd.data_ptr(), E.data_ptr(), cd.data_ptr(), nb, T, hd, code, s),
               "esa_scan_fixup")
    torch.cuda.synchronize()
    p_ref = np.prod(A.double().numpy(), axis=1).reshape(nb, hd)
    np.testing.assert_allclose(prod.double().cpu().numpy(), p_ref, rtol=max(tol, 1e-3) if acc == torch.float32
                               else 1e-10, atol=1e-30)
    ref = oracle.scan_fwd(A.double(), B.double(), cd.double().cpu().reshape(nb, H, D))
    got = E.double().cpu().numpy()
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert err < tol, err
