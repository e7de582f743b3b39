"""Sequence-parallel scan: one long sequence split along time across GPUs.

Each rank of a process group holds one contiguous time slice of A and B
(``[B, T_r, H, D]``, rank order = time order).  The recurrence couples the
slices only through one state per channel, so the exchange is tiny.  Two
forms, with the same exchange in the middle:

single pass (default):
  1. scan (local, from a zero state): E^0 of the slice and its fp32 end
     state E_end_r -- ``esa_scan_fwd`` with ``e_last``; P_r = prod_t A_t over
     the slice -- ``esa_scan_prod``, which stops where the product is zero;
  2. exchange: all-gather of the [2, B, H*D] fp32 summaries (NCCL; 64 KB per
     rank for B=4, H*D=2048; a gloo group exchanges them through host memory);
  3. carry: C_0 = e0 (or 0), C_{r+1} = P_r * C_r + E_end_r, composed in rank
     order on every rank (the same arithmetic everywhere: deterministic);
  4. fix-up (local): the head of the slice rescanned from C_r --
     ``esa_scan_fixup``, only while A_0 ... A_t is not yet zero (beyond, the
     outputs from the zero state equal those from C_r).
  Every rank reads A and B once and writes E once, plus the short heads of
  steps 1 and 4 (gates below one: a few thousand steps; A = 1 everywhere
  would make them read the whole slice).

two pass (``form="two_pass"``): 1. ``esa_scan_summary`` (reads A and B once);
  2.-3. as above; 4. ``esa_scan_fwd_resume`` from the exact incoming state
  (reads A and B again, writes E): 5 bytes-per-element passes whatever the
  data, and E bit-equal to a one-GPU scan's arithmetic from that state.

No wait spans more than the one all-gather.  Forward only: the reference has
no multi-device path at all, and its training (esa/model.py) runs one
sequence per GPU.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from . import _lib, ops


def compose_carries(summaries: list[torch.Tensor], rank: int,
                    e0: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Incoming state of `rank` from every rank's [2, ...] (E_end, prod)
    summary (rank order = time order)."""
    e_end0 = summaries[0][0]
    carry = torch.zeros_like(e_end0) if e0 is None else e0.to(e_end0.dtype).reshape(e_end0.shape)
    for r in range(rank):
        e_end, prod = summaries[r][0], summaries[r][1]
        carry = torch.addcmul(e_end, prod, carry)
    return carry


def sequence_parallel_scan(A: torch.Tensor, B: torch.Tensor, *, group=None, compass: int = 16,
                           e0: Optional[torch.Tensor] = None, form: str = "single_pass") -> torch.Tensor:
    """E for this rank's time slice of a sequence split across `group`.

    A, B: this rank's slice [B, T_r, H, D] (CUDA).  e0: the state before the
    first slice ([B, H, D] or [B, H*D]), used by every rank (only rank 0's
    carry starts from it).  form: "single_pass" (scan from zero, exchange,
    fix up the head of the slice) or "two_pass" (summary, exchange, scan from
    the exact incoming state).  Returns the slice of E in A's dtype.
    """
    if A.shape != B.shape or A.dim() != 4:
        raise ValueError(f"A and B must be the same [B,T,H,D], got {tuple(A.shape)} and {tuple(B.shape)}")
    if form not in ("single_pass", "two_pass"):
        raise ValueError(f"form must be 'single_pass' or 'two_pass', got {form!r}")
    if not A.is_cuda or not B.is_cuda:
        raise RuntimeError("sequence_parallel_scan needs CUDA tensors (no CPU fallback)")
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    A = A.contiguous()
    B = B.to(A.dtype).contiguous()
    nb, T, H, D = A.shape
    hd = H * D
    acc = ops.acc_dtype(A.dtype)
    code = ops.dtype_code(A.dtype)
    L = _lib.lib()
    stream = torch.cuda.current_stream(A.device).cuda_stream
    ws = ops._workspace(nb, T, hd, A.dtype, int(compass), A.device)
    work = T > 0 and hd > 0 and nb > 0
    E = torch.empty_like(A)
    # [E_end, prod] written in place by the kernels (every channel of both),
    # so the gather reads it without a stack copy
    mine = torch.empty(2, nb, hd, dtype=acc, device=A.device)
    if not work:
        mine[0].zero_()
        mine[1].fill_(1)
    elif form == "single_pass":
        _lib.check(L.esa_scan_fwd(A.data_ptr(), B.data_ptr(), E.data_ptr(), nb, T, hd, code, int(compass), None,
                                  mine[0].data_ptr(), ws.data_ptr(), ws.numel(), stream), "esa_scan_fwd")
        _lib.check(L.esa_scan_prod(A.data_ptr(), mine[1].data_ptr(), nb, T, hd, code, stream), "esa_scan_prod")
    else:
        _lib.check(L.esa_scan_summary(A.data_ptr(), B.data_ptr(), nb, T, hd, code, None,
                                      mine[0].data_ptr(), mine[1].data_ptr(), ws.data_ptr(), ws.numel(),
                                      stream), "esa_scan_summary")
    if dist.get_backend(group) == "gloo":
        # gloo gathers host tensors: the 2*B*H*D summaries cross to the host
        # and back (ranks that share one GPU, or no NVLink)
        host = mine.cpu()
        gathered = [torch.empty_like(host) for _ in range(world)]
        dist.all_gather(gathered, host, group=group)
        gathered = [t.to(A.device) for t in gathered]
    else:
        # one flat buffer: a single all_gather_into_tensor instead of a list
        flat = torch.empty(world * 2, nb, hd, dtype=acc, device=A.device)
        dist.all_gather_into_tensor(flat, mine, group=group)
        gathered = list(flat.view(world, 2, nb, hd).unbind(0))
    carry = compose_carries(gathered, rank, e0).contiguous()
    if not work:
        return E
    if form == "single_pass":
        if rank > 0 or e0 is not None:
            _lib.check(L.esa_scan_fixup(A.data_ptr(), B.data_ptr(), E.data_ptr(), carry.data_ptr(), nb, T, hd,
                                        code, stream), "esa_scan_fixup")
    else:
        _lib.check(L.esa_scan_fwd_resume(A.data_ptr(), B.data_ptr(), E.data_ptr(), nb, T, hd, code,
                                         int(compass), carry.data_ptr(), None, ws.data_ptr(),
                                         ws.numel(), stream), "esa_scan_fwd_resume")
    return E
