"""The fused cross-entropy of the LM head (esa_cross_entropy_fwd/bwd) against
torch's F.cross_entropy on the same logits upcast to fp32 -- the computation
PyTorch runs for the reference's `F.cross_entropy(logits, targets,
ignore_index=-1)` under autocast.

Bar: the mean loss to 2e-5 relative (fp32 arithmetic on both sides); the
logits gradient to relative Frobenius error 1e-5 for fp32 logits, 2e-3 for
fp16 and 4e-3 for bf16 logits: the gradient is rounded once to the logits'
dtype, whose RMS relative rounding error is about 2^-12/sqrt(3) = 1.4e-4 for
fp16 and 2^-9/sqrt(3) = 2.3e-3 for bf16.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

GTOL = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 4e-3}


def rel(got, ref) -> float:
    g = got.detach().double().cpu().numpy()
    r = ref.detach().double().cpu().numpy()
    assert g.shape == r.shape and np.isfinite(g).all()
    return float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-300))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,V,pad", [(37, 1000, 0),      # vector path, ragged last vectors per thread
                                        (64, 32000, 0),     # the ESAModel vocabulary
                                        (29, 1003, 0),      # V not a multiple of 8: element path
                                        (16, 2048, 8)])     # row stride V + 8 (a view of a wider buffer)
def test_cross_entropy_matches_torch(dtype, rows, V, pad):
    from esa import _lib, ops
    g = torch.Generator().manual_seed(11)
    buf = (torch.randn(rows, V + pad, generator=g) * 3).to(dtype).cuda()
    logits = buf[:, :V].requires_grad_(False)
    targets = torch.randint(0, V, (rows,), generator=g)
    targets[::5] = -1  # ignored rows
    targets = targets.cuda()
    z = logits.detach().clone().requires_grad_(True) if pad == 0 else logits.detach().requires_grad_(True)
    loss = ops.cross_entropy(z, targets, ignore_index=-1)
    zr = logits.detach().float().requires_grad_(True)
    ref = F.cross_entropy(zr, targets, ignore_index=-1)
    assert loss.dtype == torch.float32
    assert abs(loss.item() - ref.item()) <= 2e-5 * abs(ref.item())
    loss.backward()
    ref.backward()
    assert z.grad.dtype == dtype
    assert rel(z.grad, zr.grad) < GTOL[dtype]
    # ignored rows get no gradient
    assert torch.count_nonzero(z.grad[::5]) == 0
    assert _lib.last_error() == ""


def test_cross_entropy_all_ignored_is_nan_like_torch():
    from esa import ops
    z = torch.randn(4, 64, device="cuda")
    t = torch.full((4,), -1, dtype=torch.int64, device="cuda")
    assert torch.isnan(ops.cross_entropy(z, t, ignore_index=-1))
    assert torch.isnan(F.cross_entropy(z, t, ignore_index=-1))


def test_cross_entropy_out_of_range_target_poisons_its_row():
    """A target outside [0, V) that is not ignore_index: NaN loss, and NaN
    gradients on that row only (the other rows keep theirs)."""
    from esa import ops
    z = torch.randn(6, 64, device="cuda", requires_grad=True)
    t = torch.tensor([3, 70, 5, -1, 0, 63], dtype=torch.int64, device="cuda")
    loss = ops.cross_entropy(z, t, ignore_index=-1)
    assert torch.isnan(loss)
    loss.backward()
    assert torch.isnan(z.grad[1]).all()
    assert torch.isfinite(z.grad[[0, 2, 3, 4, 5]]).all()


def test_model_loss_with_fused_cross_entropy():
    """ESAModel (fp32) loss and gradients with the fused loss against the same
    model on F.cross_entropy."""
    from esa import ESAModel, ESAModelConfig, ops
    torch.manual_seed(7)
    cfg = ESAModelConfig(vocab_size=250, block=64, n_layer=2, head=4, embd=64, dropout=0.0,
                         precision="fp32", backend="thunder")
    model = ESAModel(cfg, device="cuda")
    ids = torch.randint(0, 250, (3, 65), device="cuda")
    tg = ids[:, 1:].clone()
    tg[0, :7] = -1
    _, loss = model(ids[:, :-1], tg)
    loss.backward()
    grads = {n: p.grad.clone() for n, p in model.named_parameters() if p.grad is not None}
    model.zero_grad(set_to_none=True)
    orig = ops.cross_entropy_supported
    ops.cross_entropy_supported = lambda *a: False
    try:
        _, loss2 = model(ids[:, :-1], tg)
        loss2.backward()
    finally:
        ops.cross_entropy_supported = orig
    assert abs(loss.item() - loss2.item()) <= 1e-5 * abs(loss2.item())
    for n, p in model.named_parameters():
        if p.grad is not None:
            assert rel(grads[n], p.grad) < 1e-4, n
