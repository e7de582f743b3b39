"""The fused LayerNorm of the ESAModel residual stream against torch fp64.

y = (x - mean) / sqrt(var + eps) * w + b (biased variance), computed in fp32
and written in the consumer's dtype; backward dx, dw, db.  Bar: relative
Frobenius error against the fp64 math on the same inputs -- 2e-6 for fp32
outputs, 2e-3 for fp16/bf16 outputs; dw/db reduced deterministically (two
runs give the same bits).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def rel(got, ref) -> float:
    g = got.detach().double().cpu().numpy()
    r = ref.detach().double().cpu().numpy()
    assert g.shape == r.shape
    assert np.isfinite(g).all()
    return float(np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-300))


@pytest.mark.parametrize("xdt,wdt,ydt,C", [
    (torch.float32, torch.float32, torch.float16, 768),   # autocast fp16 residual stream
    (torch.float32, torch.float32, torch.float32, 1024),  # fp32 model
    (torch.float32, torch.float32, torch.bfloat16, 256),
    (torch.float16, torch.float16, torch.float16, 2048),  # half model
    (torch.bfloat16, torch.float32, torch.bfloat16, 64),
])
def test_layer_norm_fwd_bwd(xdt, wdt, ydt, C):
    from esa import ops
    g = torch.Generator().manual_seed(31)
    shape = (3, 77, C)
    x64 = torch.randn(shape, generator=g, dtype=torch.float64) * 2 + 0.5
    w64 = 1 + 0.1 * torch.randn(C, generator=g, dtype=torch.float64)
    b64 = 0.1 * torch.randn(C, generator=g, dtype=torch.float64)
    x = x64.to(xdt).cuda().requires_grad_(True)
    w = w64.to(wdt).cuda().requires_grad_(True)
    b = b64.to(wdt).cuda().requires_grad_(True)
    y, mean, rstd = ops.layer_norm(x, w, b, 1e-5, ydt)
    assert y.dtype == ydt
    xr = x.detach().double().requires_grad_(True)
    wr = w.detach().double().requires_grad_(True)
    br = b.detach().double().requires_grad_(True)
    yr = torch.nn.functional.layer_norm(xr, (C,), wr, br, 1e-5)
    tol = 2e-6 if ydt == torch.float32 else 2e-3
    assert rel(y, yr) < tol
    dy = torch.randn(shape, generator=g, dtype=torch.float64)
    y.backward(dy.to(ydt).cuda())
    yr.backward(dy.to(ydt).double().cuda())
    gtol = 2e-5 if xdt == torch.float32 else 4e-3
    assert rel(x.grad, xr.grad) < gtol
    assert rel(w.grad, wr.grad) < gtol
    assert rel(b.grad, br.grad) < gtol
    # the column reductions are deterministic
    dw1, db1 = w.grad.clone(), b.grad.clone()
    w.grad = b.grad = None
    x.grad = None
    y2, _, _ = ops.layer_norm(x, w, b, 1e-5, ydt)
    y2.backward(dy.to(ydt).cuda())
    assert torch.equal(w.grad, dw1) and torch.equal(b.grad, db1)


def test_fused_layer_norm_row_threshold():
    from esa import ops
    w = torch.ones(768, device="cuda")
    b = torch.zeros(768, device="cuda")
    assert ops.layer_norm_supported(torch.empty(2, 2048, 768, device="cuda"), w, b)
    assert not ops.layer_norm_supported(torch.empty(1, 768, device="cuda"), w, b)   # decode: torch
    assert not ops.layer_norm_supported(torch.empty(2, 2048, 100, device="cuda"), w[:100], b[:100])


def test_model_layer_norm_matches_torch_in_a_training_step():
    """ESAModel loss and gradients with the fused LayerNorm and fused residual
    add + LayerNorm (forced on at this small size) against the same model on
    torch's add and F.layer_norm (fp32, no autocast)."""
    from esa import ESAModel, ESAModelConfig, ops
    torch.manual_seed(5)
    cfg = ESAModelConfig(vocab_size=128, block=64, n_layer=2, head=4, embd=64, dropout=0.0,
                         precision="fp32", backend="thunder")
    model = ESAModel(cfg, device="cuda")
    ids = torch.randint(0, 128, (2, 65), device="cuda")
    min_rows = ops.LAYER_NORM_MIN_ROWS
    ops.LAYER_NORM_MIN_ROWS = 0
    try:
        _, loss = model(ids[:, :-1], ids[:, 1:])
        loss.backward()
    finally:
        ops.LAYER_NORM_MIN_ROWS = min_rows
    grads = {n: p.grad.clone() for n, p in model.named_parameters() if p.grad is not None}
    model.zero_grad(set_to_none=True)
    orig = ops.layer_norm_supported
    ops.layer_norm_supported = lambda *a: False
    try:
        _, loss2 = model(ids[:, :-1], ids[:, 1:])
        loss2.backward()
    finally:
        ops.layer_norm_supported = orig
    assert abs(loss.item() - loss2.item()) < 1e-5 * abs(loss2.item())
    for n, p in model.named_parameters():
        if p.grad is not None:
            assert rel(grads[n], p.grad) < 1e-4, n


@pytest.mark.parametrize("xdt,rdt,ydt", [(torch.float32, torch.float16, torch.float16),
                                          (torch.float16, torch.float16, torch.float16),
                                          (torch.float32, torch.float32, torch.float32)])
def test_add_layer_norm_fwd_bwd(xdt, rdt, ydt):
    """xsum = x + res (x's dtype) and y = LayerNorm(xsum), against the separate
    torch add and norm; gradients through both outputs."""
    from esa import ops
    g = torch.Generator().manual_seed(32)
    C = 768
    shape = (2, 50, C)
    x = (torch.randn(shape, generator=g) * 2).to(xdt).cuda().requires_grad_(True)
    res = torch.randn(shape, generator=g).to(rdt).cuda().requires_grad_(True)
    w = (1 + 0.1 * torch.randn(C, generator=g)).cuda().requires_grad_(True)
    b = (0.1 * torch.randn(C, generator=g)).cuda().requires_grad_(True)
    xsum, y, _, _ = ops.add_layer_norm(x, res, w, b, 1e-5, ydt)
    xr = x.detach().clone().requires_grad_(True)
    rr = res.detach().clone().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    br = b.detach().clone().requires_grad_(True)
    sr = xr + rr                                   # torch's add, in x's dtype
    yr = torch.nn.functional.layer_norm(sr.double(), (C,), wr.double(), br.double(), 1e-5)
    assert xsum.dtype == xdt and torch.equal(xsum, sr)
    tol = 2e-6 if ydt == torch.float32 else 2e-3
    assert rel(y, yr) < tol
    dy = torch.randn(shape, generator=g).to(ydt).cuda()
    ds = torch.randn(shape, generator=g).to(xdt).cuda()
    ((y.double() * dy.double()).sum() + (xsum.double() * ds.double()).sum()).backward()
    ((yr * dy.double()).sum() + (sr.double() * ds.double()).sum()).backward()
    gtol = 2e-5 if xdt == torch.float32 and rdt == torch.float32 else 4e-3
    assert rel(x.grad, xr.grad) < gtol
    assert rel(res.grad, rr.grad) < gtol
    assert res.grad.dtype == rdt
    assert rel(w.grad, wr.grad) < gtol
    assert rel(b.grad, br.grad) < gtol
