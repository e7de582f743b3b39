"""Parity of the fused ESAModel decode step (esa_decode_block, esa_decode_head).

A decode step of a few rows of a 16-bit model runs each block in four
launches (residual add + LN1 + qgv GEMV; Lightning step + out_proj; add + LN2
+ fc + GELU; proj) and the head in one.  The reference is the same
computation in plain PyTorch fp32 with the 16-bit rounding at the points
where the PyTorch path rounds (residual sums, LayerNorm outputs, every Linear
output, GELU, the Lightning state and readout).  Bar: relative Frobenius error
2e-3 for fp16 and 5e-3 for bf16 (the kernels' fp32 sums run in another order,
so a few elements round one unit differently).
"""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 5e-3}


def rel(a, b) -> float:
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _block_params(C, dtype, g, bias=True):
    def w(o, i):
        return (torch.randn(o, i, generator=g) / i ** 0.5).to(dtype).cuda()

    def v(n, scale=0.1, base=0.0):
        return (base + scale * torch.randn(n, generator=g)).to(dtype).cuda()

    return dict(ln1_w=v(C, 0.1, 1.0), ln1_b=v(C) if bias else None, qgv_w=w(3 * C, C), qgv_b=v(3 * C) if bias else None,
                out_w=w(C, C), out_b=v(C) if bias else None, ln2_w=v(C, 0.1, 1.0), ln2_b=v(C) if bias else None,
                fc_w=w(4 * C, C), fc_b=v(4 * C) if bias else None, proj_w=w(C, 4 * C), proj_b=v(C) if bias else None)


def _reference_block(x, pending, state, P, gmin, gmax, eps, dtype):
    C = x.shape[1]
    f = lambda t: None if t is None else t.float()  # noqa: E731
    r = lambda t: t.to(dtype).float()  # noqa: E731

    def lin(h, w, b):
        y = h @ f(w).T
        return r(y if b is None else y + f(b))

    s1 = f(x) if pending is None else r(f(x) + f(pending))
    h1 = r(F.layer_norm(s1, (C,), f(P["ln1_w"]), f(P["ln1_b"]), 1e-5))
    qgv = lin(h1, P["qgv_w"], P["qgv_b"])
    q, gg, vv = qgv[:, :C], qgv[:, C:2 * C], qgv[:, 2 * C:]
    A = gmin + (gmax - gmin) * torch.sigmoid(gg)
    B = (1 - A) * torch.tanh(vv)
    sp = r(r(A) * f(state) + r(B))
    rr = torch.rsqrt((sp * sp).mean(dim=1, keepdim=True) + eps)
    z = r(torch.sigmoid(q) * sp * rr)
    y = lin(z, P["out_w"], P["out_b"])
    s2 = r(s1 + y)
    h2 = r(F.layer_norm(s2, (C,), f(P["ln2_w"]), f(P["ln2_b"]), 1e-5))
    a = r(F.gelu(lin(h2, P["fc_w"], P["fc_b"])))
    p = lin(a, P["proj_w"], P["proj_b"])
    return s2, p, sp


def _run_block(x, pending, state, P, gmin, gmax, eps):
    from esa import _lib, ops
    nb, C = x.shape
    L = _lib.lib()
    code = ops.dtype_code(x.dtype)
    x_out, p_out, ns = torch.empty_like(x), torch.empty_like(x), torch.empty_like(state)
    scratch = torch.empty(L.esa_decode_block_scratch_bytes(nb, C, code), dtype=torch.uint8, device="cuda")
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    rc = L.esa_decode_block(x.data_ptr(), ptr(pending), x_out.data_ptr(), p_out.data_ptr(), state.data_ptr(),
                            ns.data_ptr(), *(ptr(P[k]) for k in ("ln1_w", "ln1_b", "qgv_w", "qgv_b", "out_w", "out_b",
                                                               "ln2_w", "ln2_b", "fc_w", "fc_b", "proj_w", "proj_b")),
                            nb, C, code, gmin, gmax, eps, 1e-5, scratch.data_ptr(), scratch.numel(),
                            torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "esa_decode_block")
    torch.cuda.synchronize()
    return x_out, p_out, ns


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("nb,C,with_pending,bias", [(1, 1024, False, True), (1, 1024, True, True),
                                                    (3, 256, True, True), (4, 512, True, False),
                                                    (2, 1024, True, True)])
def test_decode_block_matches_reference(dtype, nb, C, with_pending, bias):
    g = torch.Generator().manual_seed(100 + nb + C)
    P = _block_params(C, dtype, g, bias=bias)
    x = torch.randn(nb, C, generator=g).to(dtype).cuda()
    pending = torch.randn(nb, C, generator=g).to(dtype).cuda() if with_pending else None
    state = (0.5 * torch.randn(nb, C, generator=g)).to(dtype).cuda()
    gmin, gmax, eps = 0.8, 0.995, 1e-5
    x_out, p_out, ns = _run_block(x, pending, state, P, gmin, gmax, eps)
    s2, p, sp = _reference_block(x, pending, state, P, gmin, gmax, eps, dtype)
    assert rel(ns, sp) < TOL[dtype]
    assert rel(x_out, s2) < TOL[dtype]
    assert rel(p_out, p) < TOL[dtype]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_decode_head_matches_reference(dtype):
    from esa import _lib, ops
    g = torch.Generator().manual_seed(7)
    nb, C, V = 2, 1024, 32000
    x = torch.randn(nb, C, generator=g).to(dtype).cuda()
    pending = torch.randn(nb, C, generator=g).to(dtype).cuda()
    lw = (1 + 0.1 * torch.randn(C, generator=g)).to(dtype).cuda()
    lb = (0.1 * torch.randn(C, generator=g)).to(dtype).cuda()
    W = (torch.randn(V, C, generator=g) / C ** 0.5).to(dtype).cuda()
    logits = torch.empty(nb, V, dtype=dtype, device="cuda")
    rc = _lib.lib().esa_decode_head(x.data_ptr(), pending.data_ptr(), lw.data_ptr(), lb.data_ptr(), 1e-5, W.data_ptr(),
                                    None, logits.data_ptr(), nb, C, V, ops.dtype_code(dtype),
                                    torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "esa_decode_head")
    r = lambda t: t.to(dtype).float()  # noqa: E731
    s = r(x.float() + pending.float())
    h = r(F.layer_norm(s, (C,), lw.float(), lb.float(), 1e-5))
    ref = r(h @ W.float().T)
    assert rel(logits, ref) < TOL[dtype]
    assert torch.equal(torch.argmax(logits, dim=-1), torch.argmax(ref, dim=-1))


def _small_model(dtype):
    from esa import ESAModel, ESAModelConfig
    torch.manual_seed(5)
    cfg = ESAModelConfig(vocab_size=2048, n_layer=3, embd=512, head=8, block=256, dropout=0.0, precision="fp16")
    return ESAModel(cfg, device="cuda").eval().to(dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_model_step_fused_against_unfused(dtype, monkeypatch):
    """ESAModel.lightning_step with the fused decode kernels against the same
    step on the per-op PyTorch path (the kernels switched off)."""
    from esa import ops
    model = _small_model(dtype)
    B = 3
    g = torch.Generator().manual_seed(9)
    token = torch.randint(0, 2048, (B,), generator=g).cuda()
    states = (0.3 * torch.randn(3, B, 8, 64, generator=g)).to(dtype).cuda()
    pos = torch.tensor(17, device="cuda")
    with torch.inference_mode():
        logits, new_states = model.lightning_step(token, states, pos)
        monkeypatch.setattr(ops, "decode_block_supported", lambda x, block: False)
        monkeypatch.setattr(ops, "decode_head_supported", lambda x, ln_f, head: False)
        ref_logits, ref_states = model.lightning_step(token, states, pos)
    assert rel(new_states, ref_states) < 2 * TOL[dtype]
    assert rel(logits, ref_logits) < 2 * TOL[dtype]


def test_greedy_decode_graph_equals_eager_with_fused_kernels():
    """The CUDA-graph decode driver replays the same fused kernels as the eager
    loop: identical greedy ids (both paths are deterministic)."""
    model = _small_model(torch.float16)
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, 2048, (2, 40), generator=g).cuda()
    a = model.generate(input_ids=ids, seek=24, prefill="thunder_16", temperature=0.0, compile=False,
                       decode_graph=True)
    b = model.generate(input_ids=ids, seek=24, prefill="thunder_16", temperature=0.0, compile=False,
                       decode_graph=False)
    assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_graph_prefill_equals_eager_prefill(dtype):
    """generate() with graph decoding replays a captured prefill per prompt
    shape: its logits and states equal the eager prefill's bits, on a first
    (capturing) and a second (replaying) prompt of the same shape."""
    model = _small_model(dtype)
    g = torch.Generator().manual_seed(13)
    for _ in range(2):
        ids = torch.randint(0, 2048, (2, 37), generator=g).cuda()
        with torch.inference_mode():
            logits, states, T = model._prefill_for_generate(ids, "thunder_16", "default", True)
            ref_logits, ref_states, ref_T = model._prefill_eager(ids, backend="thunder", compass=16)
        assert T == ref_T == 37
        assert torch.equal(logits, ref_logits)
        assert torch.equal(states, ref_states)
    assert len(model._prefill_graphs) == 1 and not model._prefill_graph_failures
