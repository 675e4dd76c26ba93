"""Numerics of the model kernels against plain PyTorch fp32 references."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _bf(t):
    return t.to(torch.bfloat16)


def test_native_extension_is_loaded():
    from nexar_b200 import _native
    C = _native.cuda()
    assert C.__file__.endswith(".so")


@pytest.mark.parametrize("R,C", [(64, 768), (37, 256), (16, 1024), (9, 2048)])
def test_layernorm_fwd_bwd(cuda0, R, C):
    from nexar_b200 import ops
    torch.manual_seed(0)
    x = _bf(torch.randn(R, C, device=cuda0))
    r = _bf(torch.randn(R, C, device=cuda0))
    w = _bf(1 + 0.1 * torch.randn(C, device=cuda0))
    b = _bf(0.1 * torch.randn(C, device=cuda0))
    dy = _bf(torch.randn(R, C, device=cuda0))
    ds = _bf(torch.randn(R, C, device=cuda0))
    # fused residual + LN
    xs, rs, ws, bs = (t.clone().requires_grad_(True) for t in (x, r, w, b))
    s, y = ops.residual_layer_norm(xs, rs, ws, bs, 1e-5)
    torch.autograd.backward([s, y], [ds, dy])
    # fp32 reference
    xf, rf, wf, bf = (t.float().clone().requires_grad_(True) for t in (x, r, w, b))
    sf = (xf + rf)
    sf_b = sf.to(torch.bfloat16).float()  # kernel keeps the residual stream in bf16
    yf = torch.nn.functional.layer_norm(sf_b, (C,), wf, bf, 1e-5)
    torch.autograd.backward([sf, yf], [ds.float(), dy.float()])
    torch.testing.assert_close(s.float(), sf_b, atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(y.float(), yf, atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(xs.grad.float(), xf.grad, atol=6e-2, rtol=3e-2)
    torch.testing.assert_close(rs.grad.float(), rf.grad, atol=6e-2, rtol=3e-2)
    torch.testing.assert_close(ws.grad.float(), wf.grad, atol=0.25, rtol=3e-2)
    torch.testing.assert_close(bs.grad.float(), bf.grad, atol=0.25, rtol=3e-2)


@pytest.mark.parametrize("R,C", [(8192, 768), (300, 256)])
def test_residual_layernorm_with_branch_bias(cuda0, R, C):
    """s = x + r + rb; the backward returns d(rb) = column sums of ds (fused)."""
    from nexar_b200 import ops
    torch.manual_seed(1)
    x, r = _bf(torch.randn(R, C, device=cuda0)), _bf(torch.randn(R, C, device=cuda0))
    w = _bf(1 + 0.1 * torch.randn(C, device=cuda0))
    b, rb = _bf(0.1 * torch.randn(C, device=cuda0)), _bf(0.1 * torch.randn(C, device=cuda0))
    dy, ds = _bf(torch.randn(R, C, device=cuda0)), _bf(torch.randn(R, C, device=cuda0))
    xs, rs, ws, bs, rbs = (t.clone().requires_grad_(True) for t in (x, r, w, b, rb))
    s, y = ops.residual_layer_norm(xs, rs, ws, bs, 1e-5, rbias=rbs)
    torch.autograd.backward([s, y], [ds, dy])
    xf, rf, wf, bf, rbf = (t.float().clone().requires_grad_(True) for t in (x, r, w, b, rb))
    sf = xf + rf + rbf
    yf = torch.nn.functional.layer_norm(sf.to(torch.bfloat16).float(), (C,), wf, bf, 1e-5)
    torch.autograd.backward([sf, yf], [ds.float(), dy.float()])
    torch.testing.assert_close(y.float(), yf, atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(xs.grad.float(), xf.grad, atol=6e-2, rtol=3e-2)
    for ours, ref in ((ws.grad, wf.grad), (bs.grad, bf.grad), (rbs.grad, rbf.grad)):
        assert ((ours.float() - ref).norm() / ref.norm()).item() < 1e-2


@pytest.mark.parametrize("R,C", [(8192, 2304), (1000, 768), (5, 64)])
def test_colsum(cuda0, R, C):
    from nexar_b200 import ops
    x = _bf(torch.randn(R, C, device=cuda0))
    out = torch.empty(C, device=cuda0, dtype=torch.bfloat16)
    ops.colsum(x, out)
    ref = x.float().sum(0)
    torch.testing.assert_close(out.float(), ref, atol=0.05 * math.sqrt(R) / 8 + 1e-2, rtol=1e-2)
    base = _bf(torch.randn(C, device=cuda0))
    out2 = base.clone()
    ops.colsum(x, out2, accumulate=True)
    torch.testing.assert_close(out2.float(), ref + base.float(), atol=0.05 * math.sqrt(R) / 8 + 1e-2, rtol=1e-2)


def test_plain_layernorm(cuda0):
    from nexar_b200 import ops
    x = _bf(torch.randn(128, 768, device=cuda0))
    w = _bf(torch.ones(768, device=cuda0))
    b = _bf(torch.zeros(768, device=cuda0))
    y = ops.layer_norm(x, w, b)
    ref = torch.nn.functional.layer_norm(x.float(), (768,), w.float(), b.float())
    torch.testing.assert_close(y.float(), ref, atol=3e-2, rtol=2e-2)


def test_gelu(cuda0):
    from nexar_b200 import ops
    x = _bf(3 * torch.randn(4096, device=cuda0)).requires_grad_(True)
    y = ops.gelu(x)
    dy = _bf(torch.randn(4096, device=cuda0))
    y.backward(dy)
    xf = x.detach().float().requires_grad_(True)
    yf = torch.nn.functional.gelu(xf, approximate="tanh")
    yf.backward(dy.float())
    torch.testing.assert_close(y.float(), yf, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(x.grad.float(), xf.grad, atol=3e-2, rtol=3e-2)


def test_swiglu(cuda0):
    from nexar_b200 import ops
    R, F = 33, 256
    gu = _bf(torch.randn(R, 2 * F, device=cuda0)).requires_grad_(True)
    y = ops.swiglu(gu)
    dy = _bf(torch.randn(R, F, device=cuda0))
    y.backward(dy)
    gf = gu.detach().float().requires_grad_(True)
    g, u = gf[:, :F], gf[:, F:]
    yf = torch.nn.functional.silu(g) * u
    yf.backward(dy.float())
    torch.testing.assert_close(y.float(), yf, atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(gu.grad.float(), gf.grad, atol=5e-2, rtol=3e-2)


@pytest.mark.parametrize("R,V,Vp", [(16, 50257, 50304), (7, 1000, 1024), (5, 13, 16)])
def test_cross_entropy(cuda0, R, V, Vp):
    from nexar_b200 import ops
    torch.manual_seed(1)
    logits = _bf(2 * torch.randn(R, Vp, device=cuda0))
    tgt = torch.randint(0, V, (R,), device=cuda0)
    ref_logits = logits.float()[:, :V].clone().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(ref_logits, tgt)
    ref.backward()
    l = logits.clone().requires_grad_(True)
    loss = ops.cross_entropy(l, tgt, V)
    loss.backward()
    torch.testing.assert_close(loss.float(), ref, atol=2e-3, rtol=2e-3)
    g = l.grad.float()
    torch.testing.assert_close(g[:, :V], ref_logits.grad, atol=2e-3, rtol=5e-2)
    assert torch.all(g[:, V:] == 0)


def test_embedding(cuda0):
    from nexar_b200 import ops
    B, T, C, V = 3, 16, 64, 50
    tok = torch.randint(0, V, (B, T), device=cuda0)
    wte = _bf(torch.randn(V, C, device=cuda0)).requires_grad_(True)
    wpe = _bf(torch.randn(T, C, device=cuda0)).requires_grad_(True)
    out = ops.embedding(tok, wte, wpe)
    d = _bf(torch.randn(B, T, C, device=cuda0))
    out.backward(d)
    wtef = wte.detach().float().requires_grad_(True)
    wpef = wpe.detach().float().requires_grad_(True)
    ref = wtef[tok] + wpef[torch.arange(T, device=cuda0)][None]
    ref.backward(d.float())
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(wte.grad.float(), wtef.grad, atol=5e-2, rtol=3e-2)
    torch.testing.assert_close(wpe.grad.float(), wpef.grad, atol=5e-2, rtol=3e-2)


def test_adamw_and_clip(cuda0):
    from nexar_b200 import _native
    C = _native.cuda()
    n = 10007
    torch.manual_seed(2)
    p = torch.randn(n, device=cuda0)
    m = torch.zeros(n, device=cuda0)
    v = torch.zeros(n, device=cuda0)
    g = _bf(torch.randn(n, device=cuda0))
    pb = torch.empty(n, dtype=torch.bfloat16, device=cuda0)
    scratch = torch.empty(C.grad_norm_blocks(n), device=cuda0)
    counter = torch.zeros(4, dtype=torch.int32, device=cuda0)
    norm = torch.zeros(1, device=cuda0)
    coef = torch.zeros(1, device=cuda0)
    C.grad_norm_clip(g, 1.0, scratch, counter, norm, coef)
    gn = g.float().norm()
    torch.testing.assert_close(norm[0], gn, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(coef[0], torch.clamp(1.0 / (gn + 1e-6), max=1.0), rtol=1e-4, atol=1e-6)
    decay_end = 6000
    ref_p = p.clone()
    ref = torch.optim.AdamW([ref_p.requires_grad_(True)], lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.0)
    # reference: decoupled decay only on the first decay_end elements
    for step in (1, 2):
        ref_p.grad = g.float() * coef[0]
        with torch.no_grad():
            ref_p[:decay_end] -= 1e-3 * 0.1 * ref_p[:decay_end]
        ref.step()
        step_dev = torch.full((1,), step, dtype=torch.int32, device=cuda0)
        C.adamw(p, m, v, g, pb, decay_end, 1e-3, 0.9, 0.95, 1e-8, 0.1, step, coef, step_dev, None)
    torch.testing.assert_close(p, ref_p.detach(), rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(pb.float(), p, rtol=1e-2, atol=1e-2)
