"""GPT-2 trainer on one GPU: loss decreases, CUDA-graph replay matches eager."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_gpt2_tiny_trains(cuda0):
    from nexar_b200.models.gpt2 import GPT2Config
    from nexar_b200.parallel.dp import DataParallelTrainer
    cfg = GPT2Config.tiny()
    tr = DataParallelTrainer(cfg, micro_batch=4, seq_len=cfg.block_size, use_cuda_graph=False, lr=3e-3)
    g = torch.Generator().manual_seed(0)
    idx = torch.randint(0, cfg.vocab_size, (4, cfg.block_size), generator=g)
    tgt = torch.roll(idx, -1, dims=1)
    losses = [tr.step(idx, tgt) for _ in range(30)]
    assert losses[0] == pytest.approx(torch.log(torch.tensor(float(cfg.vocab_size))).item(), rel=0.1)
    assert losses[-1] < losses[0] - 0.5, losses


def test_gpt2_graph_matches_eager(cuda0):
    from nexar_b200.models.gpt2 import GPT2Config
    from nexar_b200.parallel.dp import DataParallelTrainer
    cfg = GPT2Config.tiny()
    g = torch.Generator().manual_seed(1)
    idx = torch.randint(0, cfg.vocab_size, (2, cfg.block_size), generator=g)
    tgt = torch.randint(0, cfg.vocab_size, (2, cfg.block_size), generator=g)
    a = DataParallelTrainer(cfg, 2, cfg.block_size, use_cuda_graph=False, seed=5)
    b = DataParallelTrainer(cfg, 2, cfg.block_size, use_cuda_graph=True, seed=5)
    for tr in (a, b):
        tr.set_batch(idx, tgt)
        tr.capture(warmup=3)
    la = [a.step(idx, tgt) for _ in range(3)]
    lb = [b.step(idx, tgt) for _ in range(3)]
    assert b.graph is not None and b.graph_launches > 0
    for x, y in zip(la, lb):
        assert x == pytest.approx(y, rel=2e-2, abs=2e-2)


def test_gpt2_loss_matches_torch_reference(cuda0):
    """Forward loss of our kernel path equals a plain torch fp32 GPT-2 on the same weights."""
    import math
    import torch.nn.functional as F
    from nexar_b200.models.gpt2 import GPT2, GPT2Config
    cfg = GPT2Config.tiny()
    m = GPT2(cfg, cuda0, seed=3)
    idx = torch.randint(0, cfg.vocab_size, (2, 32), device=cuda0)
    tgt = torch.randint(0, cfg.vocab_size, (2, 32), device=cuda0)
    with torch.no_grad():
        loss = m(idx, tgt).float()
        p = {k: v.float() for k, v in m.p.items()}
        B, T = idx.shape
        C, H = cfg.n_embd, cfg.n_head
        x = p["wte"][idx] + p["wpe"][:T]
        for l in range(cfg.n_layer):
            q = f"h{l}."
            h = F.layer_norm(x, (C,), p[q + "ln1.w"], p[q + "ln1.b"])
            qkv = h @ p[q + "attn.w"].t() + p[q + "attn.b"]
            qq, kk, vv = qkv.view(B, T, 3, H, C // H).unbind(2)
            y = F.scaled_dot_product_attention(qq.transpose(1, 2), kk.transpose(1, 2), vv.transpose(1, 2), is_causal=True)
            x = x + (y.transpose(1, 2).reshape(B, T, C) @ p[q + "proj.w"].t() + p[q + "proj.b"])
            h = F.layer_norm(x, (C,), p[q + "ln2.w"], p[q + "ln2.b"])
            f = F.gelu(h @ p[q + "fc.w"].t() + p[q + "fc.b"], approximate="tanh")
            x = x + (f @ p[q + "fcproj.w"].t() + p[q + "fcproj.b"])
        h = F.layer_norm(x, (C,), p["lnf.w"], p["lnf.b"])
        logits = (h @ p["wte"].t())[..., :cfg.vocab_size]
        ref = F.cross_entropy(logits.reshape(-1, cfg.vocab_size), tgt.reshape(-1))
    assert abs(loss.item() - ref.item()) < 0.05, (loss.item(), ref.item())


def test_gpt2_grads_match_torch_reference(cuda0):
    """Every parameter gradient of the kernel path (direct gradient sinks, MN-major
    backward GEMMs, folded residual biases) against fp32 torch autograd."""
    import torch.nn.functional as F
    from nexar_b200.models.gpt2 import GPT2, GPT2Config
    cfg = GPT2Config.tiny()
    m = GPT2(cfg, cuda0, seed=4)
    with torch.no_grad():  # non-trivial biases and LayerNorm affine so every path is exercised
        g = torch.Generator(device=cuda0).manual_seed(9)
        for name, p in m.p.items():
            if name.endswith(".b"):
                p.copy_(0.05 * torch.randn(p.shape, device=cuda0, generator=g))
            elif ".ln" in name or name.startswith("lnf"):
                p.copy_(1 + 0.1 * torch.randn(p.shape, device=cuda0, generator=g))
        m.flat.grad.fill_(7.0)  # stale values must be overwritten, not accumulated onto
    idx = torch.randint(0, cfg.vocab_size, (2, 64), device=cuda0)
    tgt = torch.randint(0, cfg.vocab_size, (2, 64), device=cuda0)
    loss = m(idx, tgt, unit_grad=True)
    loss.backward()
    torch.cuda.synchronize()
    p = {k: v.detach().float().requires_grad_(True) for k, v in m.p.items()}
    B, T = idx.shape
    C, H = cfg.n_embd, cfg.n_head
    x = p["wte"][idx] + p["wpe"][:T]
    for l in range(cfg.n_layer):
        q = f"h{l}."
        h = F.layer_norm(x, (C,), p[q + "ln1.w"], p[q + "ln1.b"])
        qkv = h @ p[q + "attn.w"].t() + p[q + "attn.b"]
        qq, kk, vv = qkv.view(B, T, 3, H, C // H).unbind(2)
        y = F.scaled_dot_product_attention(qq.transpose(1, 2), kk.transpose(1, 2), vv.transpose(1, 2), is_causal=True)
        x = x + (y.transpose(1, 2).reshape(B, T, C) @ p[q + "proj.w"].t() + p[q + "proj.b"])
        h = F.layer_norm(x, (C,), p[q + "ln2.w"], p[q + "ln2.b"])
        f = F.gelu(h @ p[q + "fc.w"].t() + p[q + "fc.b"], approximate="tanh")
        x = x + (f @ p[q + "fcproj.w"].t() + p[q + "fcproj.b"])
    h = F.layer_norm(x, (C,), p["lnf.w"], p["lnf.b"])
    logits = (h @ p["wte"].t())[..., :cfg.vocab_size]
    ref = F.cross_entropy(logits.reshape(-1, cfg.vocab_size), tgt.reshape(-1))
    ref.backward()
    assert abs(loss.item() - ref.item()) < 0.05
    bad = []
    for name, par in m.p.items():
        ours = m.flat.view(m.flat.grad, name).float()
        want = p[name].grad
        if name == "wpe":
            want = want.clone()
        err = ((ours - want).norm() / (want.norm() + 1e-6)).item()
        if err > 0.05:
            bad.append((name, round(err, 4)))
    assert not bad, bad
