"""tcgen05 self-attention (head dimension 64) against a plain PyTorch fp32
reference: forward output, the per-row log-sum-exp and the gradient of qkv,
causal and full, T from 128 to 2048 (odd and even tile counts; more
(key block, head) items than SMs, so that every persistent backward CTA
walks several items of different lengths), and one GPT-2
training step with it against the same step on torch SDPA."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _reference(qkv, B, T, H, causal):
    x = qkv.float().view(B, T, 3, H, 64)
    q, k, v = (t.transpose(1, 2) for t in x.unbind(2))  # [B, H, T, 64]
    s = q @ k.transpose(-1, -2) / 8.0
    if causal:
        s = s.masked_fill(torch.ones(T, T, dtype=torch.bool, device=qkv.device).triu(1), float("-inf"))
    y = torch.softmax(s, dim=-1) @ v
    return y.transpose(1, 2).reshape(B * T, H * 64)


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("B,T,H", [(1, 128, 1), (2, 256, 2), (1, 384, 3), (2, 1024, 4), (1, 2048, 2),
                                   (3, 1024, 20)])
def test_attention_matches_fp32_reference(cuda0, B, T, H, causal):
    from nexar_b200 import _native, ops
    g = torch.Generator(device="cuda").manual_seed(3)
    qkv = torch.randn(B * T, 3 * H * 64, device=cuda0, generator=g).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(B * T, H * 64, device=cuda0, generator=g).to(torch.bfloat16)
    y = ops.attention(qkv, B, T, H, causal=causal)
    y.backward(dy)
    torch.cuda.synchronize()
    assert int(_native.cuda().gemm_error_flag()) == 0
    ref_in = qkv.detach().float().requires_grad_(True)
    ref = _reference(ref_in, B, T, H, causal)
    ref.backward(dy.float())
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=2e-2)
    gmax = ref_in.grad.abs().max().item()
    torch.testing.assert_close(qkv.grad.float(), ref_in.grad, rtol=3e-2, atol=3e-2 * gmax)


def test_gpt2_step_with_own_attention_tracks_sdpa(cuda0):
    from nexar_b200.models.gpt2 import GPT2Config
    from nexar_b200.parallel.dp import DataParallelTrainer
    cfg = GPT2Config(n_layer=2, n_head=4, n_embd=256, vocab_size=1000, padded_vocab=1024, block_size=256)
    g = torch.Generator().manual_seed(5)
    idx = torch.randint(0, cfg.vocab_size, (2, cfg.block_size), generator=g)
    tgt = torch.randint(0, cfg.vocab_size, (2, cfg.block_size), generator=g)
    losses = {}
    for own in (False, True):
        tr = DataParallelTrainer(cfg, micro_batch=2, seq_len=cfg.block_size, use_cuda_graph=False, seed=0)
        tr.model.own_attention = own
        losses[own] = [tr.step(idx, tgt) for _ in range(3)]
    for a, b in zip(losses[False], losses[True]):
        assert abs(a - b) < 2e-2 * max(1.0, abs(a)), losses


@pytest.mark.parametrize("causal", [True, False])
def test_attention_lse_matches_logsumexp(cuda0, causal):
    """The saved per-row statistic is the natural-log softmax normaliser of the scaled scores."""
    from nexar_b200 import _native
    B, T, H = 2, 640, 3
    g = torch.Generator(device="cuda").manual_seed(4)
    qkv = torch.randn(B * T, 3 * H * 64, device=cuda0, generator=g).to(torch.bfloat16)
    y = torch.empty(B * T, H * 64, device=cuda0, dtype=torch.bfloat16)
    lse = torch.empty(B * H * T, device=cuda0)
    _native.cuda().attn_fwd(qkv, y, lse, B, T, H, causal)
    torch.cuda.synchronize()
    x = qkv.float().view(B, T, 3, H, 64)
    q, k = x[:, :, 0].transpose(1, 2), x[:, :, 1].transpose(1, 2)
    s = q @ k.transpose(-1, -2) / 8.0
    if causal:
        s = s.masked_fill(torch.ones(T, T, dtype=torch.bool, device=cuda0).triu(1), float("-inf"))
    ref = torch.logsumexp(s, dim=-1).reshape(-1)
    torch.testing.assert_close(lse, ref, rtol=1e-3, atol=1e-2)
