"""Ulysses sequence-parallel attention on CPU ranks (threads over loopback):
outputs and qkv gradients of every rank's token shard equal those of plain
attention over the whole sequence."""
import pytest
import torch

from helpers_host import bootstrap, run_collective
from nexar_b200.parallel.sequence import HostAllToAll, ulysses_attention


def _full(qkv, B, T, H, D, causal):
    x = qkv.view(B, T, 3, H, D)
    q, k, v = (t.transpose(1, 2) for t in x.unbind(2))
    y = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=causal)
    return y.transpose(1, 2).reshape(B * T, H * D)


@pytest.mark.parametrize("W,causal", [(2, True), (4, True), (4, False)])
def test_ulysses_matches_full_attention(W, causal):
    B, T, H, D = 2, 32, 8, 16
    Tl = T // W
    g = torch.Generator().manual_seed(W)
    qkv = torch.randn(B, T, 3 * H * D, generator=g, dtype=torch.float64)
    dy = torch.randn(B, T, H * D, generator=g, dtype=torch.float64)
    ref_in = qkv.reshape(B * T, -1).clone().requires_grad_(True)
    ref = _full(ref_in, B, T, H, D, causal)
    ref.backward(dy.reshape(B * T, -1))
    ref_y = ref.detach().view(B, T, H * D)
    ref_g = ref_in.grad.view(B, T, -1)

    clients = bootstrap(W)
    try:
        def rank_fn(c):
            r = c.rank
            x = qkv[:, r * Tl:(r + 1) * Tl].reshape(B * Tl, -1).clone().requires_grad_(True)
            y = ulysses_attention(x, B, Tl, H, D, HostAllToAll(c), causal=causal)
            y.backward(dy[:, r * Tl:(r + 1) * Tl].reshape(B * Tl, -1))
            return y.detach().view(B, Tl, -1), x.grad.view(B, Tl, -1)

        out = run_collective(clients, rank_fn)
    finally:
        for c in clients:
            c.close()
    for r, (y, gx) in enumerate(out):
        torch.testing.assert_close(y, ref_y[:, r * Tl:(r + 1) * Tl], rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(gx, ref_g[:, r * Tl:(r + 1) * Tl], rtol=1e-10, atol=1e-10)


def test_heads_must_split_over_ranks():
    class One:
        world_size = 3
    with pytest.raises(ValueError, match="heads"):
        ulysses_attention(torch.zeros(4, 3 * 4 * 8), 1, 4, 4, 8, One())
