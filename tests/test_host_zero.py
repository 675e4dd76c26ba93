"""Sharded AdamW (nexar_b200/parallel/zero.py) on CPU ranks: after several steps
on per-rank data shards, every rank's parameters equal those of one model
trained with full-batch AdamW on the averaged gradient (fp64)."""
import pytest
import torch

from helpers_host import bootstrap, run_collective
from nexar_b200.parallel.zero import HostSharding, ShardedAdamW


def _model(seed):
    torch.manual_seed(seed)
    return torch.nn.Sequential(torch.nn.Linear(5, 7), torch.nn.Tanh(), torch.nn.Linear(7, 3)).double()


@pytest.mark.parametrize("W", [2, 3, 4])
def test_sharded_adamw_matches_full_batch(W):
    steps, rows = 3, 4
    g = torch.Generator().manual_seed(W)
    xs = torch.randn(steps, W, rows, 5, generator=g, dtype=torch.float64)
    ys = torch.randn(steps, W, rows, 3, generator=g, dtype=torch.float64)
    kw = dict(lr=1e-2, betas=(0.9, 0.99), eps=1e-8, weight_decay=0.1)

    ref = _model(0)
    opt = torch.optim.AdamW(ref.parameters(), **kw)
    for s in range(steps):
        opt.zero_grad()
        loss = sum(((ref(xs[s, r]) - ys[s, r]) ** 2).mean() for r in range(W)) / W
        loss.backward()
        opt.step()

    models = [_model(0) for _ in range(W)]
    clients = bootstrap(W)
    try:
        def rank_fn(c):
            m = models[c.rank]
            zopt = ShardedAdamW(m.parameters(), HostSharding(c), **kw)
            for s in range(steps):
                zopt.zero_grad()
                ((m(xs[s, c.rank]) - ys[s, c.rank]) ** 2).mean().backward()
                zopt.step()
            return zopt.state_bytes()

        state = run_collective(clients, rank_fn)
    finally:
        for c in clients:
            c.close()
    n = sum(p.numel() for p in ref.parameters())
    assert all(b == 3 * ((n + W - 1) // W) * 8 for b in state)
    for m in models:
        for p, q in zip(m.parameters(), ref.parameters()):
            torch.testing.assert_close(p, q, rtol=1e-10, atol=1e-12)
