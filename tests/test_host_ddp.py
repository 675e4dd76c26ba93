"""Bucketed data-parallel wrapper (nexar_b200/parallel/ddp.py) on CPU ranks:
bucket all-reduces start during backward, and SGD on the averaged gradients
follows the full-batch trajectory of one model (fp64)."""
import pytest
import torch

from helpers_host import bootstrap, run_collective
from nexar_b200.parallel.ddp import DistributedDataParallel, HostBuckets


def _model():
    torch.manual_seed(0)
    return torch.nn.Sequential(torch.nn.Linear(6, 16), torch.nn.Tanh(), torch.nn.Linear(16, 16), torch.nn.Tanh(),
                               torch.nn.Linear(16, 2)).double()


@pytest.mark.parametrize("W", [2, 3])
def test_ddp_matches_full_batch_sgd(W):
    steps, rows, lr = 3, 5, 0.1
    g = torch.Generator().manual_seed(W)
    xs = torch.randn(steps, W, rows, 6, generator=g, dtype=torch.float64)
    ys = torch.randn(steps, W, rows, 2, generator=g, dtype=torch.float64)
    ref = _model()
    opt = torch.optim.SGD(ref.parameters(), lr=lr)
    for s in range(steps):
        opt.zero_grad()
        (sum(((ref(xs[s, r]) - ys[s, r]) ** 2).mean() for r in range(W)) / W).backward()
        opt.step()

    models = [_model() for _ in range(W)]
    clients = bootstrap(W)
    try:
        def rank_fn(c):
            ddp = DistributedDataParallel(models[c.rank], HostBuckets(c), bucket_bytes=600)
            sgd = torch.optim.SGD(ddp.parameters(), lr=lr)
            started = []
            for s in range(steps):
                sgd.zero_grad()
                ((ddp(xs[s, c.rank]) - ys[s, c.rank]) ** 2).mean().backward()
                started.append(len(ddp._inflight))
                ddp.finish()
                sgd.step()
            return len(ddp.buckets), started

        res = run_collective(clients, rank_fn)
    finally:
        for c in clients:
            c.close()
    nb, started = res[0]
    assert nb > 1 and all(s == nb for s in started)  # every bucket began during backward
    for m in models:
        for p, q in zip(m.parameters(), ref.parameters()):
            torch.testing.assert_close(p, q, rtol=1e-10, atol=1e-12)


def test_ddp_gradient_accumulation_with_no_sync():
    """Two micro-batches per step (the first under no_sync) follow full-batch
    SGD over both micro-batches of every rank; a second backward outside
    no_sync before finish() raises."""
    W, steps, rows, lr = 2, 2, 4, 0.1
    g = torch.Generator().manual_seed(11)
    xs = torch.randn(steps, W, 2, rows, 6, generator=g, dtype=torch.float64)
    ys = torch.randn(steps, W, 2, rows, 2, generator=g, dtype=torch.float64)
    ref = _model()
    opt = torch.optim.SGD(ref.parameters(), lr=lr)
    for s in range(steps):
        opt.zero_grad()
        (sum(((ref(xs[s, r, m]) - ys[s, r, m]) ** 2).mean() for r in range(W) for m in range(2)) / W).backward()
        opt.step()

    models = [_model() for _ in range(W)]
    clients = bootstrap(W)
    try:
        def rank_fn(c):
            ddp = DistributedDataParallel(models[c.rank], HostBuckets(c), bucket_bytes=600)
            sgd = torch.optim.SGD(ddp.parameters(), lr=lr)
            for s in range(steps):
                sgd.zero_grad()
                with ddp.no_sync():
                    ((ddp(xs[s, c.rank, 0]) - ys[s, c.rank, 0]) ** 2).mean().backward()
                assert not ddp._inflight
                ((ddp(xs[s, c.rank, 1]) - ys[s, c.rank, 1]) ** 2).mean().backward()
                ddp.finish()
                sgd.step()
            # a second backward outside no_sync before finish() is refused
            ((ddp(xs[0, c.rank, 0]) - ys[0, c.rank, 0]) ** 2).mean().backward()
            with pytest.raises(RuntimeError, match="no_sync"):
                ((ddp(xs[0, c.rank, 1]) - ys[0, c.rank, 1]) ** 2).mean().backward()
            return True

        run_collective(clients, rank_fn)
    finally:
        for c in clients:
            c.close()
    for m in models:
        for p, q in zip(m.parameters(), ref.parameters()):
            torch.testing.assert_close(p, q, rtol=1e-10, atol=1e-12)
