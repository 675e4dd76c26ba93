"""1F1B pipeline schedule (nexar_b200/parallel/pipeline.py) on CPU ranks: the
losses and every stage's parameter gradients equal those of the whole model
run on the same micro-batches."""
import pytest
import torch

from helpers_host import bootstrap, run_collective
from nexar_b200.parallel.pipeline import HostP2P, run_1f1b, schedule_1f1b


def _stages(W, d, seed=0):
    torch.manual_seed(seed)
    return [torch.nn.Sequential(torch.nn.Linear(d, d), torch.nn.Tanh()).double() for _ in range(W)]


def test_schedule_shape():
    for W, M in [(4, 6), (4, 2), (2, 5), (1, 3)]:
        for s in range(W):
            sch = schedule_1f1b(s, W, M)
            assert [i for k, i in sch if k == "F"] == list(range(M))
            assert [i for k, i in sch if k == "B"] == list(range(M))
            inflight, peak = 0, 0
            for k, _ in sch:
                inflight += 1 if k == "F" else -1
                peak = max(peak, inflight)
            assert peak <= min(W - s, M)


@pytest.mark.parametrize("W,M", [(2, 5), (4, 6), (4, 2)])
def test_1f1b_matches_whole_model(W, M):
    d, rows = 6, 3
    g = torch.Generator().manual_seed(W * 10 + M)
    mbs = [torch.randn(rows, d, generator=g, dtype=torch.float64) for _ in range(M)]
    tgts = [torch.randn(rows, d, generator=g, dtype=torch.float64) for _ in range(M)]

    ref = _stages(W, d)
    whole = torch.nn.Sequential(*ref)
    ref_losses = []
    for x, t in zip(mbs, tgts):
        loss = ((whole(x) - t) ** 2).mean()
        loss.backward()
        ref_losses.append(float(loss.detach()))

    stages = _stages(W, d)
    clients = bootstrap(W)
    try:
        def rank_fn(c):
            mod = stages[c.rank]
            return run_1f1b(mod, HostP2P(c), mbs, (rows, d), torch.float64,
                            loss_fn=lambda y, i: ((y - tgts[i]) ** 2).mean())

        out = run_collective(clients, rank_fn)
    finally:
        for c in clients:
            c.close()
    assert out[-1] == pytest.approx(ref_losses, rel=1e-12)
    assert all(o == [] for o in out[:-1])
    for s in range(W):
        for p, q in zip(stages[s].parameters(), ref[s].parameters()):
            torch.testing.assert_close(p.grad, q.grad, rtol=1e-10, atol=1e-12)


def test_pipeline_dead_stage_errors_not_hangs():
    """A stage that leaves makes its neighbour's transfer fail within the
    collective timeout (the reference's fault-injection rule: error, not deadlock)."""
    import time

    from nexar_b200.core import NexarError
    d, rows, M = 4, 2, 3
    stages = _stages(2, d)
    clients = bootstrap(2, collective_timeout_s=2.0, heartbeat_interval_s=0.1, heartbeat_timeout_s=0.5)
    clients[1].close()
    mbs = [torch.randn(rows, d, dtype=torch.float64) for _ in range(M)]
    t0 = time.time()
    with pytest.raises(NexarError):
        run_1f1b(stages[0], HostP2P(clients[0]), mbs, (rows, d), torch.float64)
    assert time.time() - t0 < 30
    clients[0].close()
