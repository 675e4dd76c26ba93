"""The parallel training steps on CPU ranks (threads in one process): a
tensor-parallel MLP step, a two-stage 1F1B pipeline and a sharded-AdamW data
parallel step, each checked against the unsharded computation.

    PYTHONPATH=. python examples/parallel_cpu.py
"""
import torch

from nexar_b200 import NexarClient
from nexar_b200.parallel.pipeline import HostP2P, run_1f1b
from nexar_b200.parallel.tensor import HostTP, tp_mlp
from nexar_b200.parallel.zero import HostSharding, ShardedAdamW
from nexar_b200.utils.threads import run_ranks


def tensor_parallel(W=2, T=8, d=6, F=8):
    g = torch.Generator().manual_seed(0)
    x = torch.randn(T, d, generator=g, dtype=torch.float64)
    w_gu = torch.randn(2 * F, d, generator=g, dtype=torch.float64) * 0.3
    w_down = torch.randn(d, F, generator=g, dtype=torch.float64) * 0.3
    gu = x @ w_gu.t()
    want = (torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]) @ w_down.t()
    Fl = F // W
    clients = NexarClient.bootstrap_local(W)

    def rank_fn(c):
        r = c.rank
        rows = list(range(r * Fl, (r + 1) * Fl)) + list(range(F + r * Fl, F + (r + 1) * Fl))
        xs = x[r * T // W:(r + 1) * T // W]
        return tp_mlp(xs, w_gu[rows], w_down[:, r * Fl:(r + 1) * Fl], HostTP(c))

    got = torch.cat(run_ranks(clients, rank_fn))
    for c in clients:
        c.close()
    print(f"tensor parallel MLP over {W} ranks: max |error| {float((got - want).abs().max()):.2e}")


def pipeline(W=2, M=4, d=5):
    torch.manual_seed(0)
    stages = [torch.nn.Sequential(torch.nn.Linear(d, d), torch.nn.Tanh()).double() for _ in range(W)]
    mbs = [torch.randn(3, d, dtype=torch.float64) for _ in range(M)]
    clients = NexarClient.bootstrap_local(W)
    losses = run_ranks(clients, lambda c: run_1f1b(stages[c.rank], HostP2P(c), mbs, (3, d), torch.float64,
                                                  loss_fn=lambda y, i: (y ** 2).mean()))
    for c in clients:
        c.close()
    print(f"1F1B pipeline over {W} stages, {M} micro-batches: losses {[round(v, 4) for v in losses[-1]]}")


def sharded_adamw(W=2):
    def model():
        torch.manual_seed(0)
        return torch.nn.Linear(4, 3).double()
    models = [model() for _ in range(W)]
    x = torch.randn(W, 6, 4, dtype=torch.float64)
    clients = NexarClient.bootstrap_local(W)

    def rank_fn(c):
        opt = ShardedAdamW(models[c.rank].parameters(), HostSharding(c), lr=1e-2)
        models[c.rank](x[c.rank]).pow(2).mean().backward()
        opt.step()
        return opt.state_bytes()

    state = run_ranks(clients, rank_fn)
    for c in clients:
        c.close()
    same = all(torch.equal(p, q) for p, q in zip(models[0].parameters(), models[1].parameters()))
    print(f"sharded AdamW over {W} ranks: optimizer state per rank {state[0]} bytes, replicas equal: {same}")


if __name__ == "__main__":
    tensor_parallel()
    pipeline()
    sharded_adamw()
