"""In-place all-reduce (sum) over four ranks in one process.

    PYTHONPATH=. python examples/allreduce.py
"""
import numpy as np

from nexar_b200 import NexarClient, ReduceOp
from nexar_b200.utils.threads import run_ranks


def main():
    world = 4
    clients = NexarClient.bootstrap_local(world)
    # rank r contributes [r+1, r+1, ...]; the sum is 1+2+...+world everywhere
    bufs = {c.rank: np.full(8, float(c.rank + 1), np.float32) for c in clients}
    run_ranks(clients, lambda c: c.all_reduce_host(bufs[c.rank], ReduceOp.Sum))
    want = world * (world + 1) / 2
    for r in range(world):
        print(f"rank {r}: {bufs[r][:4]}")
        assert (bufs[r] == want).all()
    for c in clients:
        c.close()


if __name__ == "__main__":
    main()
