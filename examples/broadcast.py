"""Broadcast from a non-zero root over four ranks.

    PYTHONPATH=. python examples/broadcast.py
"""
import numpy as np

from nexar_b200 import NexarClient
from nexar_b200.utils.threads import run_ranks


def main():
    world, root = 4, 2
    clients = NexarClient.bootstrap_local(world)
    bufs = {c.rank: (np.arange(6, dtype=np.float32) if c.rank == root else np.zeros(6, np.float32))
            for c in clients}
    run_ranks(clients, lambda c: c.broadcast_host(bufs[c.rank], root))
    for r in range(world):
        print(f"rank {r}: {bufs[r]}")
        assert (bufs[r] == np.arange(6)).all()
    for c in clients:
        c.close()


if __name__ == "__main__":
    main()
