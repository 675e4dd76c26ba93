"""Cluster set-up the way it runs across machines: a seed node assigns ranks,
workers join through it, then every worker builds its part of the mesh.

    PYTHONPATH=. python examples/seed_worker.py                 # all roles in this process
    # or, across processes / machines:
    python -c "from nexar_b200 import SeedNode; s = SeedNode('0.0.0.0:5000'); s.form_cluster(2)"
    NEXAR_CLUSTER_TOKEN=<token> python -c "from nexar_b200 import NexarClient; \\
        c = NexarClient.bootstrap('seed-host:5000', bind_host='<this host>')"
"""
import threading

import numpy as np

from nexar_b200 import NexarClient, SeedNode, WorkerNode
from nexar_b200.utils.threads import run_ranks


def main():
    world = 2
    seed = SeedNode(local=True)  # no token on loopback
    print(f"seed listening on {seed.local_addr()}")

    infos = [None] * world

    def join(i):
        infos[i] = WorkerNode.connect(seed.local_addr())

    ts = [threading.Thread(target=join, args=(i,)) for i in range(world)]
    [t.start() for t in ts]
    seed.form_cluster(world)  # returns once every worker has joined
    [t.join() for t in ts]
    for w in infos:
        print(f"worker rank={w.rank} world_size={w.world_size} peers={w.peers}")

    clients = run_ranks(infos, lambda w: NexarClient.from_worker(w))
    bufs = {c.rank: np.full(3, float(c.rank + 1), np.float32) for c in clients}
    run_ranks(clients, lambda c: c.all_reduce_host(bufs[c.rank]))
    print(f"cluster formed: {len(clients)} ranks; all-reduce gives {bufs[0]}")
    assert all((b == 3).all() for b in bufs.values())
    for c in clients:
        c.close()
    seed.close()


if __name__ == "__main__":
    main()
