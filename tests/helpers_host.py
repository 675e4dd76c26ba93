"""Test harness for host collectives: one thread per rank in one process over
real loopback TCP (the reference's run_collective, nexar/tests/collective/helpers.rs)."""
import threading

import numpy as np

from nexar_b200.client import Config, NexarClient


def bootstrap(n, **cfg):
    config = Config(**cfg) if cfg else None
    return NexarClient.bootstrap_local(n, config)


def run_collective(clients, fn, timeout=60):
    """Run fn(client) on every rank concurrently; returns results by rank; re-raises the first error."""
    res = [None] * len(clients)
    errs = [None] * len(clients)

    def go(i):
        try:
            res[i] = fn(clients[i])
        except BaseException as e:  # noqa: BLE001
            errs[i] = e

    ts = [threading.Thread(target=go, args=(i,), daemon=True) for i in range(len(clients))]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout)
        if t.is_alive():
            raise TimeoutError("collective did not finish")
    for e in errs:
        if e is not None:
            raise e
    return res


def data(rank, n, dtype=np.float32, seed=0):
    rs = np.random.RandomState(seed * 1000 + rank)
    if np.issubdtype(dtype, np.floating):
        return (rs.uniform(-1, 1, n) + 0.1 * rank).astype(dtype)
    return rs.randint(-20, 20, n).astype(dtype)
