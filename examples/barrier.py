"""Barrier: no rank leaves before every rank has arrived.

    PYTHONPATH=. python examples/barrier.py
"""
import threading
import time

from nexar_b200 import NexarClient
from nexar_b200.utils.threads import run_ranks


def main():
    world = 4
    clients = NexarClient.bootstrap_local(world)
    arrived = []
    lock = threading.Lock()

    def rank_fn(c):
        time.sleep(0.05 * c.rank)  # ranks arrive at different times
        with lock:
            arrived.append(c.rank)
        c.barrier()
        with lock:
            return len(arrived)  # how many had arrived when this rank left

    seen = run_ranks(clients, rank_fn)
    print(f"ranks saw {seen} arrivals when leaving the barrier")
    assert all(n == world for n in seen)
    for c in clients:
        c.close()


if __name__ == "__main__":
    main()
