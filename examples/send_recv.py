"""Tagged point-to-point between two ranks in one process.

    PYTHONPATH=. python examples/send_recv.py
"""
import numpy as np

from nexar_b200 import NexarClient
from nexar_b200.utils.threads import run_ranks


def main():
    clients = NexarClient.bootstrap_local(2)

    def rank_fn(c):
        buf = np.zeros(4, np.float32)
        if c.rank == 0:
            buf[:] = [1, 2, 3, 4]
            c.send(buf.ctypes.data, buf.nbytes, dest=1, tag=42)
            return None
        c.recv(buf.ctypes.data, buf.nbytes, src=0, tag=42)
        return buf.tolist()

    got = run_ranks(clients, rank_fn)[1]
    print(f"rank 1 received {got}")
    assert got == [1, 2, 3, 4]
    for c in clients:
        c.close()


if __name__ == "__main__":
    main()
