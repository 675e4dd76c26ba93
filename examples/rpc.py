"""Remote procedure call: rank 1 serves function 7, rank 0 calls it.

    PYTHONPATH=. python examples/rpc.py
"""
import threading

from nexar_b200 import NexarClient


def main():
    clients = NexarClient.bootstrap_local(2)
    server = clients[1].rpc_dispatcher()
    server.register(7, lambda payload: payload.upper())  # handlers map bytes to bytes
    t = threading.Thread(target=server.serve_once, args=(0, 10.0))  # serve one request from rank 0
    t.start()
    reply = clients[0].rpc(1, 7, b"hello nexar", 10.0)
    t.join()
    print(f"rpc reply: {reply!r}")
    assert reply == b"HELLO NEXAR"
    for c in clients:
        c.close()


if __name__ == "__main__":
    main()
