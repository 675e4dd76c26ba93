"""Host (CPU adapter) collective sweep over loopback TCP: the reference's
"CPU ring all_reduce" configuration (``NexarClient::bootstrap_local(4,
CpuAdapter)``, f32 buffers drawn U(-1, 1) from seed = rank, Sum in place, then
all_gather and reduce_scatter; every rank must equal the elementwise sum),
timed over message sizes.

    python -m nexar_b200.bench.cpu_ring [--ranks 4] [--min-bytes 4096] [--max-bytes 67108864]
                                        [--iters 20] [--warmup 3] [--dtype f32|bf16] [--tls] [--out sweep.jsonl]

One thread per rank in one process (as the reference's tests and this
config). Each size: a barrier, ``iters`` back-to-back calls per rank, the
time of the slowest rank. Bus bandwidth uses the usual factors: all_reduce
2(n-1)/n x bytes, all_gather / reduce_scatter (n-1)/n x total bytes.
Prints one JSON line per (op, size) and a correctness line for the 1024-element
configuration.
"""
from __future__ import annotations

import argparse
import json
import threading
import time

import numpy as np


def _run(clients, fn):
    res = [None] * len(clients)
    err = [None] * len(clients)

    def go(i):
        try:
            res[i] = fn(clients[i])
        except BaseException as e:  # noqa: BLE001
            err[i] = e

    ts = [threading.Thread(target=go, args=(i,), daemon=True) for i in range(len(clients))]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    for e in err:
        if e is not None:
            raise e
    return res


def check_config(clients, n=1024):
    """Correctness check of the CPU ring configuration, 1024 f32 per rank: all-reduce and
    reduce-scatter against the float64 elementwise sum, all-gather against the concatenation."""
    W = len(clients)
    data = [np.random.RandomState(r).uniform(-1, 1, n).astype(np.float32) for r in range(W)]
    want = np.sum(np.stack(data).astype(np.float64), axis=0)
    bufs = [d.copy() for d in data]
    _run(clients, lambda c: c.all_reduce_host(bufs[c.rank]))
    ok_ar = all(np.allclose(b, want, atol=1e-5) for b in bufs)
    gath = [np.zeros(n * W, np.float32) for _ in range(W)]
    _run(clients, lambda c: c.all_gather_host(data[c.rank], gath[c.rank]))
    ok_ag = all(np.array_equal(g, np.concatenate(data)) for g in gath)
    rs = [np.zeros(n // W, np.float32) for _ in range(W)]
    _run(clients, lambda c: c.reduce_scatter_host(data[c.rank], rs[c.rank]))
    ok_rs = all(np.allclose(rs[r], want[r * (n // W):(r + 1) * (n // W)], atol=1e-5) for r in range(W))
    return ok_ar and ok_ag and ok_rs


def _values(r, n, dtype):
    x = np.random.RandomState(r).uniform(-1, 1, n).astype(np.float32)
    if dtype == "bf16":  # top 16 bits of the f32 pattern, held as uint16 (the client maps it to BF16)
        return (x.view(np.uint32) >> 16).astype(np.uint16)
    return x


def time_op(clients, op, nbytes, iters, warmup, dtype="f32"):
    W = len(clients)
    es = 2 if dtype == "bf16" else 4
    npt = np.uint16 if dtype == "bf16" else np.float32
    count = max(W, nbytes // es // W * W)
    if op == "all_reduce":
        bufs = [_values(r, count, dtype) for r in range(W)]

        def call(c):
            c.all_reduce_host(bufs[c.rank])
    elif op == "all_gather":
        send = [_values(r, count // W, dtype) for r in range(W)]
        recv = [np.empty(count, npt) for _ in range(W)]

        def call(c):
            c.all_gather_host(send[c.rank], recv[c.rank])
    elif op == "reduce_scatter":
        send = [_values(r, count, dtype) for r in range(W)]
        recv = [np.empty(count // W, npt) for _ in range(W)]

        def call(c):
            c.reduce_scatter_host(send[c.rank], recv[c.rank])
    else:
        raise ValueError(op)

    def body(c):
        for _ in range(warmup):
            call(c)
        c.barrier()
        t0 = time.perf_counter()
        for _ in range(iters):
            call(c)
        return time.perf_counter() - t0

    t = max(_run(clients, body)) / iters
    total = count * es
    factor = 2 * (W - 1) / W if op == "all_reduce" else (W - 1) / W
    return {"op": op, "ranks": W, "dtype": dtype, "bytes": total, "us": round(t * 1e6, 1),
            "algbw_gbs": round(total / t / 1e9, 3), "busbw_gbs": round(factor * total / t / 1e9, 3)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ranks", type=int, default=4)
    ap.add_argument("--min-bytes", type=int, default=4096)
    ap.add_argument("--max-bytes", type=int, default=64 << 20)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--ops", default="all_reduce,all_gather,reduce_scatter")
    ap.add_argument("--dtype", default="f32", choices=["f32", "bf16"])
    ap.add_argument("--out", default=None)
    ap.add_argument("--tls", action="store_true", help="mutually authenticated TLS 1.3 on every mesh link")
    args = ap.parse_args()
    from nexar_b200.client import Config, NexarClient
    clients = NexarClient.bootstrap_local(args.ranks, Config(tls=True) if args.tls else None)
    out = open(args.out, "w") if args.out else None
    try:
        print(json.dumps({"config": "cpu_ring", "ranks": args.ranks, "tls": args.tls,
                          "correct": check_config(clients)}), flush=True)
        size = args.min_bytes
        while size <= args.max_bytes:
            for op in args.ops.split(","):
                iters = args.iters if size <= (4 << 20) else max(3, args.iters // 4)
                rec = time_op(clients, op, size, iters, args.warmup, args.dtype)
                line = json.dumps(rec)
                print(line, flush=True)
                if out:
                    out.write(line + "\n")
            size *= 4
    finally:
        if out:
            out.close()
        for c in clients:
            c.close()


if __name__ == "__main__":
    main()
