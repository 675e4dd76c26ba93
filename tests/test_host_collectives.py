"""Host collectives over the TCP mesh (mirrors nexar/tests/collective/*.rs).

Data is rank- and index-dependent so chunk placement is pinned (the
reference's tests use uniform data; here reduce_scatter must give rank r
chunk r).
"""
import numpy as np
import pytest

from helpers_host import bootstrap, data, run_collective
from nexar_b200.core import DataType, ReduceOp

NP_OPS = {"sum": np.add, "prod": np.multiply, "min": np.minimum, "max": np.maximum}


def oracle(xs, op):
    acc = xs[0].astype(np.float64 if np.issubdtype(xs[0].dtype, np.floating) else np.int64)
    for x in xs[1:]:
        acc = NP_OPS[op](acc, x)
    return acc


@pytest.fixture(scope="module")
def c4():
    return bootstrap(4)


@pytest.fixture(scope="module")
def c3():
    return bootstrap(3)


@pytest.fixture(scope="module")
def c2():
    return bootstrap(2)


@pytest.mark.parametrize("n", [2, 3, 4])
def test_allreduce_sum_f32(n, c2, c3, c4):
    cs = {2: c2, 3: c3, 4: c4}[n]
    xs = [data(r, 1024) for r in range(n)]
    bufs = [x.copy() for x in xs]
    run_collective(cs, lambda c: c.all_reduce_host(bufs[c.rank]))
    for b in bufs:
        np.testing.assert_allclose(b, oracle(xs, "sum"), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("op", ["sum", "min", "max", "prod"])
def test_allreduce_ops_i32(op, c4):
    xs = [data(r, 257, np.int32) for r in range(4)]
    bufs = [x.copy() for x in xs]
    run_collective(c4, lambda c: c.all_reduce_host(bufs[c.rank], op))
    want = oracle(xs, op).astype(np.int32)
    for b in bufs:
        np.testing.assert_array_equal(b, want)


def test_allreduce_uneven_count(c3):
    xs = [data(r, 7) for r in range(3)]
    bufs = [x.copy() for x in xs]
    run_collective(c3, lambda c: c.all_reduce_host(bufs[c.rank]))
    for b in bufs:
        np.testing.assert_allclose(b, oracle(xs, "sum"), rtol=1e-5, atol=1e-5)


def test_allreduce_count_smaller_than_world(c4):
    xs = [data(r, 2) for r in range(4)]
    bufs = [x.copy() for x in xs]
    run_collective(c4, lambda c: c.all_reduce_host(bufs[c.rank]))
    for b in bufs:
        np.testing.assert_allclose(b, oracle(xs, "sum"), rtol=1e-5, atol=1e-5)


def test_allreduce_f64_and_bf16(c2):
    xs = [data(r, 100, np.float64) for r in range(2)]
    bufs = [x.copy() for x in xs]
    run_collective(c2, lambda c: c.all_reduce_host(bufs[c.rank]))
    np.testing.assert_allclose(bufs[0], oracle(xs, "sum"))
    import torch
    ts = [torch.tensor(data(r, 100)).to(torch.bfloat16) for r in range(2)]
    want = (ts[0].float() + ts[1].float()).to(torch.bfloat16)
    run_collective(c2, lambda c: c.all_reduce_host(ts[c.rank]))
    for t in ts:
        assert torch.equal(t, want)  # RNE rounding of the f32 sum


def test_pipelined_and_halving_doubling_paths():
    # ring_max_world=0 forces halving-doubling at 5 ranks; a tiny
    # large_msg_bytes forces the pipelined ring (tests/sparse.rs:292-316).
    cs = bootstrap(5, ring_max_world=0, small_msg_bytes=0)
    xs = [data(r, 1000) for r in range(5)]
    bufs = [x.copy() for x in xs]
    run_collective(cs, lambda c: c.all_reduce_host(bufs[c.rank]))
    for b in bufs:
        np.testing.assert_allclose(b, oracle(xs, "sum"), rtol=1e-5, atol=1e-5)
    cs = bootstrap(3, large_msg_bytes=1024, pipeline_segment_bytes=256)
    xs = [data(r, 5000) for r in range(3)]
    bufs = [x.copy() for x in xs]
    run_collective(cs, lambda c: c.all_reduce_host(bufs[c.rank]))
    for b in bufs:
        np.testing.assert_allclose(b, oracle(xs, "sum"), rtol=1e-5, atol=1e-5)


def test_halving_doubling_pow2():
    cs = bootstrap(8, ring_max_world=0, small_msg_bytes=0)
    xs = [data(r, 333) for r in range(8)]
    bufs = [x.copy() for x in xs]
    run_collective(cs, lambda c: c.all_reduce_host(bufs[c.rank]))
    for b in bufs:
        np.testing.assert_allclose(b, oracle(xs, "sum"), rtol=1e-5, atol=1e-5)


def test_reduce_to_root(c4):
    for root in (0, 2):
        xs = [data(r, 100) for r in range(4)]
        bufs = [x.copy() for x in xs]
        run_collective(c4, lambda c: c.reduce_host(bufs[c.rank], "sum", root))
        np.testing.assert_allclose(bufs[root], oracle(xs, "sum"), rtol=1e-5, atol=1e-5)


def test_reduce_scatter_rank_r_gets_chunk_r(c4):
    count = 9
    xs = [data(r, count * 4) for r in range(4)]
    outs = [np.zeros(count, np.float32) for _ in range(4)]
    run_collective(c4, lambda c: c.reduce_scatter_host(xs[c.rank], outs[c.rank]))
    full = oracle(xs, "sum")
    for r in range(4):
        np.testing.assert_allclose(outs[r], full[r * count:(r + 1) * count], rtol=1e-5, atol=1e-5)


def test_allgather(c3):
    xs = [data(r, 11) for r in range(3)]
    outs = [np.zeros(33, np.float32) for _ in range(3)]
    run_collective(c3, lambda c: c.all_gather_host(xs[c.rank], outs[c.rank]))
    for o in outs:
        np.testing.assert_array_equal(o, np.concatenate(xs))


def test_alltoall(c4):
    count = 5
    xs = [data(r, count * 4) for r in range(4)]
    outs = [np.zeros(count * 4, np.float32) for _ in range(4)]
    run_collective(c4, lambda c: c.all_to_all_host(xs[c.rank], outs[c.rank]))
    for r in range(4):
        want = np.concatenate([xs[p][r * count:(r + 1) * count] for p in range(4)])
        np.testing.assert_array_equal(outs[r], want)


@pytest.mark.parametrize("root", [0, 2])
def test_gather_scatter_roots(root, c3):
    xs = [data(r, 6) for r in range(3)]
    out = np.zeros(18, np.float32)
    run_collective(c3, lambda c: c.gather_host(xs[c.rank], out if c.rank == root else None, root))
    np.testing.assert_array_equal(out, np.concatenate(xs))
    src = data(9, 18)
    outs = [np.zeros(6, np.float32) for _ in range(3)]
    run_collective(c3, lambda c: c.scatter_host(src if c.rank == root else None, outs[c.rank], root))
    for r in range(3):
        np.testing.assert_array_equal(outs[r], src[r * 6:(r + 1) * 6])


@pytest.mark.parametrize("n,root", [(2, 0), (3, 1), (5, 0), (5, 3), (6, 5)])
def test_broadcast(n, root):
    cs = bootstrap(n)
    src = data(77, 1000)
    bufs = [src.copy() if r == root else np.zeros(1000, np.float32) for r in range(n)]
    run_collective(cs, lambda c: c.broadcast_host(bufs[c.rank], root))
    for b in bufs:
        np.testing.assert_array_equal(b, src)


@pytest.mark.parametrize("n", [4, 5])
def test_barrier_and_repeated(n):
    cs = bootstrap(n)
    for _ in range(5):
        run_collective(cs, lambda c: c.barrier())


@pytest.mark.parametrize("op", ["sum", "max", "prod"])
def test_scan_and_exclusive_scan(op, c4):
    xs = [data(r, 13) for r in range(4)]
    bufs = [x.copy() for x in xs]
    run_collective(c4, lambda c: c.scan_host(bufs[c.rank], op))
    for r in range(4):
        np.testing.assert_allclose(bufs[r], oracle(xs[:r + 1], op), rtol=1e-5, atol=1e-5)
    bufs = [x.copy() for x in xs]
    run_collective(c4, lambda c: c.exclusive_scan_host(bufs[c.rank], op))
    ident = {"sum": 0.0, "prod": 1.0, "max": np.finfo(np.float32).min}[op]
    np.testing.assert_array_equal(bufs[0], np.full(13, ident, np.float32))
    for r in range(1, 4):
        np.testing.assert_allclose(bufs[r], oracle(xs[:r], op), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("count", [12, 13])
def test_rs_ag_allreduce(count, c3):
    xs = [data(r, count) for r in range(3)]
    bufs = [x.copy() for x in xs]
    run_collective(c3, lambda c: c.all_reduce_rs_ag(bufs[c.rank].ctypes.data, count, DataType.F32, "sum"))
    for b in bufs:
        np.testing.assert_allclose(b, oracle(xs, "sum"), rtol=1e-5, atol=1e-5)


def test_bucketed_allreduce(c2):
    a = [data(r, 10) for r in range(2)]
    b = [data(r + 5, 3) for r in range(2)]
    bufs = [(a[r].copy(), b[r].copy()) for r in range(2)]
    run_collective(c2, lambda c: c.all_reduce_bucketed_host(list(bufs[c.rank])))
    for r in range(2):
        np.testing.assert_allclose(bufs[r][0], a[0] + a[1], rtol=1e-6)
        np.testing.assert_allclose(bufs[r][1], b[0] + b[1], rtol=1e-6)


def test_iov_send_recv(c2):
    a, b = np.arange(5, dtype=np.float32), np.arange(7, dtype=np.int64)
    ra, rb = np.zeros(5, np.float32), np.zeros(7, np.int64)

    def f(c):
        if c.rank == 0:
            c.send_iov([(a.ctypes.data, a.nbytes), (b.ctypes.data, b.nbytes)], 1, 3)
        else:
            c.recv_iov([(ra.ctypes.data, ra.nbytes), (rb.ctypes.data, rb.nbytes)], 0, 3)
    run_collective(c2, f)
    np.testing.assert_array_equal(ra, a)
    np.testing.assert_array_equal(rb, b)


def test_send_recv_tag_matching(c2):
    out = {}

    def f(c):
        if c.rank == 0:
            for tag in (1, 2, 3):
                x = np.full(4, tag, np.int32)
                c.send(x.ctypes.data, x.nbytes, 1, tag)
        else:
            for tag in (3, 1, 2):  # out of order: matched by tag
                y = np.zeros(4, np.int32)
                c.recv(y.ctypes.data, y.nbytes, 0, tag)
                out[tag] = y.copy()
    run_collective(c2, f)
    for tag in (1, 2, 3):
        assert (out[tag] == tag).all()


def test_tagged_bytes_isolation_and_concurrency(c2):
    def f(c):
        if c.rank == 0:
            for t in range(20):
                c.send_bytes_tagged(1, 100 + t, bytes([t]) * (t + 1))
            return None
        got = [c.recv_bytes_tagged(0, 100 + t) for t in reversed(range(20))]
        return got
    res = run_collective(c2, f)
    assert res[1] == [bytes([t]) * (t + 1) for t in reversed(range(20))]


def test_raw_bytes(c2):
    def f(c):
        if c.rank == 0:
            c.send_bytes(1, b"hello")
        else:
            return c.recv_bytes(0)
    assert run_collective(c2, f)[1] == b"hello"


def test_nonblocking_concurrent_allreduces(c4):
    xs = [data(r, 100) for r in range(4)]
    ys = [data(r + 10, 50) for r in range(4)]
    bx = [x.copy() for x in xs]
    by = [y.copy() for y in ys]

    def f(c):
        from nexar_b200.client import CollectiveGroup
        g = CollectiveGroup()
        g.push(c.all_reduce_nb(bx[c.rank].ctypes.data, 100, DataType.F32))
        g.push(c.all_reduce_nb(by[c.rank].ctypes.data, 50, DataType.F32))
        g.wait_all()
    run_collective(c4, f)
    for r in range(4):
        np.testing.assert_allclose(bx[r], oracle(xs, "sum"), rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(by[r], oracle(ys, "sum"), rtol=1e-5, atol=1e-5)


def test_nonblocking_variants(c3):
    xs = [data(r, 6) for r in range(3)]
    outs = [np.zeros(18, np.float32) for _ in range(3)]

    def f(c):
        h = c.all_gather_nb(xs[c.rank].ctypes.data, outs[c.rank].ctypes.data, 6, DataType.F32)
        h.wait()
        assert h.is_finished()
        c.barrier_nb().wait()
    run_collective(c3, f)
    for o in outs:
        np.testing.assert_array_equal(o, np.concatenate(xs))


def test_split(c4):
    subs = run_collective(c4, lambda c: c.split(c.rank % 2, c.rank))
    for r, s in enumerate(subs):
        assert s.world_size == 2 and s.rank == r // 2
    xs = [np.full(8, float(r + 1), np.float32) for r in range(4)]
    run_collective(subs, lambda s: s.all_reduce_host(xs[[i for i in range(4) if subs[i] is s][0]]))
    np.testing.assert_array_equal(xs[0], np.full(8, 1 + 3, np.float32))
    np.testing.assert_array_equal(xs[1], np.full(8, 2 + 4, np.float32))
    # parent still works after the split
    bufs = [np.ones(4, np.float32) for _ in range(4)]
    run_collective(c4, lambda c: c.all_reduce_host(bufs[c.rank]))
    assert (bufs[0] == 4).all()


def test_split_key_reorders(c3):
    subs = run_collective(c3, lambda c: c.split(0, 10 - c.rank))
    assert [s.rank for s in subs] == [2, 1, 0]


def test_rpc(c2):
    c2[1].register_rpc(7, lambda b: b[::-1] + b"!")

    def f(c):
        if c.rank == 0:
            return c.rpc(1, 7, b"abc", 10.0)
        c.serve_rpc_once(0, 10.0)
    assert run_collective(c2, f)[0] == b"cba!"


def test_rpc_unregistered_and_server(c2):
    from nexar_b200.core import RpcNotRegistered
    c2[1].register_rpc(8, lambda b: b * 2)
    c2[1].start_rpc_server()
    try:
        assert c2[0].rpc(1, 8, b"xy", 10.0) == b"xyxy"
        with pytest.raises(RpcNotRegistered):
            c2[0].rpc(1, 99, b"", 10.0)
    finally:
        c2[1].stop_rpc_server()


def test_compressed_allreduce_lossless_and_topk(c2):
    from nexar_b200.client import NoCompression, TopKCompressor
    xs = [data(r, 64) for r in range(2)]
    bufs = [x.copy() for x in xs]
    res = [np.zeros(64, np.float32) for _ in range(2)]
    run_collective(c2, lambda c: c.all_reduce_compressed_host(bufs[c.rank], TopKCompressor(1.0), res[c.rank]))
    for b in bufs:
        np.testing.assert_allclose(b, xs[0] + xs[1], rtol=1e-6)
    # ratio 0.25: each rank contributes its 16 largest |x| entries; the rest stays in the residual
    bufs = [x.copy() for x in xs]
    res = [np.zeros(64, np.float32) for _ in range(2)]
    run_collective(c2, lambda c: c.all_reduce_compressed_host(bufs[c.rank], TopKCompressor(0.25), res[c.rank]))
    want = np.zeros(64, np.float64)
    for r in range(2):
        keep = np.argsort(-np.abs(xs[r]), kind="stable")[:16]
        want[keep] += xs[r][keep]
        kept = np.zeros(64, bool)
        kept[keep] = True
        np.testing.assert_allclose(res[r][~kept], xs[r][~kept])
        assert (res[r][kept] == 0).all()
    for b in bufs:
        np.testing.assert_allclose(b, want, rtol=1e-6)
    bufs = [x.copy() for x in xs]
    res = [np.zeros(64, np.float32) for _ in range(2)]
    run_collective(c2, lambda c: c.all_reduce_compressed_host(bufs[c.rank], NoCompression(), res[c.rank]))
    np.testing.assert_allclose(bufs[0], xs[0] + xs[1], rtol=1e-6)


def test_all_gather_bytes(c3):
    res = run_collective(c3, lambda c: c.all_gather_bytes(b"x" * (c.rank + 1)))
    for r in res:
        assert r == [b"x", b"xx", b"xxx"]


ALGOS = {
    "recursive_doubling": dict(small_msg_bytes=1 << 30),
    "ring": dict(small_msg_bytes=0),
    "halving_doubling": dict(small_msg_bytes=0, ring_max_world=0),
    "pipelined": dict(small_msg_bytes=0, large_msg_bytes=1024, pipeline_segment_bytes=256),
}


@pytest.mark.parametrize("world", [3, 4, 5])
@pytest.mark.parametrize("algo", sorted(ALGOS))
def test_allreduce_every_algorithm(world, algo):
    """Each all-reduce algorithm forced through the config: close to the oracle,
    bitwise identical on every rank, for an uneven count."""
    cs = bootstrap(world, **ALGOS[algo])
    try:
        xs = [data(r, 1003, seed=7) for r in range(world)]
        bufs = [x.copy() for x in xs]
        run_collective(cs, lambda c: c.all_reduce_host(bufs[c.rank]))
        for b in bufs:
            np.testing.assert_allclose(b, oracle(xs, "sum"), rtol=1e-5, atol=1e-5)
            assert np.array_equal(b, bufs[0])
        for op in ("max", "min", "prod"):
            ys = [data(r, 37, dtype=np.int32, seed=3) % 5 + 1 for r in range(world)]
            bs = [y.copy() for y in ys]
            run_collective(cs, lambda c: c.all_reduce_host(bs[c.rank], op))
            for b in bs:
                assert np.array_equal(b, oracle(ys, op).astype(np.int32)), (algo, op)
    finally:
        for c in cs:
            c.close()


RS_AG_PATHS = {
    "pipelined": dict(pipeline_segment_bytes=256),   # chunks of 16 segments
    "ring": dict(small_msg_bytes=0),                 # one message per ring step
    "direct": dict(),                                # small: one hop over the full mesh
}


@pytest.mark.parametrize("world", [3, 4])
@pytest.mark.parametrize("path", sorted(RS_AG_PATHS))
def test_reduce_scatter_and_all_gather_paths(world, path):
    """Pipelined rings (segments forwarded as soon as they are reduced /
    stored), plain rings and the direct small-message exchange."""
    cs = bootstrap(world, **RS_AG_PATHS[path])
    try:
        count = 1000  # 16 segments of 64 f32 per chunk
        xs = [data(r, count * world, seed=11) for r in range(world)]
        outs = [np.zeros(count, np.float32) for _ in range(world)]
        run_collective(cs, lambda c: c.reduce_scatter_host(xs[c.rank], outs[c.rank]))
        full = oracle(xs, "sum")
        for r in range(world):
            np.testing.assert_allclose(outs[r], full[r * count:(r + 1) * count], rtol=1e-5, atol=1e-5)
        gs = [np.zeros(count * world, np.float32) for _ in range(world)]
        run_collective(cs, lambda c: c.all_gather_host(outs[c.rank], gs[c.rank]))
        for g in gs:
            assert np.array_equal(g, np.concatenate(outs))
    finally:
        for c in cs:
            c.close()
