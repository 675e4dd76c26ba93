"""DeviceAdapter plumbing (nexar/src/device/adapter.rs, cpu.rs; nexar-rdma/src/cuda_adapter.rs):
every collective and p2p call moves buffers through the client's adapter.

The test adapter keeps its "device" values encoded (stored = value + OFFSET)
and decodes them in stage_for_send / encodes them in receive_to_device. A call
that read or wrote the buffers directly, bypassing the adapter, would be off
by OFFSET, so exact results show that every path stages."""
import ctypes

import numpy as np
import pytest

from helpers_host import run_collective
from nexar_b200 import _native
from nexar_b200.client import CpuAdapter, CudaAdapter, NexarClient
from nexar_b200.core import DataType, ReduceOp

OFFSET = 1000.0


def _view(addr, nbytes):
    return np.ctypeslib.as_array((ctypes.c_double * (nbytes // 8)).from_address(addr))


class EncodedAdapter(_native.host().DeviceAdapter):
    def __init__(self):
        super().__init__()
        self.staged = 0
        self.received = 0

    def name(self):
        return "encoded"

    def stage_for_send(self, ptr, n, out):
        self.staged += n
        _view(out, n)[:] = _view(ptr, n) - OFFSET

    def receive_to_device(self, src, n, ptr):
        self.received += n
        _view(ptr, n)[:] = _view(src, n) + OFFSET

    def reduce_inplace(self, dst, src, count, dt, op):
        d, s = _view(dst, count * 8), _view(src, count * 8)
        d[:] = (d - OFFSET) + (s - OFFSET) + OFFSET


def enc(x):
    return np.ascontiguousarray(x, dtype=np.float64) + OFFSET


def dec(x):
    return x - OFFSET


def vals(rank, n, seed=0):
    return np.random.RandomState(seed * 100 + rank).randint(-50, 50, n).astype(np.float64)


def test_every_collective_stages_through_the_adapter():
    W, n = 3, 12
    ad = EncodedAdapter()
    cs = NexarClient.bootstrap_local(W, adapter=ad)
    assert all(c.adapter() == "encoded" for c in cs)
    F64 = DataType.F64
    try:
        # all-reduce (ring / recursive doubling), rs+ag all-reduce, broadcast, reduce, scans
        bufs = [enc(vals(r, n)) for r in range(W)]
        run_collective(cs, lambda c: c.all_reduce(bufs[c.rank].ctypes.data, n, F64, ReduceOp.Sum))
        want = sum(vals(r, n) for r in range(W))
        for b in bufs:
            np.testing.assert_array_equal(dec(b), want)
        bufs = [enc(vals(r, n, 1)) for r in range(W)]
        run_collective(cs, lambda c: c.all_reduce_rs_ag(bufs[c.rank].ctypes.data, n, F64, ReduceOp.Max))
        for b in bufs:
            np.testing.assert_array_equal(dec(b), np.max([vals(r, n, 1) for r in range(W)], axis=0))
        bufs = [enc(vals(r, n, 2)) for r in range(W)]
        run_collective(cs, lambda c: c.broadcast(bufs[c.rank].ctypes.data, n, F64, 1))
        for b in bufs:
            np.testing.assert_array_equal(dec(b), vals(1, n, 2))
        bufs = [enc(vals(r, n, 3)) for r in range(W)]
        run_collective(cs, lambda c: c.reduce(bufs[c.rank].ctypes.data, n, F64, ReduceOp.Sum, 2))
        np.testing.assert_array_equal(dec(bufs[2]), sum(vals(r, n, 3) for r in range(W)))
        bufs = [enc(vals(r, n, 4)) for r in range(W)]
        run_collective(cs, lambda c: c.exclusive_scan(bufs[c.rank].ctypes.data, n, F64, ReduceOp.Sum))
        np.testing.assert_array_equal(dec(bufs[2]), vals(0, n, 4) + vals(1, n, 4))
        np.testing.assert_array_equal(dec(bufs[0]), np.zeros(n))

        # out-of-place collectives: send staged in, receive written back
        k = 4
        send = [enc(vals(r, k * W, 5)) for r in range(W)]
        recv = [enc(np.zeros(k)) for _ in range(W)]
        run_collective(cs, lambda c: c.reduce_scatter(send[c.rank].ctypes.data, recv[c.rank].ctypes.data, k, F64,
                                                      ReduceOp.Sum))
        total = sum(vals(r, k * W, 5) for r in range(W))
        for r in range(W):
            np.testing.assert_array_equal(dec(recv[r]), total[r * k:(r + 1) * k])
        send = [enc(vals(r, k, 6)) for r in range(W)]
        recv = [enc(np.zeros(k * W)) for _ in range(W)]
        run_collective(cs, lambda c: c.all_gather(send[c.rank].ctypes.data, recv[c.rank].ctypes.data, k, F64))
        for r in range(W):
            np.testing.assert_array_equal(dec(recv[r]), np.concatenate([vals(p, k, 6) for p in range(W)]))
        send = [enc(vals(r, k * W, 7)) for r in range(W)]
        recv = [enc(np.zeros(k * W)) for _ in range(W)]
        run_collective(cs, lambda c: c.all_to_all(send[c.rank].ctypes.data, recv[c.rank].ctypes.data, k, F64))
        for r in range(W):
            np.testing.assert_array_equal(dec(recv[r]), np.concatenate([vals(p, k * W, 7)[r * k:(r + 1) * k]
                                                                        for p in range(W)]))
        send = [enc(vals(r, k, 8)) for r in range(W)]
        recv = [enc(np.zeros(k * W)) for _ in range(W)]
        run_collective(cs, lambda c: c.gather(send[c.rank].ctypes.data, recv[c.rank].ctypes.data, k, F64, 1))
        np.testing.assert_array_equal(dec(recv[1]), np.concatenate([vals(p, k, 8) for p in range(W)]))
        np.testing.assert_array_equal(dec(recv[0]), np.zeros(k * W))  # non-root untouched
        send = [enc(vals(r, k * W, 9)) for r in range(W)]
        recv = [enc(np.zeros(k)) for _ in range(W)]
        run_collective(cs, lambda c: c.scatter(send[c.rank].ctypes.data, recv[c.rank].ctypes.data, k, F64, 2))
        for r in range(W):
            np.testing.assert_array_equal(dec(recv[r]), vals(2, k * W, 9)[r * k:(r + 1) * k])

        # p2p and iov
        a, b = enc(vals(0, n, 10)), enc(np.zeros(n))
        run_collective(cs[:2], lambda c: c.send(a.ctypes.data, a.nbytes, 1, 7) if c.rank == 0
                       else c.recv(b.ctypes.data, b.nbytes, 0, 7))
        np.testing.assert_array_equal(dec(b), vals(0, n, 10))
        x, y = enc(vals(0, 3, 11)), enc(vals(0, 5, 12))
        u, v = enc(np.zeros(3)), enc(np.zeros(5))
        run_collective(cs[:2], lambda c: c.send_iov([(x.ctypes.data, x.nbytes), (y.ctypes.data, y.nbytes)], 1, 9)
                       if c.rank == 0 else c.recv_iov([(u.ctypes.data, u.nbytes), (v.ctypes.data, v.nbytes)], 0, 9))
        np.testing.assert_array_equal(dec(u), vals(0, 3, 11))
        np.testing.assert_array_equal(dec(v), vals(0, 5, 12))

        # bucketed all-reduce gathers every region through the adapter
        p1 = [enc(vals(r, 5, 13)) for r in range(W)]
        p2 = [enc(vals(r, 2, 14)) for r in range(W)]
        run_collective(cs, lambda c: c.all_reduce_bucketed([(p1[c.rank].ctypes.data, 5), (p2[c.rank].ctypes.data, 2)],
                                                           F64, ReduceOp.Sum))
        for r in range(W):
            np.testing.assert_array_equal(dec(p1[r]), sum(vals(q, 5, 13) for q in range(W)))
            np.testing.assert_array_equal(dec(p2[r]), sum(vals(q, 2, 14) for q in range(W)))
        assert ad.staged > 0 and ad.received > 0
    finally:
        for c in cs:
            c.close()


def test_split_children_inherit_the_adapter():
    ad = EncodedAdapter()
    cs = NexarClient.bootstrap_local(4, adapter=ad)
    try:
        subs = run_collective(cs, lambda c: c.split(c.rank % 2, c.rank))
        assert all(s.adapter() == "encoded" for s in subs)
        bufs = [enc(np.full(4, float(r))) for r in range(4)]
        run_collective(list(range(4)), lambda i: subs[i].all_reduce(bufs[i].ctypes.data, 4, DataType.F64,
                                                                    ReduceOp.Sum))
        for i in range(4):
            np.testing.assert_array_equal(dec(bufs[i]), np.full(4, 2.0 if i % 2 == 0 else 4.0))
    finally:
        for c in cs:
            c.close()


def test_adapter_objects_and_direct_calls():
    cpu, cuda = CpuAdapter(), CudaAdapter()
    assert cpu.name() == "cpu" and cpu.host_addressable() and cpu.supports_host_offload()
    assert cuda.name() == "cuda" and not cuda.host_addressable() and not cuda.supports_device_collectives()
    a = np.arange(6, dtype=np.float32)
    b = np.full(6, 2.0, np.float32)
    out = np.zeros(6, np.float32)
    for ad in (cpu, cuda):  # host memory on both (the CUDA adapter copies host-to-host)
        out[:] = 0
        ad.stage_for_send(a.ctypes.data, a.nbytes, out.ctypes.data)
        np.testing.assert_array_equal(out, a)
        ad.reduce_inplace(out.ctypes.data, b.ctypes.data, 6, int(DataType.F32), int(ReduceOp.Sum))
        np.testing.assert_array_equal(out, a + 2)
        ad.receive_to_device(b.ctypes.data, b.nbytes, out.ctypes.data)
        np.testing.assert_array_equal(out, b)
    with pytest.raises(TypeError):
        NexarClient.bootstrap_local(2, adapter=object())


def test_cuda_adapter_collectives_on_host_buffers():
    """With the CUDA adapter, host buffers still reduce correctly (the copies
    fall back to memcpy when neither side is GPU memory)."""
    cs = NexarClient.bootstrap_local(2, adapter="cuda")
    try:
        assert [c.adapter() for c in cs] == ["cuda", "cuda"]
        bufs = [np.full(8, float(r + 1), np.float32) for r in range(2)]
        run_collective(cs, lambda c: c.all_reduce_host(bufs[c.rank]))
        assert all((b == 3).all() for b in bufs)
        with pytest.raises(RuntimeError):
            cs[0].set_adapter("cpu")
            cs[0].all_reduce_device(np.zeros(2, np.float32))
    finally:
        for c in cs:
            c.close()
