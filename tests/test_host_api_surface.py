"""The reference's public client API names on the Python client (peer, raw messages,
rpc_dispatcher, non-blocking bucketed / compressed all-reduce, rs_ag host variant,
bootstrap_elastic)."""
import threading

import numpy as np
import pytest

from helpers_host import run_collective


def test_peer_messages_and_rpc_dispatcher():
    from nexar_b200.client import NexarClient
    from nexar_b200.core import NexarError
    cs = NexarClient.bootstrap_local(3)
    p = cs[0].peer(1)
    assert p["rank"] == 1 and p["alive"] and not p["encrypted"]
    with pytest.raises(NexarError):
        cs[0].peer(7)
    cs[0].send_message_to(2, 42, b"hello")
    assert cs[2].recv_message_from(0, 42, 5.0) == b"hello"
    d = cs[1].rpc_dispatcher()
    d.register(5, lambda b: b[::-1])
    t = threading.Thread(target=d.serve_once, args=(0, 5.0))
    t.start()
    assert cs[0].rpc(1, 5, b"abc", 5.0) == b"cba"
    t.join()


def test_p2p_send_is_a_data_message_on_the_root_communicator():
    """send / recv on the root communicator carry Data messages (as the
    reference's client.send), so they pair with send_message_to /
    recv_message_from; a split communicator's p2p traffic stays apart from the
    root's even under the same tag."""
    from nexar_b200.client import NexarClient
    cs = NexarClient.bootstrap_local(2)
    # send -> recv_message_from
    x = np.arange(64, dtype=np.uint8)
    cs[0].send(x.ctypes.data, x.nbytes, 1, 77)
    assert cs[1].recv_message_from(0, 77, 5.0) == x.tobytes()
    # send_message_to -> recv (large enough to take several socket reads)
    payload = bytes(np.random.default_rng(0).integers(0, 256, 300_000, dtype=np.uint8))
    cs[1].send_message_to(0, 78, payload)
    out = np.empty(len(payload), np.uint8)
    cs[0].recv(out.ctypes.data, out.nbytes, 1, 78)
    assert out.tobytes() == payload
    # messages with other tags wait their turn; the oldest with the tag is taken
    a, b = np.full(8, 1, np.uint8), np.full(8, 2, np.uint8)
    cs[0].send(a.ctypes.data, 8, 1, 5)
    cs[0].send(b.ctypes.data, 8, 1, 6)
    got6, got5 = np.empty(8, np.uint8), np.empty(8, np.uint8)
    cs[1].recv(got6.ctypes.data, 8, 0, 6)
    cs[1].recv(got5.ctypes.data, 8, 0, 5)
    assert (got6 == 2).all() and (got5 == 1).all()
    # a split communicator's message under the same tag is not the root's
    subs = run_collective(cs, lambda c: c.split(0, c.rank))
    s_msg, r_msg = np.full(4, 9, np.uint8), np.full(4, 3, np.uint8)
    subs[0].send(s_msg.ctypes.data, 4, 1, 11)
    cs[0].send(r_msg.ctypes.data, 4, 1, 11)
    root_got, sub_got = np.empty(4, np.uint8), np.empty(4, np.uint8)
    cs[1].recv(root_got.ctypes.data, 4, 0, 11)
    subs[1].recv(sub_got.ctypes.data, 4, 0, 11)
    assert (root_got == 3).all() and (sub_got == 9).all()


def test_nonblocking_bucketed_and_compressed_and_rs_ag_host():
    from nexar_b200.client import NexarClient
    from nexar_b200.core import DataType
    from nexar_b200 import _native
    cs = NexarClient.bootstrap_local(4)
    a = [np.full(100, float(c.rank + 1), np.float32) for c in cs]
    b = [np.full(37, float(2 * c.rank), np.float32) for c in cs]
    hs = {}

    def start(c):
        hs[c.rank] = c.all_reduce_bucketed_nb([(a[c.rank].ctypes.data, 100), (b[c.rank].ctypes.data, 37)],
                                              DataType.F32)
        hs[c.rank].wait()
    run_collective(cs, start)
    assert all((x == 10).all() for x in a) and all((x == 12).all() for x in b)
    g = [np.random.default_rng(c.rank).standard_normal(1000).astype(np.float32) for c in cs]
    res = [np.zeros(1000, np.float32) for _ in cs]
    comp = _native.host().TopKCompressor(0.1)

    def cmp(c):
        c.all_reduce_compressed_nb(g[c.rank].ctypes.data, 1000, DataType.F32, "sum", comp,
                                   res[c.rank].ctypes.data).wait()
    run_collective(cs, cmp)
    assert all(np.allclose(g[0], x) for x in g)  # every rank holds the same (sparse) sum
    v = [np.full(64, float(c.rank), np.float32) for c in cs]
    run_collective(cs, lambda c: c.all_reduce_rs_ag_host(v[c.rank]))
    assert all((x == 6).all() for x in v)


def test_bootstrap_elastic_grows():
    from nexar_b200.client import Config, NexarClient
    from nexar_b200 import _native
    H = _native.host()
    eb = NexarClient.bootstrap_elastic(2, max_world=4, config=Config(heartbeat_interval_s=0.1))
    joined = {}
    jt = threading.Thread(target=lambda: joined.setdefault(
        "c", H.ElasticManager.join(eb.seed_addr, None, Config(heartbeat_interval_s=0.1), 20.0)))
    jt.start()
    import time
    time.sleep(0.5)
    assert run_collective(eb.managers, lambda m: m.elastic_checkpoint()) == [True, True]
    jt.join(20)
    grown = [NexarClient(m.client()) for m in eb.managers] + [NexarClient(joined["c"])]
    assert sorted(c.world_size for c in grown) == [3, 3, 3]
    eb.seed.close()


def test_worker_node_connect_then_from_worker():
    """Seed / worker bootstrap in two steps (nexar/src/cluster/worker.rs:34,
    nexar/src/client/bootstrap.rs): WorkerNode.connect, then the mesh."""
    from nexar_b200.client import Config, NexarClient, SeedNode, WorkerNode
    seed = SeedNode(local=True)
    infos = [None] * 3
    ts = [threading.Thread(target=lambda i=i: infos.__setitem__(i, WorkerNode.connect(seed.local_addr())))
          for i in range(3)]
    [t.start() for t in ts]
    seed.form_cluster(3)
    [t.join(30) for t in ts]
    assert sorted(i.rank for i in infos) == [0, 1, 2]
    assert all(i.world_size == 3 and len(i.peers) == 3 and not i.consumed for i in infos)
    clients = [None] * 3
    ts = [threading.Thread(target=lambda k=k: clients.__setitem__(k, NexarClient.from_worker(infos[k], Config())))
          for k in range(3)]
    [t.start() for t in ts]
    [t.join(30) for t in ts]
    assert all(i.consumed for i in infos)
    with pytest.raises(Exception):
        NexarClient.from_worker(infos[0], Config())
    bufs = {c.rank: np.full(5, float(c.rank), np.float32) for c in clients}
    run_collective(clients, lambda c: c.all_reduce_host(bufs[c.rank]))
    assert all((b == 3).all() for b in bufs.values())
    for c in clients:
        c.close()
    seed.close()


def test_crate_root_exports_and_elastic_config():
    import nexar_b200 as nx
    for name in list(nx._EXPORTS) + ["TopologyStrategy", "Compressor", "RecoveryEvent", "ElasticEvent"]:
        assert getattr(nx, name) is not None, name
    assert nx.IoVec(16, 4) == (16, 4) and nx.Rank is int
    with pytest.raises(AttributeError):
        nx.NoSuchThing  # noqa: B018
    ec = nx.ElasticConfig(min_world_size=2, max_world_size=3, checkpoint_timeout_s=5.0)
    eb = nx.NexarClient.bootstrap_elastic(2, elastic=ec, adapter="cpu")
    assert [c.world_size for c in eb.clients] == [2, 2]
    assert run_collective(eb.managers, lambda m: m.elastic_checkpoint()) == [False, False]
    eb.seed.close()


def test_single_rank_bootstrap_and_collectives():
    """nexar/src/client/bootstrap.rs test_bootstrap_single_node, sync_client.rs test_sync_client_single_node."""
    from nexar_b200.client import NexarClient
    (c,) = NexarClient.bootstrap_local(1)
    a = np.arange(5, dtype=np.float32)
    c.all_reduce_host(a)
    assert (a == np.arange(5)).all()
    out = np.zeros(5, np.float32)
    c.all_gather_host(a, out)
    assert (out == a).all()
    c.barrier()
    assert c.split(0, 0).world_size == 1
    c.close()


def test_rpc_handler_overwrite():
    """nexar/src/rpc/registry.rs test_overwrite_handler: the last registration wins."""
    from nexar_b200.client import NexarClient
    cs = NexarClient.bootstrap_local(2)
    d = cs[1].rpc_dispatcher()
    d.register(3, lambda b: b"first")
    d.register(3, lambda b: b"second")
    t = threading.Thread(target=d.serve_once, args=(0, 5.0))
    t.start()
    assert cs[0].rpc(1, 3, b"", 5.0) == b"second"
    t.join()
    for c in cs:
        c.close()


def test_global_ptr_identity():
    """nexar/src/memory/global_ptr.rs: construction, is_local, display, eq / hash."""
    from nexar_b200.device.comm import GlobalPtr

    class FakeComm:
        rank = 1
    comm = FakeComm()
    a, b, c = GlobalPtr(comm, 1, 256, 64), GlobalPtr(comm, 1, 256, 64), GlobalPtr(comm, 2, 256, 64)
    assert a == b and hash(a) == hash(b) and a != c and len({a, b, c}) == 2
    assert a.is_local() and not c.is_local() and c.is_local(2)
    assert "rank 1" in str(a) and "64 bytes" in str(a)


def test_receive_buffers_come_from_the_client_pool():
    """Large receives are served by the client's buffer pool and reuse its
    blocks (nexar's routers read into pooled buffers; new_with_pool)."""
    from nexar_b200.client import NexarClient
    from nexar_b200.memory import BufferPool, PoolBuilder, TierConfig
    pool = PoolBuilder().small(TierConfig(8, 64 << 10)).large(TierConfig(4, 8 << 20)).build()
    cs = NexarClient.bootstrap_local(2, pool=pool)
    assert cs[0].pool is pool and cs[1].pool is pool
    n = 1 << 20  # large tier
    x = np.arange(n, dtype=np.uint8)
    y = np.empty(n, np.uint8)
    for _ in range(6):
        cs[0].send(x.ctypes.data, n, 1, 9)
        cs[1].recv(y.ctypes.data, n, 0, 9)
        assert (y == x).all()
    large = 1
    assert pool.blocks_fresh(large) >= 1
    assert pool.blocks_reused(large) >= 4  # later receives reuse the freed block
    # collectives' receives go through the same pool
    a = [np.full(300_000, float(c.rank + 1), np.float32) for c in cs]
    run_collective(cs, lambda c: c.all_reduce(a[c.rank].ctypes.data, a[c.rank].size, 0))
    assert all((v == 3.0).all() for v in a)
    default = NexarClient.bootstrap_local(2)
    assert default[0].pool is not default[1].pool  # one Training-profile pool per rank
    BufferPool.with_profile(0)
