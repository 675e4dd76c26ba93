"""Sparse overlays, fault injection, recovery and elastic membership on CPU
ranks (mirrors nexar/tests/{sparse,fault_injection,recovery,elastic}.rs).

Failures are injected on the host only: a rank closes its connections
(`close()`), never joins, or raises.
"""
import multiprocessing as mp
import os
import threading
import time

import numpy as np
import pytest

from helpers_host import bootstrap, data, run_collective
from nexar_b200.client import Config, NexarClient
from nexar_b200.core import CollectiveFailed, NexarError, DataType


# ------------------------------------------------------------ sparse overlays
@pytest.mark.parametrize("topo", ["k_regular:6", "hypercube"])
def test_sparse_16_ranks_relay(topo):
    cs = bootstrap(16, topology=topo)
    assert all(c.is_sparse() for c in cs)
    assert not cs[0].has_direct_peer(5) and not cs[0].has_direct_peer(9)
    # relayed point-to-point
    def f(c):
        if c.rank == 0:
            c.send_bytes_tagged(9, 5, b"via relay")
        if c.rank == 9:
            return c.recv_bytes_tagged(0, 5, 10.0)
    assert run_collective(cs, f)[9] == b"via relay"
    # collectives over the overlay
    xs = [data(r, 100) for r in range(16)]
    bufs = [x.copy() for x in xs]
    run_collective(cs, lambda c: c.all_reduce_host(bufs[c.rank]))
    want = np.sum([x.astype(np.float64) for x in xs], axis=0)
    for b in bufs:
        np.testing.assert_allclose(b, want, rtol=1e-4, atol=1e-4)
    src = data(42, 64)
    bb = [src.copy() if r == 3 else np.zeros(64, np.float32) for r in range(16)]
    run_collective(cs, lambda c: c.broadcast_host(bb[c.rank], 3))
    for b in bb:
        np.testing.assert_array_equal(b, src)
    run_collective(cs, lambda c: c.barrier())
    count = 4
    xs = [data(r, count * 16) for r in range(16)]
    outs = [np.zeros(count, np.float32) for _ in range(16)]
    run_collective(cs, lambda c: c.reduce_scatter_host(xs[c.rank], outs[c.rank]))
    full = np.sum([x.astype(np.float64) for x in xs], axis=0)
    for r in range(16):
        np.testing.assert_allclose(outs[r], full[r * count:(r + 1) * count], rtol=1e-4, atol=1e-4)


def test_quic_only_ring_7_ranks():
    cs = bootstrap(7, enable_tcp_bulk_sidecar=False, ring_max_world=8)
    xs = [data(r, 77) for r in range(7)]
    bufs = [x.copy() for x in xs]
    run_collective(cs, lambda c: c.all_reduce_host(bufs[c.rank]))
    np.testing.assert_allclose(bufs[3], np.sum([x.astype(np.float64) for x in xs], axis=0), rtol=1e-5, atol=1e-5)


# ------------------------------------------------------------ fault injection
FAST = dict(collective_timeout_s=2.0, barrier_timeout_s=2.0, heartbeat_interval_s=0.1, heartbeat_timeout_s=1.0,
            recovery_timeout_s=5.0, rpc_timeout_s=2.0)


def test_dead_peer_before_allreduce_errors_not_deadlocks():
    cs = bootstrap(3, **FAST)
    cs[2].close()
    x = np.ones(10, np.float32)
    t0 = time.time()
    with pytest.raises(NexarError):
        run_collective(cs[:2], lambda c: c.all_reduce_host(x.copy()))
    assert time.time() - t0 < 10


def test_barrier_with_dead_peer_errors():
    cs = bootstrap(3, **FAST)
    cs[1].close()
    with pytest.raises(NexarError):
        run_collective([cs[0], cs[2]], lambda c: c.barrier())


def test_dead_root_in_broadcast():
    cs = bootstrap(4, **FAST)
    cs[0].close()
    with pytest.raises(NexarError):
        run_collective(cs[1:], lambda c: c.broadcast_host(np.zeros(8, np.float32), 0))


def test_rank_never_joins_collective_times_out():
    cs = bootstrap(2, **FAST)
    t0 = time.time()
    with pytest.raises(CollectiveFailed):
        cs[0].all_reduce_host(np.ones(4, np.float32))
    assert 1.5 < time.time() - t0 < 10


def test_mid_collective_kill():
    cs = bootstrap(3, **FAST)

    def killer():
        time.sleep(0.05)
        cs[2].close()
    threading.Thread(target=killer).start()
    with pytest.raises(NexarError):
        run_collective(cs[:2], lambda c: [c.barrier() or c.all_reduce_host(np.ones(1000, np.float32)) for _ in range(200)])


def test_health_monitor_detects_failure_within_3s():
    cs = bootstrap(3, **FAST)
    cs[1].close()
    t0 = time.time()
    dead = []
    while time.time() - t0 < 3 and 1 not in dead:
        dead = cs[0].wait_failure(0.2)
    assert 1 in dead


# ------------------------------------------------------------ recovery
def _h():
    from nexar_b200 import _native
    return _native.host()


def test_recovery_abort_policy():
    cs = bootstrap(3, **FAST)
    orch = _h().RecoveryOrchestrator(cs[0].native, 2)
    orch.start()
    cs[2].close()
    t0 = time.time()
    while not orch.error() and time.time() - t0 < 5:
        time.sleep(0.05)
    assert "Abort" in orch.error()
    orch.shutdown()


def test_recovery_manual_policy_emits_event():
    cs = bootstrap(3, **FAST)
    orch = _h().RecoveryOrchestrator(cs[0].native, 1)
    orch.start()
    cs[2].close()
    ev = orch.next_event(5.0)
    assert ev is not None and 2 in ev.dead_ranks and ev.new_world_size == 3
    orch.shutdown()


@pytest.mark.parametrize("dead", [[2], [0], [1, 3]])
def test_recovery_automatic_rebuild_and_collective(dead):
    cs = bootstrap(4, **FAST)
    survivors = [c for c in cs if c.rank not in dead]
    orchs = [_h().RecoveryOrchestrator(c.native, 0) for c in survivors]
    for o in orchs:
        o.start()
    for d in dead:
        cs[d].close()
    evs = [o.next_event(10.0) for o in orchs]
    assert all(e is not None for e in evs)
    assert all(sorted(e.dead_ranks) == sorted(dead) for e in evs)
    new = [NexarClient(o.client()) for o in orchs]
    assert sorted(c.rank for c in new) == list(range(4 - len(dead)))
    bufs = [np.full(6, float(c.rank + 1), np.float32) for c in new]
    run_collective(new, lambda c: c.all_reduce_host(bufs[c.rank]))
    n = len(new)
    assert (bufs[0] == n * (n + 1) / 2).all()
    for o in orchs:
        o.shutdown()


def test_recovery_cascading_failures():
    cs = bootstrap(5, **FAST)
    survivors = cs[:3]
    orchs = [_h().RecoveryOrchestrator(c.native, 0) for c in survivors]
    for o in orchs:
        o.start()
    cs[4].close()
    time.sleep(0.3)
    cs[3].close()
    deadline = time.time() + 15
    final = [None] * 3
    while time.time() < deadline and any(f is None or f.new_world_size != 3 for f in final):
        for i, o in enumerate(orchs):
            e = o.next_event(0.2)
            if e is not None:
                final[i] = e
    assert all(f is not None and f.new_world_size == 3 for f in final)
    new = [NexarClient(o.client()) for o in orchs]
    run_collective(new, lambda c: c.barrier())
    for o in orchs:
        o.shutdown()


def test_rebuild_excluding_direct():
    cs = bootstrap(4)
    sub = run_collective([cs[0], cs[1], cs[3]], lambda c: c.rebuild_excluding([2]))
    assert [s.rank for s in sub] == [0, 1, 2] and len({s.comm_id for s in sub}) == 1
    bufs = [np.full(4, float(i), np.float32) for i in range(3)]
    run_collective(sub, lambda s: s.all_reduce_host(bufs[s.rank]))
    assert (bufs[2] == 3).all()


# ------------------------------------------------------------ elastic
@pytest.mark.parametrize("tls", [False, True])
def test_elastic_noop_checkpoint_and_grow_and_shrink(tls):
    H = _h()
    seed = H.SeedNode.bind_local(tls)
    cfg = Config(tls=tls, **FAST)
    clients = [None, None]

    def boot(i):
        clients[i] = H.NexarClient.bootstrap_worker(seed.local_addr(), None, cfg, "127.0.0.1")
    ts = [threading.Thread(target=boot, args=(i,)) for i in range(2)]
    [t.start() for t in ts]
    seed.form_cluster(2)
    [t.join() for t in ts]
    clients.sort(key=lambda c: c.rank)
    seed.accept_elastic(8)
    mgrs = [H.ElasticManager(clients[0], seed, 1, 8, 10.0), H.ElasticManager(clients[1], None, 1, 8, 10.0)]
    # no-op checkpoint
    assert run_collective(mgrs, lambda m: m.elastic_checkpoint()) == [False, False]
    # grow: a third rank joins through the seed
    joined = {}

    def joiner():
        joined["c"] = H.ElasticManager.join(seed.local_addr(), None, cfg, 20.0)
    jt = threading.Thread(target=joiner)
    jt.start()
    time.sleep(0.5)  # the seed queues the join
    assert run_collective(mgrs, lambda m: m.elastic_checkpoint()) == [True, True]
    jt.join(20)
    grown = [NexarClient(mgrs[0].client()), NexarClient(mgrs[1].client()), NexarClient(joined["c"])]
    assert sorted(c.world_size for c in grown) == [3, 3, 3]
    assert sorted(c.rank for c in grown) == [0, 1, 2]
    assert len({c.comm_id for c in grown}) == 1
    bufs = [np.full(5, float(c.rank + 1), np.float32) for c in grown]
    run_collective(grown, lambda c: c.all_reduce_host(bufs[c.rank]))
    assert all((b == 6).all() for b in bufs)
    assert all(c.native.transport_encrypted() == tls for c in grown)
    # shrink: rank 1 leaves at the next checkpoint
    m3 = [H.ElasticManager(c.native, seed if c.rank == 0 else None, 1, 8, 10.0) for c in sorted(grown, key=lambda c: c.rank)]
    m3[0].remove_node(1)
    subs = [m.subscribe() for m in m3]
    assert run_collective(m3, lambda m: m.elastic_checkpoint()) == [True, True, True]
    evs = [s.recv(5.0) for s in subs]
    assert all(e is not None and e.left == [1] and e.new_world_size == 2 for e in evs)
    assert m3[1].client() is None
    rest = [NexarClient(m3[0].client()), NexarClient(m3[2].client())]
    assert sorted(c.world_size for c in rest) == [2, 2]
    run_collective(rest, lambda c: c.barrier())
    seed.close()


# ------------------------------------------------------------ multi-process
def _proc_rank(seed_addr, q):
    import numpy as np
    from nexar_b200.client import NexarClient
    c = NexarClient.bootstrap(seed_addr)
    x = np.full(16, float(c.rank + 1), np.float32)
    c.all_reduce_host(x)
    out = np.zeros(16 * c.world_size, np.float32)
    c.all_gather_host(x, out)
    c.barrier()
    q.put((c.rank, float(x[0]), float(out.sum())))


def test_multiprocess_seed_worker_bootstrap():
    H = _h()
    seed = H.SeedNode.bind("127.0.0.1:0", b"secret-token")
    os.environ["NEXAR_CLUSTER_TOKEN"] = "secret-token"
    try:
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        ps = [ctx.Process(target=_proc_rank, args=(seed.local_addr(), q)) for _ in range(3)]
        [p.start() for p in ps]
        seed.with_formation_timeout(60.0).form_cluster(3)
        res = sorted(q.get(timeout=120) for _ in range(3))
        [p.join(30) for p in ps]
    finally:
        del os.environ["NEXAR_CLUSTER_TOKEN"]
        seed.close()
    assert [r[0] for r in res] == [0, 1, 2]
    assert all(r[1] == 6.0 for r in res) and all(r[2] == 6.0 * 16 * 3 for r in res)


def test_seed_rejects_wrong_token():
    from nexar_b200.core import ClusterFormationTimeout
    H = _h()
    seed = H.SeedNode.bind("127.0.0.1:0", b"right").with_formation_timeout(1.5)
    errs = []

    def bad():
        try:
            H.NexarClient.bootstrap_worker(seed.local_addr(), b"wrong", Config(), "127.0.0.1")
        except Exception as e:  # noqa: BLE001
            errs.append(e)
    t = threading.Thread(target=bad)
    t.start()
    with pytest.raises(ClusterFormationTimeout):
        seed.form_cluster(1)
    t.join(30)
    assert errs
    seed.close()


def test_recovery_run_subscribe_broadcast():
    """run() blocks on its thread until shutdown; every subscriber sees the event
    (broadcast receivers, nexar/src/cluster/recovery.rs:56-81)."""
    import threading
    from nexar_b200.client import RecoveryOrchestrator, RecoveryPolicy
    from nexar_b200.core import NexarError
    cs = bootstrap(3, **FAST)
    (o0, r0a), (o1, r1) = RecoveryOrchestrator.new(cs[0]), RecoveryOrchestrator.new(cs[1], RecoveryPolicy.Automatic)
    r0b = o0.subscribe()
    t = threading.Thread(target=o0.run, daemon=True)
    t.start()
    o1.start()
    with pytest.raises(NexarError):
        o1.run()  # its loop already runs on start()'s thread
    cs[2].close()
    evs = [r.recv(10.0) for r in (r0a, r0b, r1)]
    assert all(e is not None and e.dead_ranks == [2] and e.new_world_size == 2 for e in evs)
    assert r0a.recv(0.05) is None and r0a.dropped == 0
    new = [o0.client(), o1.client()]
    run_collective(new, lambda c: c.barrier())
    o0.shutdown()
    t.join(5.0)
    assert not t.is_alive()
    assert r0a.recv(0.05) is None  # closed and drained
    o1.shutdown()
