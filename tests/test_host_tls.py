"""TLS 1.3 on host links: cluster CA, mutual authentication, collectives over TLS
(in one process and across processes), and rejection of a foreign certificate."""
import multiprocessing as mp
import os

import numpy as np
import pytest

from helpers_host import run_collective


def _h():
    from nexar_b200 import _native
    return _native.host()


def test_tls_handshake_requires_the_cluster_ca():
    H = _h()
    assert H.tls_pair_check(True)       # both certificates from the same cluster CA
    assert not H.tls_pair_check(False)  # client certificate from an unrelated CA: refused


def test_bootstrap_local_tls_collectives():
    from nexar_b200.client import Config, NexarClient
    cs = NexarClient.bootstrap_local(4, Config(tls=True))
    assert all(c.native.transport_encrypted() for c in cs)
    bufs = [np.full(1000, float(c.rank + 1), np.float32) for c in cs]
    run_collective(cs, lambda c: c.all_reduce_host(bufs[c.rank]))
    assert all((b == 10.0).all() for b in bufs)
    big = [np.full(3 << 20, float(c.rank), np.float32) for c in cs]  # 12 MB: pipelined ring over TLS
    run_collective(cs, lambda c: c.all_reduce_host(big[c.rank]))
    assert all((b == 6.0).all() for b in big)
    outs = [np.zeros(16 * 4, np.float32) for _ in cs]
    run_collective(cs, lambda c: c.all_gather_host(np.full(16, float(c.rank), np.float32), outs[c.rank]))
    assert all(o.sum() == 16 * (0 + 1 + 2 + 3) for o in outs)
    plain = NexarClient.bootstrap_local(2)
    assert not any(c.native.transport_encrypted() for c in plain)


def _proc_rank_tls(seed_addr, q):
    from nexar_b200.client import Config, NexarClient
    c = NexarClient.bootstrap(seed_addr, config=Config(tls=True))
    x = np.full(16, float(c.rank + 1), np.float32)
    c.all_reduce_host(x)
    c.barrier()
    q.put((c.rank, float(x[0]), bool(c.native.transport_encrypted())))


def test_multiprocess_seed_worker_tls():
    H = _h()
    seed = H.SeedNode.bind("127.0.0.1:0", b"tls-token", True)
    assert seed.tls()
    os.environ["NEXAR_CLUSTER_TOKEN"] = "tls-token"
    try:
        ctx = mp.get_context("spawn")
        q = ctx.Queue()
        ps = [ctx.Process(target=_proc_rank_tls, args=(seed.local_addr(), q)) for _ in range(3)]
        [p.start() for p in ps]
        seed.with_formation_timeout(60.0).form_cluster(3)
        res = sorted(q.get(timeout=120) for _ in range(3))
        [p.join(30) for p in ps]
    finally:
        del os.environ["NEXAR_CLUSTER_TOKEN"]
        seed.close()
    assert [r[0] for r in res] == [0, 1, 2]
    assert all(r[1] == 6.0 and r[2] for r in res)


def test_cluster_ca_persist_and_restore():
    """The CA key pair survives a PEM round trip; identities issued by the
    restored CA are trusted by holders of the original's (tls.rs:122-143)."""
    from nexar_b200 import _native
    H = _native.host()
    ca = H.ClusterCA.generate("persisted-ca")
    key, cert = ca.key_pem(), ca.cert_pem()
    assert "PRIVATE KEY" in key and "BEGIN CERTIFICATE" in cert
    back = H.ClusterCA.from_pem(key, cert)
    assert back.cert_pem() == cert
    old_id, new_id = ca.issue("old-node"), back.issue("new-node")
    assert H.tls_identities_check(old_id, new_id) and H.tls_identities_check(new_id, old_id)
    other = H.ClusterCA.generate("other")
    assert not H.tls_identities_check(old_id, other.issue("x"))
    with pytest.raises(Exception):
        H.ClusterCA.from_pem(other.key_pem(), cert)  # key of another CA


def test_seed_reuses_persisted_ca():
    """A TLS seed given a restored CA forms a cluster whose mesh links chain to it."""
    import threading
    from nexar_b200 import _native
    from nexar_b200.client import NexarClient
    H = _native.host()
    ca = H.ClusterCA.generate("site-ca")
    saved = (ca.key_pem(), ca.cert_pem())
    seed = H.SeedNode.bind("127.0.0.1:0", b"tok", True)
    seed.use_ca(H.ClusterCA.from_pem(*saved))
    assert seed.ca().cert_pem() == saved[1]
    cfg = H.Config()
    cfg.tls = True
    out = {}

    def worker(i):
        out[i] = H.NexarClient.bootstrap_worker(seed.local_addr(), b"tok", cfg, "127.0.0.1")

    ts = [threading.Thread(target=worker, args=(i,)) for i in range(2)]
    for t in ts:
        t.start()
    seed.form_cluster(2)
    for t in ts:
        t.join(30)
    cs = [NexarClient(out[i]) for i in range(2)]
    assert all(c.native.transport_encrypted() for c in cs)
    import numpy as np
    bufs = [np.full(3, float(c.rank + 1), np.float32) for c in cs]
    from helpers_host import run_collective
    run_collective(cs, lambda c: c.all_reduce_host(bufs[c.rank]))
    assert (bufs[0] == 3).all()
    for c in cs:
        c.close()
    seed.close()
