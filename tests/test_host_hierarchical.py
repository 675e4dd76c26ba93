"""Hierarchical (node x cross-node) collectives on CPU tensors, with nodes
emulated by host-name overrides on one machine (one thread per rank over
loopback TCP). Parity: nexar-nccl/src/topology.rs, bootstrap.rs and
collective/*.rs, whose tests need GPUs and several hosts."""
import pytest
import torch

from helpers_host import bootstrap, run_collective
from nexar_b200.parallel.hierarchical import HierarchicalComm, NodeTopology

LAYOUTS = {
    "blocks": ["a", "a", "b", "b"],
    "interleaved": ["a", "b", "a", "b"],
    "uneven": ["a", "a", "a", "b"],
    "singletons": ["a", "b", "c", "d"],
    "one_node": ["a", "a", "a", "a"],
}


def test_topology_from_hostnames():
    t = NodeTopology.from_hostnames(3, ["x", "y", "x", "z", "y"])
    assert t.nodes == [[0, 2], [1, 4], [3]]
    assert t.node_idx == 2 and t.local_rank == 0 and t.is_lead
    assert t.inter_node_leads == [0, 1, 3]
    assert not t.uniform
    t4 = NodeTopology.from_hostnames(4, ["x", "y", "x", "z", "y"])
    assert t4.node_idx == 1 and t4.local_rank == 1 and not t4.is_lead and t4.lead == 1
    assert NodeTopology.from_hostnames(0, ["a", "b", "a", "b"]).uniform


def _comms(layout, **kw):
    names = LAYOUTS[layout]
    clients = bootstrap(len(names))
    comms = run_collective(clients, lambda c: HierarchicalComm(c, hostname=names[c.rank], **kw))
    return clients, comms


def _val(rank, n, seed=0):
    g = torch.Generator().manual_seed(seed * 100 + rank)
    return torch.randint(-50, 50, (n,), generator=g).float()


@pytest.mark.parametrize("layout", sorted(LAYOUTS))
def test_hierarchical_collectives(layout):
    clients, comms = _comms(layout, small_bytes=1024)
    W = len(clients)
    try:
        assert [c.rank for c in comms] == list(range(W))
        assert {c.num_nodes for c in comms} == {len(set(LAYOUTS[layout]))}
        for n in (7, 64, 4096):  # small path, large path, large path with many chunks
            want = sum(_val(r, n) for r in range(W))
            outs = run_collective(comms, lambda c: c.all_reduce(_val(c.rank, n)))
            for o in outs:
                assert torch.equal(o, want), (layout, n)
            mx = torch.stack([_val(r, n) for r in range(W)]).max(0).values
            outs = run_collective(comms, lambda c: c.all_reduce(_val(c.rank, n), op="max"))
            for o in outs:
                assert torch.equal(o, mx)

        c_per = 33
        full = sum(_val(r, W * c_per, 1) for r in range(W)).view(W, c_per)
        outs = run_collective(comms, lambda c: c.reduce_scatter(_val(c.rank, W * c_per, 1), torch.empty(c_per)))
        for r, o in enumerate(outs):
            assert torch.equal(o, full[r]), (layout, r)

        outs = run_collective(comms, lambda c: c.all_gather(_val(c.rank, c_per, 2), torch.empty(W * c_per)))
        want = torch.cat([_val(r, c_per, 2) for r in range(W)])
        for o in outs:
            assert torch.equal(o, want)

        for root in range(W):
            outs = run_collective(comms, lambda c: c.broadcast(_val(c.rank, 19, 3), root))
            for o in outs:
                assert torch.equal(o, _val(root, 19, 3)), (layout, root)
            outs = run_collective(comms, lambda c: c.reduce(_val(c.rank, 19, 4), root))
            assert torch.equal(outs[root], sum(_val(r, 19, 4) for r in range(W))), (layout, root)

        # the collectives the reference's facade lacks (carried by the flat client)
        k = 5
        outs = run_collective(comms, lambda c: c.all_to_all(_val(c.rank, W * k, 5), torch.empty(W * k)))
        for r, o in enumerate(outs):
            assert torch.equal(o, torch.cat([_val(q, W * k, 5)[r * k:(r + 1) * k] for q in range(W)])), layout
        outs = run_collective(comms, lambda c: c.gather(_val(c.rank, k, 6), torch.empty(W * k) if c.rank == 1
                                                        else None, root=1))
        assert torch.equal(outs[1], torch.cat([_val(q, k, 6) for q in range(W)]))
        outs = run_collective(comms, lambda c: c.scatter(_val(c.rank, W * k, 7) if c.rank == 2 else None,
                                                         torch.empty(k), root=2))
        for r, o in enumerate(outs):
            assert torch.equal(o, _val(2, W * k, 7)[r * k:(r + 1) * k])
        outs = run_collective(comms, lambda c: c.scan(_val(c.rank, k, 8)))
        for r, o in enumerate(outs):
            assert torch.equal(o, sum(_val(q, k, 8) for q in range(r + 1)))
        outs = run_collective(comms, lambda c: c.exclusive_scan(_val(c.rank, k, 9)))
        assert torch.equal(outs[0], torch.zeros(k))
        assert torch.equal(outs[W - 1], sum(_val(q, k, 9) for q in range(W - 1)))

        run_collective(comms, lambda c: c.barrier())
    finally:
        for c in clients:
            c.close()


def test_hierarchical_facade_properties():
    clients, comms = _comms("interleaved")
    try:
        c1 = comms[1]
        assert (c1.rank, c1.world_size, c1.num_nodes, c1.node_idx, c1.local_rank, c1.local_world_size) == \
            (1, 4, 2, 1, 0, 2)
        assert c1.is_lead and not comms[3].is_lead
        with pytest.raises(ValueError):
            comms[0].all_gather(torch.zeros(3), torch.zeros(5))
    finally:
        for c in clients:
            c.close()
