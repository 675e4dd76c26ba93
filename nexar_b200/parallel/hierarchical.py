"""Two-level communicator: the device (or host) communicator inside a node,
the host transport across nodes.

Parity with the reference's NCCL extension crate:
  * node discovery (nexar-nccl/src/topology.rs:7-145): every rank all-gathers
    its host name; nodes are numbered in first-appearance order by rank, the
    lead of a node is its lowest rank, local ranks follow global rank order;
  * bootstrap (nexar-nccl/src/bootstrap.rs:24-120): sub-communicators for the
    node and for the node leads are split off the flat client;
  * collectives (nexar-nccl/src/collective/*.rs) and the facade
    (nexar-nccl/src/comm.rs:17-181: rank, world, num_nodes, local_rank,
    is_lead, all_reduce, broadcast, all_gather, reduce, barrier), plus
    reduce_scatter, which the reference's facade lacks.

Algorithms. Let N be the number of nodes and L the ranks per node. When every
node has the same L ("uniform"), each local rank l is also a member of the
cross-node communicator of all ranks with local index l (one per node):
  * all_reduce (large, numel divisible by L): local reduce-scatter, all-reduce
    of the rank's own 1/L chunk across nodes by EVERY local rank in parallel,
    local all-gather. (The reference runs the cross-node step on the lead only,
    for the lead's chunk, and leaves the other chunks unreduced across nodes;
    this build reduces all of them.)
  * all_reduce (small, indivisible, or non-uniform nodes): local all-reduce,
    leads all-reduce across nodes, local broadcast from the lead (the
    reference's small-message path).
  * reduce_scatter: chunks permuted to (local index, node) order, local
    reduce-scatter (each local rank gets its N chunks summed over the node),
    reduce-scatter across nodes: bandwidth-optimal in both levels.
  * all_gather: the inverse (gather across nodes, then in the node, then the
    permutation back to global rank order).
  * broadcast / reduce: through the cross-node communicator of the root's
    local index, then within every node.
Non-uniform layouts fall back to lead-based forms that are correct for any
node sizes.

Tensors: CUDA tensors use the node's ``DeviceCommunicator`` (sm_100a
peer-memory / NVLS kernels) and cross nodes through pinned host staging;
CPU tensors use the node's host sub-communicator. One process per rank (or
one thread per rank with ``NexarClient.bootstrap_local``).
"""
from __future__ import annotations

import os
import socket
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch

from ..core import ReduceOp

__all__ = ["NodeTopology", "discover_topology", "HierarchicalComm", "form_hierarchical_comm"]


@dataclass
class NodeTopology:
    rank: int
    world_size: int
    hostnames: List[str]
    nodes: List[List[int]] = field(default_factory=list)  # ranks of each node, ascending
    node_of: List[int] = field(default_factory=list)      # node index of every rank

    @classmethod
    def from_hostnames(cls, rank: int, hostnames: List[str]) -> "NodeTopology":
        order: Dict[str, int] = {}
        nodes: List[List[int]] = []
        node_of: List[int] = []
        for r, h in enumerate(hostnames):
            if h not in order:
                order[h] = len(nodes)
                nodes.append([])
            nodes[order[h]].append(r)
            node_of.append(order[h])
        return cls(rank, len(hostnames), list(hostnames), nodes, node_of)

    @property
    def num_nodes(self) -> int:
        return len(self.nodes)

    @property
    def node_idx(self) -> int:
        return self.node_of[self.rank]

    @property
    def local_ranks(self) -> List[int]:
        return self.nodes[self.node_idx]

    @property
    def local_rank(self) -> int:
        return self.local_ranks.index(self.rank)

    @property
    def local_world_size(self) -> int:
        return len(self.local_ranks)

    @property
    def lead(self) -> int:
        return self.local_ranks[0]

    @property
    def is_lead(self) -> bool:
        return self.rank == self.lead

    @property
    def inter_node_leads(self) -> List[int]:
        return [n[0] for n in self.nodes]

    @property
    def uniform(self) -> bool:
        return len({len(n) for n in self.nodes}) == 1

    def local_index_of(self, rank: int) -> int:
        return self.nodes[self.node_of[rank]].index(rank)


def discover_topology(client, hostname: Optional[str] = None) -> NodeTopology:
    """All-gather host names over ``client`` (collective). ``hostname``
    overrides the machine's name (``NEXAR_HOSTNAME`` as well), which lets one
    machine emulate several nodes."""
    name = hostname or os.environ.get("NEXAR_HOSTNAME") or socket.gethostname()
    names = [b.decode() for b in client.all_gather_bytes(name.encode())]
    return NodeTopology.from_hostnames(client.rank, names)


class _HostTensorComm:
    """Tensor-level collectives of a host client, with the DeviceCommunicator's
    signatures (CPU tensors, in place where the device API is)."""

    def __init__(self, client):
        self.client = client
        self.rank = client.rank
        self.world_size = client.world_size

    def all_reduce(self, t, op="sum"):
        if self.world_size > 1:
            self.client.all_reduce_host(t, ReduceOp.parse(op))
        return t

    def reduce_scatter(self, inp, out, op="sum"):
        if self.world_size == 1:
            return out.copy_(inp)
        self.client.reduce_scatter_host(inp, out, ReduceOp.parse(op))
        return out

    def all_gather(self, inp, out):
        if self.world_size == 1:
            return out.copy_(inp.reshape(out.shape))
        self.client.all_gather_host(inp, out)
        return out

    def broadcast(self, t, root=0):
        if self.world_size > 1:
            self.client.broadcast_host(t, root)
        return t

    def reduce(self, t, root=0, op="sum"):
        if self.world_size > 1:
            self.client.reduce_host(t, ReduceOp.parse(op), root)
        return t

    def barrier(self):
        self.client.barrier()


class HierarchicalComm:
    """Node-aware collectives over a flat ``NexarClient`` (collective construction:
    every rank calls it in the same order). ``device_comm`` is the node's
    ``DeviceCommunicator`` for CUDA tensors (``attach_device=True`` builds
    one over the node sub-communicator; ``nccl=True`` adds the node's NCCL
    communicator for device send / recv, its id sent by the node's lead);
    CPU tensors need none."""

    SMALL_BYTES = 256 << 10  # below this, all_reduce takes the lead path (as the reference)
    PINNED_CACHE = 8         # pinned staging buffers kept (by dtype and size, least recently used out)

    def __init__(self, client, topology: Optional[NodeTopology] = None, hostname: Optional[str] = None,
                 attach_device: bool = False, device: Optional[int] = None, small_bytes: Optional[int] = None,
                 nccl: bool = False, **device_kw):
        self.client = client
        self.topo = topology or discover_topology(client, hostname)
        t = self.topo
        # Node communicator (local rank order = global rank order) and, for
        # every local index l, the communicator of the ranks with index l on
        # each node (node order); index 0 is the node leads.
        self.local_client = client.split(t.node_idx, t.rank)
        self.cross_client = client.split(t.local_rank, t.node_idx)
        self.local = _HostTensorComm(self.local_client)
        self.cross = _HostTensorComm(self.cross_client)
        self.device_comm = None
        if attach_device:
            self.device_comm = self.local_client.attach_device(device, nccl=nccl, **device_kw)
        self.small_bytes = self.SMALL_BYTES if small_bytes is None else int(small_bytes)
        self._pinned: Dict[Tuple[torch.dtype, int], torch.Tensor] = {}

    # ------------------------------------------------------------ facade
    @property
    def rank(self) -> int:
        return self.topo.rank

    @property
    def world_size(self) -> int:
        return self.topo.world_size

    @property
    def num_nodes(self) -> int:
        return self.topo.num_nodes

    @property
    def node_idx(self) -> int:
        return self.topo.node_idx

    @property
    def local_rank(self) -> int:
        return self.topo.local_rank

    @property
    def local_world_size(self) -> int:
        return self.topo.local_world_size

    @property
    def is_lead(self) -> bool:
        return self.topo.is_lead

    # ------------------------------------------------------------ plumbing
    def _intra(self, t: torch.Tensor):
        if t.is_cuda:
            if self.device_comm is None:
                raise RuntimeError("CUDA tensor but no device communicator: build with attach_device=True")
            return self.device_comm
        return self.local

    def _host(self, t: torch.Tensor) -> torch.Tensor:
        """Host tensor holding t's values (t itself for CPU tensors)."""
        if not t.is_cuda:
            return t
        key = (t.dtype, t.numel())
        h = self._pinned.pop(key, None)
        if h is None:
            h = torch.empty(t.numel(), dtype=t.dtype, pin_memory=True)
            while len(self._pinned) >= self.PINNED_CACHE:
                self._pinned.pop(next(iter(self._pinned)))  # least recently used
        self._pinned[key] = h
        h.copy_(t.reshape(-1), non_blocking=True)
        torch.cuda.current_stream(t.device).synchronize()
        return h

    @staticmethod
    def _back(t: torch.Tensor, h: torch.Tensor):
        if t.is_cuda:
            t.view(-1).copy_(h, non_blocking=True)

    def _cross_op(self, t: torch.Tensor, fn):
        """Run a host collective of the cross-node communicator on t's values."""
        if self.cross.world_size == 1:
            return
        h = self._host(t)
        fn(h)
        self._back(t, h)

    # ------------------------------------------------------------ collectives
    def all_reduce(self, t: torch.Tensor, op="sum") -> torch.Tensor:
        """In-place all-reduce of a contiguous tensor over all ranks."""
        intra = self._intra(t)
        topo = self.topo
        if topo.num_nodes == 1:
            return intra.all_reduce(t, op=op) if intra.world_size > 1 else t
        L = topo.local_world_size
        flat = t.view(-1)
        large = t.numel() * t.element_size() >= self.small_bytes and t.numel() % L == 0
        if topo.uniform and large:
            chunk = torch.empty(t.numel() // L, dtype=t.dtype, device=t.device)
            if L > 1:
                intra.reduce_scatter(flat, chunk, op=op)
            else:
                chunk.copy_(flat)
            self._cross_op(chunk, lambda h: self.cross.all_reduce(h, op))
            if L > 1:
                intra.all_gather(chunk, flat)
            else:
                flat.copy_(chunk)
            return t
        return self._all_reduce_lead(t, op)

    def _all_reduce_lead(self, t, op):
        intra = self._intra(t)
        if intra.world_size > 1:
            intra.all_reduce(t, op=op)
        if self.topo.is_lead:
            self._cross_op(t, lambda h: self.cross.all_reduce(h, op))
        if intra.world_size > 1:
            intra.broadcast(t, 0)
        return t

    def reduce_scatter(self, inp: torch.Tensor, out: torch.Tensor, op="sum") -> torch.Tensor:
        """out (numel c) = chunk `rank` of the reduction of inp (numel world * c)."""
        topo = self.topo
        W, c = topo.world_size, out.numel()
        if inp.numel() != W * c:
            raise ValueError("reduce_scatter: inp must hold world_size * out.numel() elements")
        intra = self._intra(inp)
        if topo.num_nodes == 1:
            if intra.world_size == 1:
                return out.copy_(inp.view(out.shape))
            intra.reduce_scatter(inp.view(-1), out.view(-1), op=op)
            return out
        if not topo.uniform:
            full = inp.clone()
            self._all_reduce_lead(full, op)
            return out.copy_(full.view(W, c)[topo.rank].view(out.shape))
        N, L = topo.num_nodes, topo.local_world_size
        # chunk of rank (node n, local l) goes to slot l * N + n
        order = [topo.nodes[n][l] for l in range(L) for n in range(N)]
        perm = inp.view(W, c)[torch.tensor(order, device=inp.device)].contiguous().view(-1)
        mine = torch.empty(N * c, dtype=inp.dtype, device=inp.device)
        if L > 1:
            intra.reduce_scatter(perm, mine, op=op)
        else:
            mine.copy_(perm)
        # mine: N chunks (ranks (n', l) for every node n'), summed over this node
        if N > 1:
            hm = self._host(mine)
            ho = torch.empty(c, dtype=inp.dtype)
            self.cross.reduce_scatter(hm, ho, op)
            out.view(-1).copy_(ho)
        else:
            out.view(-1).copy_(mine)
        return out

    def all_gather(self, inp: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """out (world * c) = every rank's inp (c) in rank order."""
        topo = self.topo
        W, c = topo.world_size, inp.numel()
        if out.numel() != W * c:
            raise ValueError("all_gather: out must hold world_size * inp.numel() elements")
        intra = self._intra(inp)
        if topo.num_nodes == 1:
            if intra.world_size == 1:
                return out.copy_(inp.view(out.shape))
            intra.all_gather(inp.view(-1), out.view(-1))
            return out
        if not topo.uniform:
            buf = torch.zeros(W, c, dtype=inp.dtype, device=inp.device)
            buf[topo.rank].copy_(inp.view(-1))
            self._all_reduce_lead(buf.view(-1), "sum")
            return out.copy_(buf.view(out.shape))
        N, L = topo.num_nodes, topo.local_world_size
        hi = self._host(inp.contiguous())
        ho = torch.empty(N * c, dtype=inp.dtype)
        if N > 1:
            self.cross.all_gather(hi, ho)
        else:
            ho.copy_(hi)
        node_blk = ho.to(inp.device) if inp.is_cuda else ho
        slots = torch.empty(L * N * c, dtype=inp.dtype, device=inp.device)
        if L > 1:
            intra.all_gather(node_blk.contiguous(), slots)
        else:
            slots.copy_(node_blk)
        # slots[l * N + n] holds rank (n, l); scatter back to rank order
        order = [topo.nodes[n][l] for l in range(L) for n in range(N)]
        dst = out.view(W, c)
        dst[torch.tensor(order, device=out.device)] = slots.view(L * N, c)
        return out

    def broadcast(self, t: torch.Tensor, root: int = 0) -> torch.Tensor:
        topo = self.topo
        intra = self._intra(t)
        rn, rl = topo.node_of[root], topo.local_index_of(root)
        if topo.num_nodes == 1:
            return intra.broadcast(t, rl) if intra.world_size > 1 else t
        if all(len(n) > rl for n in topo.nodes):
            # the ranks with the root's local index carry it across nodes
            if topo.local_rank == rl:
                self._cross_op(t, lambda h: self.cross.broadcast(h, rn))
            if intra.world_size > 1:
                intra.broadcast(t, rl)
            return t
        # lead form: root -> its node, leads, every other node
        if topo.node_idx == rn and intra.world_size > 1:
            intra.broadcast(t, rl)
        if topo.is_lead:
            self._cross_op(t, lambda h: self.cross.broadcast(h, rn))
        if topo.node_idx != rn and intra.world_size > 1:
            intra.broadcast(t, 0)
        return t

    def reduce(self, t: torch.Tensor, root: int = 0, op="sum") -> torch.Tensor:
        """Reduction lands in the root's t; other ranks' t hold partial results."""
        topo = self.topo
        intra = self._intra(t)
        rn, rl = topo.node_of[root], topo.local_index_of(root)
        if topo.num_nodes == 1:
            return intra.reduce(t, rl, op=op) if intra.world_size > 1 else t
        if all(len(n) > rl for n in topo.nodes):
            if intra.world_size > 1:
                intra.reduce(t, rl, op=op)
            if topo.local_rank == rl:
                self._cross_op(t, lambda h: self.cross.reduce(h, rn, op))
            return t
        return self._all_reduce_lead(t, op)

    # The collectives below run over the flat client (host transport, CUDA
    # tensors staged through host memory): correct for every node layout,
    # without a two-level schedule. nexar-nccl's facade has none of them.
    @staticmethod
    def _to_host(t: torch.Tensor) -> torch.Tensor:
        return t.detach().contiguous().reshape(-1).cpu() if t.is_cuda else t.contiguous().reshape(-1)

    def all_to_all(self, inp: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Rank r's out chunk q = rank q's inp chunk r (world_size equal chunks)."""
        hi = self._to_host(inp)
        ho = torch.empty_like(hi)
        self.client.all_to_all_host(hi, ho)
        out.view(-1).copy_(ho)
        return out

    def gather(self, inp: torch.Tensor, out: Optional[torch.Tensor], root: int = 0) -> Optional[torch.Tensor]:
        """The root's out (world_size x inp) receives every rank's inp in rank order."""
        hi = self._to_host(inp)
        ho = torch.empty(hi.numel() * self.world_size, dtype=hi.dtype) if self.rank == root else None
        self.client.gather_host(hi, ho, root)
        if self.rank == root:
            out.view(-1).copy_(ho)
        return out

    def scatter(self, inp: Optional[torch.Tensor], out: torch.Tensor, root: int = 0) -> torch.Tensor:
        """Rank r's out receives chunk r of the root's inp."""
        hi = self._to_host(inp) if self.rank == root else None
        ho = torch.empty(out.numel(), dtype=out.dtype)
        self.client.scatter_host(hi, ho, root)
        out.view(-1).copy_(ho)
        return out

    def scan(self, t: torch.Tensor, op="sum") -> torch.Tensor:
        """In place: rank r holds op over ranks 0..r."""
        h = self._to_host(t).clone()
        self.client.scan_host(h, ReduceOp.parse(op))
        t.view(-1).copy_(h)
        return t

    def exclusive_scan(self, t: torch.Tensor, op="sum") -> torch.Tensor:
        """In place: rank r holds op over ranks 0..r-1 (the identity on rank 0)."""
        h = self._to_host(t).clone()
        self.client.exclusive_scan_host(h, ReduceOp.parse(op))
        t.view(-1).copy_(h)
        return t

    def barrier(self):
        self.local.barrier()
        if self.topo.is_lead and self.cross.world_size > 1:
            self.cross.barrier()
        self.local.barrier()

    def close(self):
        self._pinned.clear()


def form_hierarchical_comm(client, hostname: Optional[str] = None, attach_device: bool = True,
                           device: Optional[int] = None, **kw) -> HierarchicalComm:
    """Topology discovery + sub-communicators + (optionally) the node's device
    communicator (nexar-nccl/src/bootstrap.rs: form_hierarchical_comm)."""
    if attach_device and device is None and torch.cuda.is_available():
        device = torch.cuda.current_device()
    return HierarchicalComm(client, hostname=hostname, attach_device=attach_device and torch.cuda.is_available(),
                            device=device, **kw)
