"""DeviceCommunicator: device-pointer collectives over NVLink peer memory.

One process (or one thread) per GPU. Each rank allocates a symmetric heap of
the same size; handles are exchanged out of band (``torch.distributed`` or a
``nexar_b200`` host client) and every rank maps every peer's heap. All the
collectives below then run as single sm_100a kernels that load and store peer
HBM directly, with the reduction, scaling and dtype cast fused in.

This is the on-box device path that the reference delegates to NCCL
(nexar-nccl/src/comm.rs:122-181, nexar-nccl/src/group.rs:72-225), widened to
every collective of the host API (nexar/src/client/collectives.rs:12-262):
all_reduce, reduce_scatter, all_gather, all_to_all, broadcast, reduce, gather,
scatter, scan, exclusive_scan and barrier, plus ``*_nb`` variants returning a
handle (nexar/src/collective/handle.rs:12-91).

Semantics that differ from the reference's host ring, on purpose:
  * reduce_scatter gives rank r the reduction of chunk r (NCCL/MPI), not chunk
    (r+1) mod N (nexar/src/collective/reduce_scatter.rs:73-77).
Every device wait is bounded (``NEXAR_DEVICE_WAIT_TIMEOUT_US``); a kernel that
times out records it in a host-mapped status word and returns, and
:meth:`check` raises :class:`~nexar_b200.core.CollectiveFailed`.
"""
from __future__ import annotations

import contextlib
import functools
import os
from typing import Callable, List, Optional, Sequence

import torch

from .. import _native
from ..core import CollectiveFailed, DataType, ReduceOp

_ALGOS = {"auto": 0, "oneshot": 1, "one_shot": 1, "twoshot": 2, "two_shot": 2, "nvls": 3}
_OP_NAMES = {1: "all_reduce", 2: "reduce_scatter", 3: "all_gather", 4: "all_to_all",
             5: "broadcast", 6: "reduce", 7: "gather", 8: "scatter", 9: "scan",
             10: "barrier", 11: "moe_dispatch", 12: "moe_combine", 13: "gemm_reduce_scatter",
             14: "all_gather_gemm", 15: "compressed_all_reduce"}


_CHECK_NAMES = {1: "rank / world out of range", 2: "root or peer >= world", 3: "extent beyond its buffer",
                4: "barrier epoch not increasing"}


def _env_int(name: str, default: int) -> int:
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


class DeviceHandle:
    """Completion handle of a non-blocking device collective.

    ``wait()`` makes the caller's current stream wait for the collective
    (no host block), ``synchronize()`` blocks the host, ``is_finished()``
    polls. Mirrors ``CollectiveHandle`` (nexar/src/collective/handle.rs).
    """

    def __init__(self, event: torch.cuda.Event, keep: tuple, comm: "DeviceCommunicator"):
        self._event = event
        self._keep = keep
        self._comm = comm

    def wait(self):
        torch.cuda.current_stream(self._comm.device).wait_event(self._event)
        return self._keep[-1] if self._keep else None

    def synchronize(self):
        self._event.synchronize()
        self._comm.check()
        return self._keep[-1] if self._keep else None

    def is_finished(self) -> bool:
        return self._event.query()


_NVTX = os.environ.get("NEXAR_NVTX", "0") == "1"
_AR_ALGO_NAMES = {0: "local", 1: "one_shot", 2: "two_shot", 3: "nvls_staged", 4: "nvls_in_place",
                  5: "two_shot_in_place"}


_TIMING = os.environ.get("NEXAR_COMM_TIMING", "0") == "1"


class DeviceTimeHistogram:
    """Device time of every collective call, from CUDA events recorded around
    the launch on its stream and read back lazily (no synchronisation on the
    call path). Buckets are counts of calls up to each bound in microseconds
    (the last bucket is everything above the largest bound)."""

    EDGES_US = (10, 30, 100, 300, 1000, 3000, 10000)

    def __init__(self):
        self.pending: list = []
        self.per_op: dict = {}

    def record(self, op: str, start, end):
        self.pending.append((op, start, end))

    def resolve(self):
        keep = []
        for op, start, end in self.pending:
            if not end.query():
                keep.append((op, start, end))
                continue
            us = start.elapsed_time(end) * 1e3
            h = self.per_op.setdefault(op, {"count": 0, "total_us": 0.0, "min_us": float("inf"), "max_us": 0.0,
                                            "buckets": [0] * (len(self.EDGES_US) + 1)})
            h["count"] += 1
            h["total_us"] += us
            h["min_us"] = min(h["min_us"], us)
            h["max_us"] = max(h["max_us"], us)
            b = 0
            while b < len(self.EDGES_US) and us > self.EDGES_US[b]:
                b += 1
            h["buckets"][b] += 1
        self.pending = keep

    def summary(self) -> dict:
        self.resolve()
        out = {}
        for op, h in self.per_op.items():
            out[op] = dict(h, mean_us=h["total_us"] / h["count"], bucket_edges_us=list(self.EDGES_US))
        return out


def _observed(op: str):
    """Count calls and bytes per collective; NVTX range around it with NEXAR_NVTX=1;
    device time per call with NEXAR_COMM_TIMING=1 (``stats()["device_time"]``)."""
    def deco(fn):
        @functools.wraps(fn)
        def wrapper(self, *args, **kwargs):
            t = args[0] if args and isinstance(args[0], torch.Tensor) else None
            st = self._stats.setdefault(op, {"calls": 0, "bytes": 0})
            st["calls"] += 1
            if t is not None:
                st["bytes"] += t.numel() * t.element_size()
            if _NVTX:
                torch.cuda.nvtx.range_push(f"nexar.{op}")
            self.order_launch()
            timed = self._timer is not None and not torch.cuda.is_current_stream_capturing()
            if timed:
                ev0 = torch.cuda.Event(enable_timing=True)
                ev0.record()
            try:
                return fn(self, *args, **kwargs)
            finally:
                if timed:
                    ev1 = torch.cuda.Event(enable_timing=True)
                    ev1.record()
                    self._timer.record(op, ev0, ev1)
                if _NVTX:
                    torch.cuda.nvtx.range_pop()
                if op == "all_reduce":
                    name = _AR_ALGO_NAMES.get(self._comm.last_allreduce_algo, "?")
                    algos = self._stats.setdefault("all_reduce_algorithms", {})
                    algos[name] = algos.get(name, 0) + 1
        return wrapper
    return deco


class GlobalPtr:
    """(rank, heap offset, bytes) of a symmetric allocation (nexar's GlobalPtr,
    nexar/src/memory/global_ptr.rs:8-41, which the reference defines but never
    uses). Here it resolves: ``address()`` is the device virtual address of
    rank ``rank``'s copy, mapped into this process (peer memory over NVLink),
    usable by kernels that load or store another GPU's buffer directly."""

    def __init__(self, comm: "DeviceCommunicator", rank: int, offset: int, nbytes: int):
        self.comm, self.rank, self.offset, self.nbytes = comm, rank, offset, nbytes

    def address(self) -> int:
        return int(self.comm.native.peer_ptr(self.rank)) + self.offset

    def is_local(self, rank: Optional[int] = None) -> bool:
        """Whether the memory is on ``rank`` (default: the communicator's own rank)."""
        return self.rank == (self.comm.rank if rank is None else rank)

    def _key(self):
        return (id(self.comm), self.rank, self.offset, self.nbytes)

    def __eq__(self, other):
        return isinstance(other, GlobalPtr) and self._key() == other._key()

    def __hash__(self):
        return hash(self._key())

    def __repr__(self):
        return f"GlobalPtr(rank={self.rank}, offset={self.offset}, nbytes={self.nbytes})"

    def __str__(self):  # the reference's Display: rank and address range
        return f"rank {self.rank} [+{self.offset:#x}, {self.nbytes} bytes]"


class DeviceCommunicator:
    """Symmetric-memory communicator over the GPUs of one box."""

    def __init__(self, rank: int, world_size: int, device: int,
                 exchange: Callable[[bytes], List[bytes]],
                 heap_bytes: Optional[int] = None, slot_bytes: Optional[int] = None,
                 timeout_us: Optional[int] = None, barrier: Optional[Callable[[], None]] = None):
        C = _native.cuda()
        self.rank = rank
        self.world_size = world_size
        self.device = device
        slot = slot_bytes or _env_int("NEXAR_SLOT_BYTES", 256 << 20)
        user = _env_int("NEXAR_SYMM_USER_BYTES", 1 << 30)
        heap = heap_bytes or (1 << 20) + 2 * slot + user  # 1 MiB signal area first
        tmo = timeout_us if timeout_us is not None else _env_int("NEXAR_DEVICE_WAIT_TIMEOUT_US", 10_000_000)
        # One-shot (one barrier, every rank reads every peer's whole buffer)
        # against two-shot (two barriers, a staging round trip): in the sweeps
        # two-shot cost 30-42 us from 512 KB to 2 MB at every world size while
        # one-shot grew by about 1.5 us per doubling from 256 KB (18-20 us),
        # so one-shot runs to 2 MB up to 4 ranks and to 1 MB at 8, where every
        # rank reads seven peers.
        self.oneshot_max_bytes = _env_int(
            "NEXAR_AR_ONESHOT_MAX", (2 << 20) if world_size <= 4 else (1 << 20))
        self._comm = C.DeviceComm(rank, world_size, device, heap, slot, tmo)
        # Grid cap of a standalone collective (`NEXAR_MAX_BLOCKS`); the 2-, 4-
        # and 8-GPU sweeps ran with 148. Collectives that overlap compute
        # take a smaller grid through block_limit().
        self._comm.max_blocks = _env_int("NEXAR_MAX_BLOCKS", 148)
        # Device argument checks in every collective kernel (root / peer <
        # world, staged and symmetric extents, increasing barrier epochs); a
        # failed check is reported by check() and the kernel touches nothing.
        self._comm.checks = os.environ.get("NEXAR_DEVICE_CHECKS", "0") == "1"
        handles = exchange(self._comm.export_handle())
        if world_size > 1:
            self._comm.connect(list(handles))
        # NVSwitch multicast region: large all-reduce / reduce-scatter /
        # all-gather / broadcast reduce and replicate inside the switch.
        self._comm.nvls_min_bytes = _env_int("NEXAR_NVLS_MIN_BYTES", 16 << 20)
        nvls_user = _env_int("NEXAR_NVLS_USER_BYTES", 1 << 30)
        from . import nvls as _nvls
        self.nvls = _nvls.setup_nvls(self._comm, rank, world_size, exchange,
                                     (1 << 20) + C.nvls_stage_bytes() + nvls_user)
        self.nvls_reason = _nvls.LAST_REASON
        # NVLS moves about S bytes per GPU and direction for an all-reduce of S
        # bytes, the peer-to-peer two-shot 2 S (W-1)/W, but multimem runs
        # well below link rate: it only wins from 4 ranks up. Below that the
        # region stays available for explicit use (algo="nvls", nvls=True).
        self.nvls_preferred = self.nvls and world_size >= _env_int("NEXAR_NVLS_MIN_RANKS", 4)
        if self.nvls and not self.nvls_preferred:
            never = (1 << 64) - 1
            for k in ("nvls_min_bytes", "nvls_min_rs_bytes", "nvls_min_ag_bytes", "nvls_min_bcast_bytes"):
                setattr(self._comm, k, never)
        self._barrier = barrier
        if barrier is not None:
            barrier()  # every rank has mapped its peers before any kernel runs
        self._side_stream = None
        self._C = C
        self._stats = {}
        self._nccl = None
        self._timer = DeviceTimeHistogram() if _TIMING else None
        self._last_stream = None
        self._last_raw = None
        self._dev_index = torch.device(self.device).index if torch.device(self.device).index is not None else 0

    # ----------------------------------------------------------- construction
    @classmethod
    def from_torch(cls, group=None, device: Optional[int] = None, nccl: bool = False,
                   **kw) -> "DeviceCommunicator":
        """Build from an initialised ``torch.distributed`` process group
        (``nccl=True`` also attaches an NcclGroup over it for device send / recv)."""
        import torch.distributed as dist
        rank = dist.get_rank(group)
        world = dist.get_world_size(group)
        dev = torch.cuda.current_device() if device is None else device

        def exchange(h: bytes) -> List[bytes]:
            out: List = [None] * world
            dist.all_gather_object(out, h, group=group)
            return out

        def barrier():
            dist.barrier(group=group)

        out = cls(rank, world, dev, exchange, barrier=barrier, **kw)
        if nccl:
            from .nccl import NcclGroup
            out.attach_nccl(NcclGroup.from_torch(group, device=dev))
        return out

    @classmethod
    def from_client(cls, client, device: Optional[int] = None, **kw) -> "DeviceCommunicator":
        """Build from a ``nexar_b200`` host client (handles travel over its TCP mesh)."""
        dev = torch.cuda.current_device() if device is None else device

        def exchange(h: bytes) -> List[bytes]:
            return client.all_gather_bytes(h)

        return cls(client.rank, client.world_size, dev, exchange, barrier=client.barrier, **kw)

    # ----------------------------------------------------------- memory
    def symmetric_empty(self, shape: Sequence[int], dtype=torch.bfloat16, align: int = 256,
                        nvls: bool = False) -> torch.Tensor:
        """Allocate a tensor in symmetric memory (collective: same order and sizes on all ranks).

        Default: the peer-mapped heap. Peers can address the tensor directly
        (fused kernels store into it) and the two-shot all-reduce runs on it
        in place. ``nvls=True`` (when the NVLS region is active) places it in
        the multicast-bound region instead: large all-reduces on it run in
        place inside the NVSwitch, but peers cannot address it directly.
        """
        numel = 1
        for d in shape:
            numel *= int(d)
        nbytes = numel * torch.empty((), dtype=dtype).element_size()
        if self.nvls and nvls:
            off = self._comm.nvls_alloc(nbytes, align)
            return self._C.nvls_tensor(self._comm, off, list(shape), int(DataType.from_torch(dtype)))
        off = self._comm.alloc_symmetric(nbytes, align)
        return self._C.symmetric_tensor(self._comm, off, list(shape), int(DataType.from_torch(dtype)))

    def global_ptr(self, t: torch.Tensor, rank: int) -> GlobalPtr:
        """GlobalPtr to rank ``rank``'s copy of symmetric-heap tensor ``t``."""
        off = self._comm.symmetric_offset(t)
        if off < 0:
            raise ValueError("global_ptr needs a tensor from symmetric_empty() (peer-mapped heap)")
        if not 0 <= rank < self.world_size:
            raise ValueError(f"rank {rank} out of range")
        return GlobalPtr(self, rank, int(off), t.numel() * t.element_size())

    def is_symmetric(self, t: torch.Tensor) -> bool:
        """Whether t lies in this communicator's symmetric memory (heap or NVLS region)."""
        return self._comm.symmetric_offset(t) >= 0 or (self.nvls and self._comm.nvls_offset(t) >= 0)

    @property
    def native(self):
        return self._comm

    # ----------------------------------------------------------- launch order
    def order_launch(self):
        """Order the next kernel of this communicator after its previous one.

        Every collective kernel of one communicator shares a device call
        counter, the signal pad and the staging slots, so its kernels must run
        one after another. Kernels on one stream already do; when this launch
        goes to another stream than the previous one (a blocking collective on
        the current stream after a ``*_nb`` on the side stream, or the other
        way round), the new stream first waits for the old one. Collectives
        then complete in call order on every rank, as the reference's
        call-time tags keep concurrent non-blocking collectives apart
        (nexar/src/client/collectives_nb.rs:33-47). The fused kernels and the
        MoE dispatch / combine call this too."""
        # The raw handle is a cheap check on every call; Stream objects are
        # made only when the stream changed.
        raw = torch._C._cuda_getCurrentRawStream(self._dev_index)
        if raw == self._last_raw:
            return
        cur = torch.cuda.current_stream(self.device)
        last = self._last_stream
        if last is not None and last != cur:
            cap_now = torch.cuda.is_current_stream_capturing()
            with torch.cuda.stream(last):
                cap_last = torch.cuda.is_current_stream_capturing()
            # A capturing stream cannot wait on work outside its capture (and
            # the reverse): graph replays are ordered by the caller.
            if cap_now == cap_last:
                cur.wait_stream(last)
        self._last_stream = cur
        self._last_raw = raw

    @contextlib.contextmanager
    def block_limit(self, max_blocks: int):
        """Launch this communicator's kernels with at most ``max_blocks`` CTAs
        inside the block (e.g. collectives that overlap persistent compute
        kernels on the other SMs); the previous limit is restored after."""
        old = self._comm.max_blocks
        self._comm.max_blocks = max(1, int(max_blocks))
        try:
            yield
        finally:
            self._comm.max_blocks = old

    # ----------------------------------------------------------- status
    def close(self):
        """Release this communicator's device resources now (symmetric heap,
        peer mappings, NVLS region) instead of at garbage collection. Every
        rank closes together; tensors from ``symmetric_empty`` must not be
        used afterwards. The recovery and elastic paths close the old
        communicator before attaching one over the rebuilt client
        (``NexarClient.reattach_device``)."""
        if self._comm is None:
            return
        torch.cuda.synchronize(self.device)
        if self._nccl is not None:
            self._nccl.destroy()
            self._nccl = None
        self._side_stream = None
        self._comm = None

    @property
    def closed(self) -> bool:
        return self._comm is None

    @property
    def device_checks(self) -> bool:
        """Whether the collective kernels verify their arguments on the device."""
        return bool(self._comm.checks)

    @device_checks.setter
    def device_checks(self, on: bool):
        self._comm.checks = bool(on)

    def check(self):
        """Raise CollectiveFailed if any device wait of this communicator timed
        out or (with device checks on) a kernel refused its arguments."""
        st = self._comm.status()
        if st["code"] == 3:
            op = _OP_NAMES.get(st["op"], str(st["op"]))
            what = _CHECK_NAMES.get(st["block"], str(st["block"]))
            raise CollectiveFailed(
                f"{op} refused at rank {self.rank}: device check '{what}' failed "
                f"(value {st['rank']}, limit {st['epoch']}); the kernel stopped at the check")
        if st["code"] != 0:
            op = _OP_NAMES.get(st["op"], str(st["op"]))
            raise CollectiveFailed(
                f"{op} failed at rank {self.rank}: device wait for rank {st['rank']} timed out "
                f"(block {st['block']}, epoch {st['epoch']})")

    def status(self) -> dict:
        """The host-mapped status word (code, rank, op, block, epoch of the last failed wait)."""
        return self._comm.status()

    def stats(self) -> dict:
        """Per-collective call and byte counts, how often each all-reduce
        algorithm ran and, with timing on, each collective's device-time
        histogram (``device_time``)."""
        import copy
        out = copy.deepcopy(self._stats)
        if self._timer is not None:
            out["device_time"] = self._timer.summary()
        return out

    def enable_timing(self, on: bool = True):
        """Record the device time of every collective call from now on
        (``NEXAR_COMM_TIMING=1`` turns it on at construction)."""
        self._timer = (self._timer or DeviceTimeHistogram()) if on else None

    def clear_status(self):
        """Reset the status word after a reported failure."""
        self._comm.clear_status()

    # ----------------------------------------------------------- collectives
    @_observed("all_reduce")
    def all_reduce(self, t: torch.Tensor, op="sum", out: Optional[torch.Tensor] = None,
                   scale: Optional[float] = None, algo: str = "auto") -> torch.Tensor:
        """Reduce ``t`` across ranks. In place unless ``out`` is given.

        ``out`` may have a different dtype (fused cast, Sum only); ``scale``
        multiplies the result (e.g. 1/world for gradient averaging).
        """
        out = t if out is None else out
        self._C.all_reduce(self._comm, t, out, int(ReduceOp.parse(op)),
                           1.0 if scale is None else float(scale), _ALGOS[algo], self.oneshot_max_bytes)
        return out

    @_observed("reduce_scatter")
    def reduce_scatter(self, inp: torch.Tensor, out: Optional[torch.Tensor] = None, op="sum",
                       scale: Optional[float] = None) -> torch.Tensor:
        """``inp`` holds world*count elements; rank r receives the reduction of chunk r."""
        if out is None:
            if inp.numel() % self.world_size:
                from ..core import IndivisibleCount
                raise IndivisibleCount(f"count {inp.numel()} is not divisible by world size {self.world_size}")
            out = torch.empty(inp.numel() // self.world_size, dtype=inp.dtype, device=inp.device)
        self._C.reduce_scatter(self._comm, inp, out, int(ReduceOp.parse(op)), 1.0 if scale is None else float(scale))
        return out

    @_observed("all_gather")
    def all_gather(self, inp: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """out (world x inp) = every rank's inp in rank order (peer-memory or NVLS kernel)."""
        if out is None:
            out = torch.empty(inp.numel() * self.world_size, dtype=inp.dtype, device=inp.device)
        self._C.all_gather(self._comm, inp, out)
        return out

    @_observed("all_to_all")
    def all_to_all(self, inp: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """out chunk q = chunk r of rank q's inp (world equal chunks, peer stores)."""
        out = torch.empty_like(inp) if out is None else out
        self._C.all_to_all(self._comm, inp, out)
        return out

    @_observed("broadcast")
    def broadcast(self, t: torch.Tensor, root: int = 0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """t (or out) on every rank = the root's t (peer loads, scatter + all-gather, or NVLS multicast)."""
        out = t if out is None else out
        self._C.broadcast(self._comm, t, out, int(root))
        return out

    @_observed("reduce")
    def reduce(self, t: torch.Tensor, root: int = 0, op="sum", out: Optional[torch.Tensor] = None,
               scale: Optional[float] = None) -> torch.Tensor:
        """The root's t (or out) = op over all ranks' t."""
        out = t if out is None else out
        self._C.reduce(self._comm, t, out, int(root), int(ReduceOp.parse(op)), 1.0 if scale is None else float(scale))
        return out

    @_observed("gather")
    def gather(self, inp: torch.Tensor, root: int = 0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The root's out (world x inp) = every rank's inp in rank order."""
        if out is None:
            out = torch.empty(inp.numel() * self.world_size, dtype=inp.dtype, device=inp.device)
        self._C.gather(self._comm, inp, out, int(root))
        return out

    @_observed("scatter")
    def scatter(self, inp: torch.Tensor, root: int = 0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """out on rank r = chunk r of the root's inp."""
        if out is None:
            out = torch.empty(inp.numel() // self.world_size, dtype=inp.dtype, device=inp.device)
        self._C.scatter(self._comm, inp, out, int(root))
        return out

    @_observed("scan")
    def scan(self, inp: torch.Tensor, op="sum", out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """out on rank r = op over ranks 0..r of inp."""
        out = torch.empty_like(inp) if out is None else out
        self._C.scan(self._comm, inp, out, int(ReduceOp.parse(op)), False)
        return out

    @_observed("exclusive_scan")
    def exclusive_scan(self, inp: torch.Tensor, op="sum", out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """out on rank r = op over ranks 0..r-1 of inp (identity on rank 0)."""
        out = torch.empty_like(inp) if out is None else out
        self._C.scan(self._comm, inp, out, int(ReduceOp.parse(op)), True)
        return out

    @_observed("barrier")
    def barrier(self):
        """Device barrier: returns once every rank's stream has reached it (bounded waits)."""
        self._C.barrier(self._comm)

    # ----------------------------------------------------------- compressed all-reduce
    def all_reduce_compressed(self, t: torch.Tensor, ratio: float, residual: torch.Tensor,
                              out: Optional[torch.Tensor] = None, scale: float = 1.0) -> torch.Tensor:
        """Sum over ranks of each rank's top-k (by |residual + t|) entries, fp8-quantised.

        Error feedback as in the reference's TopKCompressor
        (nexar/src/compression/topk.rs): ``residual`` (fp32, same shape) keeps
        everything this rank has not sent yet, including the fp8 rounding error.
        k = ceil(numel * ratio). Every rank's (index, e4m3) blob is exchanged
        with the device all-gather and added into ``out`` (bf16) in rank
        order, so all ranks produce identical results. ``scale`` multiplies
        the result (e.g. 1/world for gradient averaging).
        """
        import math
        n = t.numel()
        k = max(1, min(n, math.ceil(n * ratio)))
        out = torch.empty_like(t) if out is None else out
        bb = self._C.compress_blob_bytes(k)
        ws = getattr(self, "_cmp_ws", {})
        self._cmp_ws = ws
        key = (n, k)
        if key not in ws:
            ws[key] = (torch.empty(self._C.compress_workspace_bytes(n), dtype=torch.uint8, device=t.device),
                       torch.empty(bb, dtype=torch.uint8, device=t.device),
                       torch.empty(bb * self.world_size, dtype=torch.uint8, device=t.device))
        work, blob, gathered = ws[key]
        self._C.topk_fp8_compress(t.reshape(-1), residual.reshape(-1), k, blob, work)
        if self.world_size > 1:
            self.all_gather(blob, gathered)
        else:
            gathered.copy_(blob)
        out.zero_()
        for p in range(self.world_size):
            self._C.decompress_accumulate(gathered[p * bb:(p + 1) * bb], k, out.reshape(-1), float(scale))
        return out

    # ----------------------------------------------------------- fused GEMM + collective
    def gemm_reduce_scatter(self, A: torch.Tensor, B: torch.Tensor, out: Optional[torch.Tensor] = None,
                            bias: Optional[torch.Tensor] = None, alpha: float = 1.0) -> torch.Tensor:
        """Row-parallel linear: returns this rank's rows of sum_r (A_r @ B_r^T) (+ bias).

        One persistent tcgen05 kernel: output tiles go straight into the owning
        rank's memory over NVLink while later tiles are still being multiplied.
        A: [M, K_local] bf16, B: [N, K_local] bf16 (nn.Linear layout); out: [M/world, N].
        """
        M, N = A.shape[0], B.shape[0]
        if out is None:
            out = torch.empty(M // self.world_size, N, dtype=A.dtype, device=A.device)
        self.order_launch()
        self._C.gemm_reduce_scatter(self._comm, A, B, out, bias, float(alpha))
        return out

    def gemm_fp8_reduce_scatter(self, A_q: torch.Tensor, A_s: torch.Tensor, B_q: torch.Tensor, B_s: torch.Tensor,
                                out: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None,
                                alpha: float = 1.0) -> torch.Tensor:
        """Block-scaled fp8 row-parallel linear fused with reduce-scatter (bf16 output).

        A_q: [M, K] e4m3 with 1x128 scales A_s [M, K/128]; B_q: [N, K] e4m3 with
        128x128 block scales B_s [N/128, K/128]; out: [M/world, N] bf16.
        """
        M, N = A_q.shape[0], B_q.shape[0]
        if out is None:
            out = torch.empty(M // self.world_size, N, dtype=torch.bfloat16, device=A_q.device)
        self.order_launch()
        self._C.gemm_fp8_reduce_scatter(self._comm, A_q, A_s, B_q, B_s, out, bias, float(alpha))
        return out

    def all_gather_gemm(self, x: torch.Tensor, B: torch.Tensor, out: Optional[torch.Tensor] = None,
                        bias: Optional[torch.Tensor] = None, act: Optional[str] = None,
                        pre: Optional[torch.Tensor] = None, alpha: float = 1.0) -> torch.Tensor:
        """Column-parallel linear on sequence-sharded input: act(all_gather(x) @ B^T + bias).

        One persistent tcgen05 kernel whose copy warps pull the peers' shards over
        NVLink (each remote row crosses once) while the tensor cores start on the
        local shard. x: [M/world, K] bf16, B: [N, K]; out: [M, N].
        """
        M, K = x.shape[0] * self.world_size, x.shape[1]
        if out is None:
            out = torch.empty(M, B.shape[0], dtype=x.dtype, device=x.device)
        afull, cnt = self._ag_workspace(M, K, x.device)
        self.order_launch()
        self._C.all_gather_gemm(self._comm, x, B, out, afull, cnt, bias, 1 if act == "gelu" else 0, pre, float(alpha))
        return out

    def gathered(self, M: int, K: int) -> torch.Tensor:
        """The gathered [M, K] input of the last ``all_gather_gemm`` of that
        shape (its local workspace; valid until the next call of the shape)."""
        ws = getattr(self, "_ag_ws", {}).get((M, K))
        if ws is None:
            raise RuntimeError(f"no all_gather_gemm of shape [{M}, {K}] has run on this communicator")
        return ws[0].view(M, K)

    def _ag_workspace(self, M: int, K: int, device):
        key = (M, K)
        ws = getattr(self, "_ag_ws", None)
        if ws is None:
            ws = self._ag_ws = {}
        if key not in ws:
            ws[key] = (torch.empty(M * K, dtype=torch.bfloat16, device=device),
                       torch.zeros(M // 128 + 2, dtype=torch.int32, device=device))
        return ws[key]

    # ----------------------------------------------------------- non-blocking
    def side_stream(self) -> torch.cuda.Stream:
        """The high-priority stream the non-blocking collectives run on."""
        if self._side_stream is None:
            self._side_stream = torch.cuda.Stream(device=self.device, priority=-1)
        return self._side_stream

    def _nb(self, fn, tensors, result):
        cur = torch.cuda.current_stream(self.device)
        side = self.side_stream()
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            fn()
        for t in tensors:
            if t is not None and t.is_cuda:
                t.record_stream(side)
        ev = torch.cuda.Event()
        ev.record(side)
        return DeviceHandle(ev, tuple(tensors) + (result,), self)

    def all_reduce_nb(self, t, op="sum", out=None, scale=None, algo="auto") -> DeviceHandle:
        """Non-blocking ``all_reduce`` on the side stream; returns a DeviceHandle."""
        out_ = t if out is None else out
        return self._nb(lambda: self.all_reduce(t, op, out_, scale, algo), (t, out_), out_)

    def reduce_scatter_nb(self, inp, out, op="sum", scale=None) -> DeviceHandle:
        """Non-blocking ``reduce_scatter`` on the side stream; returns a DeviceHandle."""
        return self._nb(lambda: self.reduce_scatter(inp, out, op, scale), (inp, out), out)

    def all_gather_nb(self, inp, out) -> DeviceHandle:
        """Non-blocking ``all_gather`` on the side stream; returns a DeviceHandle."""
        return self._nb(lambda: self.all_gather(inp, out), (inp, out), out)

    def all_to_all_nb(self, inp, out) -> DeviceHandle:
        """Non-blocking ``all_to_all`` on the side stream; returns a DeviceHandle."""
        return self._nb(lambda: self.all_to_all(inp, out), (inp, out), out)

    def broadcast_nb(self, t, root=0) -> DeviceHandle:
        """Non-blocking ``broadcast`` on the side stream; returns a DeviceHandle."""
        return self._nb(lambda: self.broadcast(t, root), (t,), t)

    def reduce_nb(self, t, root=0, op="sum") -> DeviceHandle:
        """Non-blocking ``reduce`` on the side stream; returns a DeviceHandle."""
        return self._nb(lambda: self.reduce(t, root, op), (t,), t)

    def gather_nb(self, inp, out, root=0) -> DeviceHandle:
        """Non-blocking ``gather`` on the side stream; returns a DeviceHandle."""
        return self._nb(lambda: self.gather(inp, root, out), (inp, out), out)

    def scatter_nb(self, inp, out, root=0) -> DeviceHandle:
        """Non-blocking ``scatter`` on the side stream; returns a DeviceHandle."""
        return self._nb(lambda: self.scatter(inp, root, out), (inp, out), out)

    def scan_nb(self, inp, out, op="sum") -> DeviceHandle:
        """Non-blocking ``scan`` on the side stream; returns a DeviceHandle."""
        return self._nb(lambda: self.scan(inp, op, out), (inp, out), out)

    def exclusive_scan_nb(self, inp, out, op="sum") -> DeviceHandle:
        """Non-blocking ``exclusive_scan`` on the side stream; returns a DeviceHandle."""
        return self._nb(lambda: self.exclusive_scan(inp, op, out), (inp, out), out)

    def barrier_nb(self) -> DeviceHandle:
        """Non-blocking ``barrier`` on the side stream; returns a DeviceHandle."""
        return self._nb(self.barrier, (), None)

    # ----------------------------------------------------------- p2p (NCCL)
    def attach_nccl(self, group) -> None:
        """Carry ``send`` / ``recv`` on ``group`` (a
        :class:`~nexar_b200.device.nccl.NcclGroup` over the same ranks in the
        same order) instead of ``torch.distributed``."""
        if group.local_world != self.world_size or group.local_rank != self.rank:
            raise ValueError(f"NCCL group is rank {group.local_rank} of {group.local_world}, "
                             f"this communicator rank {self.rank} of {self.world_size}")
        self._nccl = group

    @property
    def nccl(self):
        """The attached NCCL group (None: p2p goes through ``torch.distributed``)."""
        return self._nccl

    def send(self, t: torch.Tensor, dst: int, group=None):
        """Pipeline-style device send; stays on NCCL p2p (the attached
        ``NcclGroup``, else ``torch.distributed``)."""
        if self._nccl is not None and group is None:
            self._nccl.send(t, dst)
            return
        import torch.distributed as dist
        dist.send(t, dst, group=group)

    def recv(self, t: torch.Tensor, src: int, group=None):
        """Pipeline-style device receive of t from rank src (NCCL p2p)."""
        if self._nccl is not None and group is None:
            self._nccl.recv(t, src)
            return
        import torch.distributed as dist
        dist.recv(t, src, group=group)

    def isend(self, t: torch.Tensor, dst: int, group=None):
        """Non-blocking send: an ``NcclHandle`` with an attached group, else a torch ``Work``."""
        if self._nccl is not None and group is None:
            return self._nccl.send_nb(t, dst)
        import torch.distributed as dist
        return dist.isend(t, dst, group=group)

    def irecv(self, t: torch.Tensor, src: int, group=None):
        """Non-blocking receive: an NcclHandle with an attached group, else a torch Work."""
        if self._nccl is not None and group is None:
            return self._nccl.recv_nb(t, src)
        import torch.distributed as dist
        return dist.irecv(t, src, group=group)

    def send_nb(self, t: torch.Tensor, dst: int):
        """Non-blocking send (see isend)."""
        return self.isend(t, dst)

    def recv_nb(self, t: torch.Tensor, src: int):
        """Non-blocking receive (see irecv)."""
        return self.irecv(t, src)
