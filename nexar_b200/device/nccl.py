"""NCCL communicator for what stays on NCCL: device point-to-point and the comparator.

``NcclGroup`` is one raw NCCL communicator on one GPU and one stream, with the
surface of the reference's ``NcclGroup`` (nexar-nccl/src/group.rs:16-326):
in-place and out-of-place all-reduce, reduce-scatter, all-gather, in-place
broadcast and reduce, stream synchronisation, events for overlap, abort on
drop. It adds ncclSend / ncclRecv, which carry pipeline-style transfers
(every other device collective of this package runs on the peer-memory
kernels of :class:`~nexar_b200.device.DeviceCommunicator`).

Two call styles:
  * raw pointers, counts in elements and nexar ``DataType`` / ``ReduceOp``
    values, on the group's stream (``all_reduce_inplace(ptr, count, dtype, op)``,
    as the reference; the caller orders and synchronises);
  * tensors (``all_reduce(t)``, ``send(t, peer)``, ...), ordered after the
    caller's current stream and before whatever the caller enqueues next, with
    ``*_nb`` variants that return a :class:`NcclHandle`.

The 128-byte NCCL id travels over the nexar control plane, from each node's
lead to its local ranks under tag ``0xACC1_0000 | node_idx``
(nexar-nccl/src/bootstrap.rs:82-118): :func:`form_nccl_group`.
"""
from __future__ import annotations

import functools
import glob
import os
from typing import Optional

import torch

from ..core import DataType, NexarError, ReduceOp

NCCL_ID_TAG_BASE = 0xACC1_0000  # nexar-nccl/src/bootstrap.rs: tag 0xACC1_0000 | node_idx
UNIQUE_ID_BYTES = 128


# ------------------------------------------------------------------- errors
class NcclCommError(NexarError):
    """Errors of the NCCL layer (nexar-nccl/src/error.rs:7-34)."""


class NcclError(NcclCommError):
    """An NCCL call returned an error."""


class CudaDriverError(NcclCommError):
    """A CUDA stream or event call failed."""


class TopologyError(NcclCommError):
    """The node layout cannot carry the request."""


class InvalidRank(NcclCommError):
    """A rank outside ``[0, world_size)``."""


class NotLeadRank(NcclCommError):
    """A lead-only operation on a rank that does not lead its node."""


class BootstrapError(NcclCommError):
    """The NCCL id exchange or communicator creation failed."""


def _translate(e: RuntimeError) -> NcclCommError:
    msg = str(e)
    kind, _, rest = msg.partition(": ")
    if kind == "nccl":
        return NcclError(rest)
    if kind == "cuda":
        return CudaDriverError(rest)
    if kind == "usage" and rest.startswith("invalid rank"):
        return InvalidRank(rest)
    if kind == "usage":
        return NcclCommError(rest)
    return NcclCommError(msg)


def _native_call(fn, *args):
    try:
        return fn(*args)
    except NcclCommError:
        raise
    except RuntimeError as e:
        raise _translate(e) from None


@functools.lru_cache(maxsize=None)
def _lib():
    """The ``nexar_b200._nccl`` extension with libnccl resolved."""
    try:
        from .. import _nccl  # type: ignore
    except ImportError as e:
        raise RuntimeError("nexar_b200._nccl is not built; run `python setup.py build_ext --inplace`") from e
    _native_call(_nccl.load, _library_path())
    return _nccl


def _library_path() -> str:
    """libnccl of the NCCL wheel that torch uses ('' lets the loader search)."""
    try:
        import nvidia  # type: ignore
        for base in nvidia.__path__:
            hits = sorted(glob.glob(os.path.join(base, "nccl", "lib", "libnccl.so*")))
            if hits:
                return hits[0]
    except ImportError:
        pass
    return ""


def version() -> int:
    """NCCL version code of the loaded library (e.g. 22809 for 2.28.9)."""
    return int(_native_call(_lib().version))


# ------------------------------------------------------------------- mapping
def to_nccl_dtype(dtype) -> int:
    """``ncclDataType_t`` value for a nexar DataType (nexar-nccl/src/types.rs:5-19)."""
    dt = DataType.from_torch(dtype) if isinstance(dtype, torch.dtype) else DataType(int(dtype))
    return int(_native_call(_lib().nccl_dtype, int(dt)))


def to_nccl_op(op) -> int:
    """``ncclRedOp_t`` value for a nexar ReduceOp (nexar-nccl/src/types.rs:21-28)."""
    return int(_native_call(_lib().nccl_op, int(ReduceOp.parse(op))))


# ------------------------------------------------------------------- ids
def unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes); the lead creates one per group."""
    return bytes(_native_call(_lib().unique_id))


def id_to_bytes(uid: bytes) -> bytes:
    """Serialised form of an id: its 128 bytes (nexar-nccl/src/group.rs: id_to_bytes)."""
    b = bytes(uid)
    if len(b) != UNIQUE_ID_BYTES:
        raise BootstrapError(f"an NCCL id is {UNIQUE_ID_BYTES} bytes, got {len(b)}")
    return b


def id_from_bytes(data: bytes) -> bytes:
    """Inverse of :func:`id_to_bytes`; rejects anything but 128 bytes."""
    return id_to_bytes(data)


# ------------------------------------------------------------------- handle
class NcclHandle:
    """Completion of a non-blocking NCCL operation. ``wait()`` orders the
    caller's current stream after it (no host block); ``synchronize()`` blocks
    the host; ``is_finished()`` polls.

    The handle holds the operation's tensors. The caching allocator may hand
    their memory out again on the caller's stream once they are freed, so the
    caller's stream is ordered after the operation (an event wait) before the
    handle lets them go, also when it is dropped without ``wait()``. No
    ``record_stream`` ties them to the group's own stream, which a torn-down
    group destroys."""

    def __init__(self, group: "NcclGroup", event: torch.cuda.Event, keep: tuple, stream: torch.cuda.Stream):
        self._group, self._event, self._keep, self._stream = group, event, keep, stream
        self._ordered = False

    def wait(self):
        self._stream.wait_event(self._event)
        self._ordered = True
        return self._keep[-1] if self._keep else None

    def __del__(self):
        try:
            if not self._ordered and self._keep:
                self._stream.wait_event(self._event)
        except Exception:  # noqa: BLE001  (interpreter teardown)
            pass

    def synchronize(self):
        """Block the host until the operation has finished; raises if the communicator reports an error."""
        self._event.synchronize()
        st = self._group.async_error()
        if st != 0:
            raise NcclError(f"communicator reports asynchronous error {st}")
        return self._keep[-1] if self._keep else None

    def is_finished(self) -> bool:
        return self._event.query()


def _ptr(t: torch.Tensor) -> int:
    if not t.is_cuda:
        raise NcclCommError("NCCL operations take CUDA tensors")
    if not t.is_contiguous():
        raise NcclCommError("NCCL operations take contiguous tensors")
    return t.data_ptr()


# ------------------------------------------------------------------- group
class NcclGroup:
    """One NCCL communicator over ``local_world`` GPUs (one rank per GPU).

    Every rank constructs it with the same ``uid`` (from :func:`unique_id` on
    one rank, shared out of band) and its own ``local_rank``; construction
    blocks until all ranks have joined. ``stream`` (a ``torch.cuda.Stream``
    other than the legacy default stream) is used as is; by default the group
    makes a private non-blocking stream.
    """

    def __init__(self, local_rank: int, local_world: int, uid: bytes, device: Optional[int] = None,
                 stream: Optional[torch.cuda.Stream] = None):
        lib = _lib()
        dev = torch.cuda.current_device() if device is None else int(device)
        handle = 0 if stream is None else int(stream.cuda_stream)
        if stream is not None and handle == 0:
            # the legacy default stream has handle 0, which the native group reads as "make a private stream"
            raise NcclCommError("NcclGroup needs a non-default stream (the legacy default stream has no handle)")
        try:
            self._g = lib.NcclGroup(int(local_rank), int(local_world), id_to_bytes(uid), dev, handle)
        except RuntimeError as e:
            err = _translate(e)
            if isinstance(err, NcclError):
                raise BootstrapError(str(err)) from None
            raise err from None
        self._stream = stream if stream is not None else torch.cuda.ExternalStream(self._g.stream, device=dev)

    @classmethod
    def from_torch(cls, group=None, device: Optional[int] = None,
                   stream: Optional[torch.cuda.Stream] = None) -> "NcclGroup":
        """Build over an initialised ``torch.distributed`` process group (its
        rank 0 creates the id; collective over the group)."""
        import torch.distributed as dist
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        holder = [unique_id() if rank == 0 else None]
        dist.broadcast_object_list(holder, src=dist.get_global_rank(group, 0) if group is not None else 0,
                                   group=group)
        return cls(rank, world, holder[0], device=device, stream=stream)

    # reference-style constructor name
    @classmethod
    def init(cls, stream: Optional[torch.cuda.Stream], local_rank: int, local_world: int, uid: bytes,
             device: Optional[int] = None) -> "NcclGroup":
        return cls(local_rank, local_world, uid, device=device, stream=stream)

    # ------------------------------------------------------------ facade
    @property
    def local_rank(self) -> int:
        return self._g.local_rank

    @property
    def local_world(self) -> int:
        return self._g.local_world

    @property
    def device(self) -> int:
        return self._g.device

    @property
    def stream(self) -> torch.cuda.Stream:
        return self._stream

    @property
    def closed(self) -> bool:
        return self._g.closed

    # ------------------------------------------------------------ raw pointers (group stream)
    def allreduce_inplace(self, ptr: int, count: int, dtype, op=ReduceOp.Sum):
        """ncclAllReduce in place on `count` elements at `ptr` (group stream)."""
        _native_call(self._g.all_reduce_inplace, int(ptr), int(count), int(DataType(dtype)), int(ReduceOp.parse(op)))

    def allreduce(self, send_ptr: int, recv_ptr: int, count: int, dtype, op=ReduceOp.Sum):
        """ncclAllReduce from send_ptr into recv_ptr (group stream)."""
        _native_call(self._g.all_reduce, int(send_ptr), int(recv_ptr), int(count), int(DataType(dtype)),
                     int(ReduceOp.parse(op)))

    def reduce_scatter_ptr(self, send_ptr: int, recv_ptr: int, recv_count: int, dtype, op=ReduceOp.Sum):
        """ncclReduceScatter: recv_count elements per rank; rank r receives chunk r."""
        _native_call(self._g.reduce_scatter, int(send_ptr), int(recv_ptr), int(recv_count), int(DataType(dtype)),
                     int(ReduceOp.parse(op)))

    def allgather(self, send_ptr: int, recv_ptr: int, send_count: int, dtype):
        """ncclAllGather: send_count elements per rank into recv in rank order."""
        _native_call(self._g.all_gather, int(send_ptr), int(recv_ptr), int(send_count), int(DataType(dtype)))

    def broadcast_inplace(self, ptr: int, count: int, dtype, root: int):
        """ncclBroadcast in place from `root`."""
        _native_call(self._g.broadcast_inplace, int(ptr), int(count), int(DataType(dtype)), int(root))

    def reduce_inplace(self, ptr: int, count: int, dtype, op, root: int):
        """ncclReduce in place onto `root`."""
        _native_call(self._g.reduce_inplace, int(ptr), int(count), int(DataType(dtype)), int(ReduceOp.parse(op)),
                     int(root))

    def send_ptr(self, ptr: int, count: int, dtype, peer: int):
        """ncclSend of `count` elements to `peer` (group stream)."""
        _native_call(self._g.send, int(ptr), int(count), int(DataType(dtype)), int(peer))

    def recv_ptr(self, ptr: int, count: int, dtype, peer: int):
        """ncclRecv of `count` elements from `peer` (group stream)."""
        _native_call(self._g.recv, int(ptr), int(count), int(DataType(dtype)), int(peer))

    def synchronize(self):
        """Block the host until the group's stream has drained."""
        _native_call(self._g.synchronize)

    def create_event(self) -> int:
        """A CUDA event (no timing) on the group's device; returns its handle."""
        return int(_native_call(self._g.create_event))

    def record_event(self, event: int):
        """Record `event` on the group's stream."""
        _native_call(self._g.record_event, int(event))

    def stream_wait_event(self, event: int, stream: Optional[torch.cuda.Stream] = None):
        """Make ``stream`` (default: this group's stream) wait for ``event``."""
        _native_call(self._g.stream_wait_event, 0 if stream is None else int(stream.cuda_stream), int(event))

    def event_query(self, event: int) -> bool:
        """Whether `event` has completed."""
        return bool(_native_call(self._g.event_query, int(event)))

    def destroy_event(self, event: int):
        """Destroy an event made by create_event."""
        _native_call(self._g.destroy_event, int(event))

    def async_error(self) -> int:
        """The communicator's asynchronous error state (0 while healthy)."""
        return int(_native_call(self._g.async_error))

    def abort(self):
        """Tear down without waiting on peers (the reference's drop)."""
        _native_call(self._g.abort)

    def destroy(self):
        """Orderly teardown after this rank's last operation."""
        _native_call(self._g.destroy)

    # ------------------------------------------------------------ tensors (caller's stream order)
    def _run(self, fn, tensors, result, blocking: bool):
        cur = torch.cuda.current_stream(self.device)
        self._stream.wait_stream(cur)
        fn()
        ev = torch.cuda.Event()
        ev.record(self._stream)
        h = NcclHandle(self, ev, tuple(tensors) + (result,), cur)
        if blocking:
            h.wait()
            return result
        return h

    def all_reduce(self, t: torch.Tensor, op="sum", out: Optional[torch.Tensor] = None, blocking: bool = True):
        """All-reduce of t (into out) ordered after the caller's current stream."""
        out_ = t if out is None else out
        if out_.numel() != t.numel() or out_.dtype != t.dtype:
            raise NcclCommError("all_reduce: out must match the input's size and dtype")
        dt = DataType.from_torch(t.dtype)
        return self._run(lambda: self.allreduce(_ptr(t), _ptr(out_), t.numel(), dt, op), (t, out_), out_, blocking)

    def reduce_scatter(self, inp: torch.Tensor, out: torch.Tensor, op="sum", blocking: bool = True):
        """Rank r's out = op over ranks of chunk r of inp."""
        if inp.numel() != out.numel() * self.local_world or inp.dtype != out.dtype:
            raise NcclCommError("reduce_scatter: input must hold world_size x out elements of out's dtype")
        dt = DataType.from_torch(out.dtype)
        return self._run(lambda: self.reduce_scatter_ptr(_ptr(inp), _ptr(out), out.numel(), dt, op),
                         (inp, out), out, blocking)

    def all_gather(self, inp: torch.Tensor, out: torch.Tensor, blocking: bool = True):
        """out (world x inp) = every rank's inp in rank order."""
        if out.numel() != inp.numel() * self.local_world or inp.dtype != out.dtype:
            raise NcclCommError("all_gather: out must hold world_size x input elements of the input's dtype")
        dt = DataType.from_torch(inp.dtype)
        return self._run(lambda: self.allgather(_ptr(inp), _ptr(out), inp.numel(), dt), (inp, out), out, blocking)

    def broadcast(self, t: torch.Tensor, root: int = 0, blocking: bool = True):
        """t on every rank = the root's t."""
        dt = DataType.from_torch(t.dtype)
        return self._run(lambda: self.broadcast_inplace(_ptr(t), t.numel(), dt, root), (t,), t, blocking)

    def reduce(self, t: torch.Tensor, root: int = 0, op="sum", blocking: bool = True):
        """The root's t = op over all ranks' t."""
        dt = DataType.from_torch(t.dtype)
        return self._run(lambda: self.reduce_inplace(_ptr(t), t.numel(), dt, op, root), (t,), t, blocking)

    def send(self, t: torch.Tensor, peer: int, blocking: bool = True):
        """Send t to `peer` (ordered after the caller's current stream)."""
        dt = DataType.from_torch(t.dtype)
        return self._run(lambda: self.send_ptr(_ptr(t), t.numel(), dt, peer), (t,), t, blocking)

    def recv(self, t: torch.Tensor, peer: int, blocking: bool = True):
        """Receive t from `peer`."""
        dt = DataType.from_torch(t.dtype)
        return self._run(lambda: self.recv_ptr(_ptr(t), t.numel(), dt, peer), (t,), t, blocking)

    def send_recv(self, send_t: torch.Tensor, send_peer: int, recv_t: torch.Tensor, recv_peer: int,
                  blocking: bool = True):
        """Send and receive as one NCCL group (ring shifts and pipeline
        exchanges cannot deadlock on call order)."""
        if send_t.dtype != recv_t.dtype:
            raise NcclCommError("send_recv: both tensors must have the same dtype")
        dt = int(DataType.from_torch(send_t.dtype))
        return self._run(lambda: _native_call(self._g.send_recv, _ptr(send_t), send_t.numel(), int(send_peer),
                                              _ptr(recv_t), recv_t.numel(), int(recv_peer), dt),
                         (send_t, recv_t), recv_t, blocking)

    def all_reduce_nb(self, t, op="sum", out=None) -> NcclHandle:
        """Non-blocking all_reduce; returns an NcclHandle."""
        return self.all_reduce(t, op, out, blocking=False)

    def send_nb(self, t, peer) -> NcclHandle:
        """Non-blocking send; returns an NcclHandle."""
        return self.send(t, peer, blocking=False)

    def recv_nb(self, t, peer) -> NcclHandle:
        """Non-blocking receive; returns an NcclHandle."""
        return self.recv(t, peer, blocking=False)

    def send_recv_nb(self, send_t, send_peer, recv_t, recv_peer) -> NcclHandle:
        """Non-blocking send_recv; returns an NcclHandle."""
        return self.send_recv(send_t, send_peer, recv_t, recv_peer, blocking=False)


# ------------------------------------------------------------------- bootstrap
def exchange_nccl_id(client, local_ranks, node_idx: int, lead: int) -> bytes:
    """Share one NCCL id among ``local_ranks`` (global ranks of ``client``):
    the lead creates it and sends it to every other local rank with tag
    ``0xACC1_0000 | node_idx``; the others receive it from the lead
    (nexar-nccl/src/bootstrap.rs:79-118)."""
    import numpy as np
    tag = NCCL_ID_TAG_BASE | (int(node_idx) & 0xFFFF)
    if client.rank == lead:
        uid = unique_id()
        buf = np.frombuffer(uid, dtype=np.uint8).copy()
        for r in local_ranks:
            if r != lead:
                client.send(buf.ctypes.data, buf.nbytes, r, tag)
        return uid
    buf = np.empty(UNIQUE_ID_BYTES, dtype=np.uint8)
    client.recv(buf.ctypes.data, buf.nbytes, lead, tag)
    try:
        return id_from_bytes(buf.tobytes())
    except BootstrapError as e:
        raise BootstrapError(f"NCCL id from rank {lead}: {e}") from None


def form_nccl_group(client, topology=None, device: Optional[int] = None,
                    stream: Optional[torch.cuda.Stream] = None) -> NcclGroup:
    """NCCL communicator over the ranks of this rank's node (collective over
    ``client``): topology from host names (or ``topology``), the id from the
    node's lead, then ``ncclCommInitRank`` (nexar-nccl/src/bootstrap.rs:24-74)."""
    if topology is None:
        from ..parallel.hierarchical import discover_topology
        topology = discover_topology(client)
    t = topology
    if t.rank != client.rank:
        raise TopologyError(f"topology is for rank {t.rank}, client is rank {client.rank}")
    uid = exchange_nccl_id(client, t.local_ranks, t.node_idx, t.lead)
    return NcclGroup(t.local_rank, t.local_world_size, uid, device=device, stream=stream)


def nccl_group_for_client(client, device: Optional[int] = None,
                          stream: Optional[torch.cuda.Stream] = None) -> NcclGroup:
    """NCCL communicator over every rank of ``client`` in its rank order
    (collective over ``client``; rank 0 creates the id). This is the group a
    :class:`~nexar_b200.device.DeviceCommunicator` built from the same client
    takes for device send / recv."""
    uid = exchange_nccl_id(client, list(range(client.world_size)), 0, 0)
    return NcclGroup(client.rank, client.world_size, uid, device=device, stream=stream)
