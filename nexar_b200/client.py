"""NexarClient: the host communicator (C++ runtime) with nexar's public API.

Bootstrap (nexar/src/client/bootstrap.rs): ``NexarClient.bootstrap_local(n)``
builds n ranks in this process over loopback TCP through a real seed/worker
exchange; ``NexarClient.bootstrap(seed_addr)`` joins a multi-process cluster
(one process per rank / GPU), with ``SeedNode`` hosting discovery.

Every collective of the reference is available with the reference's pointer
signature (``all_reduce(ptr, count, dtype, op)``; ``count`` is elements per
rank-chunk for all_gather / reduce_scatter / all_to_all / gather / scatter and
total elements otherwise), plus ``*_host`` helpers that take numpy arrays or
CPU torch tensors, ``*_device`` helpers that take CUDA tensors and run the
sm_100a peer-memory kernels (the CUDA DeviceAdapter), and ``*_nb`` variants
returning a :class:`CollectiveHandle`.
"""
from __future__ import annotations

from typing import Iterable, List, Optional, Sequence, Tuple

from . import _native
from .core import DataType, Priority, ReduceOp

_H = None


def _h():
    global _H
    if _H is None:
        _H = _native.host()
    return _H


def Config(**kw):
    """NexarConfig with the reference's defaults; override fields by keyword."""
    c = _h().Config()
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def config_from_env():
    return _h().Config.from_env()


def CpuAdapter():
    """Host buffers used in place (nexar/src/device/cpu.rs)."""
    return _h().CpuAdapter()


def CudaAdapter():
    """CUDA device buffers staged through host memory for host collectives and
    p2p (nexar-rdma/src/cuda_adapter.rs): the cross-host path for device
    pointers. On one box, ``attach_device`` runs device collectives on the
    peer-memory kernels instead."""
    return _h().CudaAdapter()


def _pool(p):
    """A native BufferPool from None / a PoolProfile / a pool object."""
    if p is None:
        return None
    if isinstance(p, _h().BufferPool):
        return p
    from .memory import PoolProfile
    if isinstance(p, (PoolProfile, int)):
        return _h().BufferPool.with_profile(int(p))
    raise TypeError(f"not a BufferPool or PoolProfile: {p!r}")


def _adapter(a):
    """A native adapter from None / "cpu" / "cuda" / an adapter object."""
    if a is None or a == "cpu":
        return CpuAdapter()
    if a == "cuda":
        return CudaAdapter()
    if isinstance(a, _h().DeviceAdapter):
        if type(a).__module__ != _h().__name__:
            # A Python subclass: the native clients keep only the C++ part
            # alive, so its Python half (the overrides) is kept here for the
            # life of the process.
            _PY_ADAPTERS.append(a)
        return a
    raise TypeError(f"not a DeviceAdapter: {a!r}")


_PY_ADAPTERS: list = []


def __getattr__(name):
    # DeviceAdapter: subclass it in Python to bring another memory space
    # (override name, stage_for_send, receive_to_device, reduce_inplace and,
    # for plain host memory, host_addressable). Resolved lazily so importing
    # this module does not load the extension.
    if name == "DeviceAdapter":
        return _h().DeviceAdapter
    raise AttributeError(name)


_NP_CODES = None


def _np_codes():
    """numpy dtype -> DataType (bf16 travels as raw uint16 bits)."""
    global _NP_CODES
    if _NP_CODES is None:
        import numpy as np
        _NP_CODES = {np.dtype(np.float32): DataType.F32, np.dtype(np.float64): DataType.F64,
                     np.dtype(np.float16): DataType.F16, np.dtype(np.int8): DataType.I8,
                     np.dtype(np.int32): DataType.I32, np.dtype(np.int64): DataType.I64,
                     np.dtype(np.uint8): DataType.U8, np.dtype(np.uint32): DataType.U32,
                     np.dtype(np.uint64): DataType.U64, np.dtype(np.uint16): DataType.BF16}
    return _NP_CODES


def _buf(x, host_only: bool = False) -> Tuple[int, int, DataType]:
    """(address, numel, dtype) of a contiguous numpy array or torch tensor
    (host_only: reject CUDA tensors)."""
    iface = getattr(x, "__array_interface__", None)
    if iface is not None and not hasattr(x, "data_ptr"):  # numpy array: the fast path
        if not x.flags["C_CONTIGUOUS"]:
            raise ValueError("array must be C-contiguous")
        try:
            return iface["data"][0], x.size, _np_codes()[x.dtype]
        except KeyError:
            raise TypeError(f"unsupported array dtype {x.dtype}") from None
    import torch
    if isinstance(x, torch.Tensor):
        if host_only and x.is_cuda:
            raise TypeError("*_host calls take host buffers; use the *_device call for CUDA tensors")
        if not x.is_contiguous():
            raise ValueError("tensor must be contiguous")
        return x.data_ptr(), x.numel(), DataType.from_torch(x.dtype)
    raise TypeError(f"unsupported buffer type {type(x)}")


def _host_buf(x) -> Tuple[int, int, DataType]:
    """``_buf`` for the typed ``*_host`` calls: host memory only."""
    return _buf(x, host_only=True)


class CollectiveHandle:
    """Handle of a non-blocking collective (nexar/src/collective/handle.rs)."""

    def __init__(self, native, keep=()):
        self._h = native
        self._keep = keep

    def wait(self):
        self._h.wait()

    def is_finished(self) -> bool:
        return self._h.is_finished()


class CollectiveGroup:
    """Wait for several handles; raises the first error (handle.rs:50-91)."""

    def __init__(self):
        self._handles: List[CollectiveHandle] = []

    def push(self, h: CollectiveHandle):
        self._handles.append(h)

    def wait_all(self):
        first = None
        for h in self._handles:
            try:
                h.wait()
            except Exception as e:  # noqa: BLE001
                first = first or e
        if first is not None:
            raise first

    def __len__(self):
        return len(self._handles)


class NexarClient:
    """A rank of a communicator (wraps the C++ ``NexarClient``)."""

    def __init__(self, native, device_comm=None):
        self._c = native
        self._device = device_comm

    # ------------------------------------------------------------ bootstrap
    @staticmethod
    def bootstrap_local(world_size: int, config=None, adapter=None, pool=None) -> List["NexarClient"]:
        """``world_size`` ranks in this process over loopback (nexar/src/client/bootstrap.rs:22).
        ``adapter`` ("cpu", "cuda" or a DeviceAdapter) is shared by every rank.
        ``pool``: a :class:`~nexar_b200.memory.BufferPool` (or a ``PoolProfile``)
        whose tiers serve every rank's receive buffers (the reference's
        ``new_with_pool`` / ``new_with_profile``); default one Training-profile
        pool per rank."""
        cfg = config if config is not None else _h().Config()
        ad = _adapter(adapter)
        natives = _h().NexarClient.bootstrap_local(world_size, cfg, _pool(pool))
        for c in natives:
            c.set_adapter(ad)
        return [NexarClient(c) for c in natives]

    bootstrap_local_with_config = bootstrap_local

    @staticmethod
    def bootstrap(seed_addr: str, token: Optional[bytes] = None, config=None,
                  bind_host: str = "127.0.0.1", adapter=None, pool=None) -> "NexarClient":
        """Join a cluster through the seed at `seed_addr` (one process per rank);
        ``pool`` as in :meth:`bootstrap_local`."""
        cfg = config if config is not None else _h().Config.from_env()
        c = _h().NexarClient.bootstrap_worker(seed_addr, token, cfg, bind_host, _pool(pool))
        c.set_adapter(_adapter(adapter))
        return NexarClient(c)

    @staticmethod
    def from_worker(info, config=None, adapter=None, pool=None) -> "NexarClient":
        """Build the mesh from a ``WorkerNode.connect`` result (the second half
        of ``bootstrap``); ``config`` must match the cluster's (TLS, topology)."""
        cfg = config if config is not None else _h().Config.from_env()
        c = _h().NexarClient.from_worker_info(info, cfg, _pool(pool))
        c.set_adapter(_adapter(adapter))
        return NexarClient(c)

    @staticmethod
    def bootstrap_elastic(initial_world: int, min_world: int = 1, max_world: int = 0, config=None,
                          checkpoint_timeout_s: float = 60.0, elastic: Optional["ElasticConfig"] = None,
                          adapter=None) -> "ElasticBootstrap":
        """In-process cluster with elastic scaling (nexar/src/client/bootstrap.rs:41).

        A local seed forms ``initial_world`` ranks, then keeps accepting joiners
        (``ElasticManager.join(seed_addr, ...)`` from any process) up to
        ``max_world`` (0 = unbounded); each rank gets an ElasticManager (rank 0's
        owns the seed) whose ``elastic_checkpoint()`` admits joiners and applies
        ``remove_node`` requests at a step boundary.
        """
        import threading
        if elastic is not None:
            min_world, max_world = elastic.min_world_size, elastic.max_world_size
            checkpoint_timeout_s = elastic.checkpoint_timeout_s
        H = _h()
        cfg = config if config is not None else H.Config()
        ad = _adapter(adapter)
        seed = H.SeedNode.bind_local(bool(getattr(cfg, "tls", False)))
        natives = [None] * initial_world
        errs = []

        def boot(i):
            try:
                natives[i] = H.NexarClient.bootstrap_worker(seed.local_addr(), None, cfg, "127.0.0.1")
            except Exception as e:  # noqa: BLE001
                errs.append(e)
        ts = [threading.Thread(target=boot, args=(i,)) for i in range(initial_world)]
        [t.start() for t in ts]
        seed.form_cluster(initial_world)
        [t.join() for t in ts]
        if errs:
            raise errs[0]
        natives.sort(key=lambda c: c.rank)
        for c in natives:
            c.set_adapter(ad)
        seed.accept_elastic(max_world)
        mgrs = [H.ElasticManager(c, seed if c.rank == 0 else None, min_world, max_world, checkpoint_timeout_s)
                for c in natives]
        return ElasticBootstrap(seed, [NexarClient(c) for c in natives], mgrs)

    # ------------------------------------------------------------ identity
    @property
    def rank(self) -> int:
        return self._c.rank

    @property
    def world_size(self) -> int:
        return self._c.world_size

    @property
    def comm_id(self) -> int:
        return self._c.comm_id

    @property
    def native(self):
        return self._c

    def config(self):
        """The NexarConfig this communicator was built with."""
        return self._c.config()

    def has_direct_peer(self, rank: int) -> bool:
        """Whether `rank` has a direct connection (False when a sparse topology relays to it)."""
        return self._c.has_direct_peer(rank)

    def is_sparse(self) -> bool:
        """Whether this communicator runs on a sparse topology (k-regular or hypercube)."""
        return self._c.is_sparse()

    def adapter(self) -> str:
        """Name of the memory adapter in use ("cuda" when a device communicator is attached)."""
        return "cuda" if self._device is not None else self._c.adapter_name

    def device_adapter(self):
        """The native DeviceAdapter host collectives and p2p stage through."""
        return self._c.adapter()

    def set_adapter(self, adapter):
        """Replace the adapter ("cpu", "cuda" or a DeviceAdapter) before the
        operations that should use it; split / rebuild children inherit it."""
        self._c.set_adapter(_adapter(adapter))

    # ------------------------------------------------------------ p2p
    @property
    def pool(self):
        """The buffer pool that serves this client's receive buffers."""
        return self._c.pool

    def send(self, ptr: int, size: int, dest: int, tag: int):
        """Send `size` bytes at `ptr` to rank `dest` under `tag` (staged through the adapter for non-host memory)."""
        self._c.send(ptr, size, dest, tag)

    def recv(self, ptr: int, size: int, src: int, tag: int):
        """Receive the oldest message from `src` with `tag` into `size` bytes at `ptr`; the size must match."""
        self._c.recv(ptr, size, src, tag)

    def send_iov(self, iov: Sequence[Tuple[int, int]], dest: int, tag: int):
        """Send the (ptr, len) regions back to back as one tagged message."""
        self._c.send_iov(list(iov), dest, tag)

    def recv_iov(self, iov: Sequence[Tuple[int, int]], src: int, tag: int):
        """Receive one tagged message and scatter it over the (ptr, len) regions."""
        self._c.recv_iov(list(iov), src, tag)

    def send_bytes(self, dest: int, data: bytes):
        """Send a byte string to `dest` on this communicator's raw lane."""
        self._c.send_bytes(dest, data)

    def recv_bytes(self, src: int) -> bytes:
        """Receive the next byte string from `src` on the raw lane."""
        return self._c.recv_bytes(src)

    def send_bytes_tagged(self, dest: int, tag: int, data: bytes):
        """Send a byte string to `dest` under a 64-bit tag."""
        self._c.send_bytes_tagged(dest, tag, data)

    def recv_bytes_tagged(self, src: int, tag: int, timeout_s: float = -1.0) -> bytes:
        """Receive the byte string from `src` with `tag` (timeout_s < 0: the collective timeout)."""
        return self._c.recv_bytes_tagged(src, tag, timeout_s)

    # ------------------------------------------------------------ rpc
    def register_rpc(self, fn_id: int, handler):
        """handler(bytes) -> bytes, served by ``serve_rpc_once`` / ``start_rpc_server``."""
        self._c.register_rpc(fn_id, handler)

    def rpc(self, target: int, fn_id: int, args: bytes, timeout_s: float = -1.0) -> bytes:
        """Call function `fn_id` on rank `target` with `args`; returns its reply (timeout_s < 0: the RPC timeout)."""
        return self._c.rpc(target, fn_id, args, timeout_s)

    rpc_with_timeout = rpc

    def recv_rpc_request(self, src: int, timeout_s: float = -1.0) -> dict:
        """Take the next RPC request from `src` (fields: req_id, fn_id, payload)."""
        return self._c.recv_rpc_request(src, timeout_s)

    def serve_rpc_once(self, src: int, timeout_s: float = -1.0):
        """Serve one RPC request from `src` with the registered handlers."""
        self._c.serve_rpc_once(src, timeout_s)

    def start_rpc_server(self):
        """Serve RPC requests from every peer on a background thread."""
        self._c.start_rpc_server()

    def stop_rpc_server(self):
        """Stop the background RPC server."""
        self._c.stop_rpc_server()

    def rpc_dispatcher(self) -> "RpcDispatcher":
        """The dispatcher that serves this client's registered RPC handlers."""
        return RpcDispatcher(self)

    # ------------------------------------------------------------ peers / raw messages
    def peer(self, rank: int) -> dict:
        """Direct connection to ``rank``: {rank, mesh_rank, alive, encrypted}; UnknownPeer if none."""
        return self._c.peer_info(rank)

    def send_message_to(self, dest: int, tag: int, payload: bytes, priority=Priority.Critical):
        """One framed data message to ``dest`` (root communicator); see ``recv_message_from``."""
        self._c.send_message_to(dest, tag, payload, int(priority))

    def recv_message_from(self, src: int, tag: int, timeout_s: float = -1.0) -> bytes:
        """Receive the payload that `src` sent with ``send_message_to`` under `tag`."""
        return self._c.recv_message_from(src, tag, timeout_s)

    # ------------------------------------------------------------ collectives (pointer API)
    def all_reduce(self, ptr: int, count: int, dtype, op=ReduceOp.Sum):
        """In place: `count` elements at `ptr` become op over all ranks."""
        self._c.all_reduce(ptr, count, int(dtype), int(ReduceOp.parse(op)))

    def all_reduce_rs_ag(self, ptr: int, count: int, dtype, op=ReduceOp.Sum):
        """All-reduce as reduce-scatter then all-gather (uneven counts allowed)."""
        self._c.all_reduce_rs_ag(ptr, count, int(dtype), int(ReduceOp.parse(op)))

    def all_reduce_bucketed(self, entries: Sequence[Tuple[int, int]], dtype, op=ReduceOp.Sum):
        """One all-reduce over several (ptr, count) regions packed together."""
        self._c.all_reduce_bucketed(list(entries), int(dtype), int(ReduceOp.parse(op)))

    def all_reduce_compressed(self, ptr: int, count: int, dtype, op, compressor, residual_ptr: int):
        """All-reduce of compressed contributions (compressor with error feedback in `residual`)."""
        self._c.all_reduce_compressed(ptr, count, int(dtype), int(ReduceOp.parse(op)), compressor, residual_ptr)

    def broadcast(self, ptr: int, count: int, dtype, root: int):
        """In place: every rank's `count` elements at `ptr` become the root's."""
        self._c.broadcast(ptr, count, int(dtype), root)

    def all_gather(self, send_ptr: int, recv_ptr: int, count: int, dtype):
        """recv (count x world) = every rank's send (count) in rank order."""
        self._c.all_gather(send_ptr, recv_ptr, count, int(dtype))

    def reduce_scatter(self, send_ptr: int, recv_ptr: int, count: int, dtype, op=ReduceOp.Sum):
        """recv (count) on rank r = op over ranks of chunk r of send (count x world)."""
        self._c.reduce_scatter(send_ptr, recv_ptr, count, int(dtype), int(ReduceOp.parse(op)))

    def reduce(self, ptr: int, count: int, dtype, op, root: int):
        """In place: the root's buffer becomes op over all ranks (other ranks keep partial results)."""
        self._c.reduce(ptr, count, int(dtype), int(ReduceOp.parse(op)), root)

    def all_to_all(self, send_ptr: int, recv_ptr: int, count: int, dtype):
        """recv chunk q (count) = chunk r of rank q's send (count x world)."""
        self._c.all_to_all(send_ptr, recv_ptr, count, int(dtype))

    def gather(self, send_ptr: int, recv_ptr: int, count: int, dtype, root: int):
        """The root's recv (count x world) receives every rank's send (count) in rank order."""
        self._c.gather(send_ptr, recv_ptr, count, int(dtype), root)

    def scatter(self, send_ptr: int, recv_ptr: int, count: int, dtype, root: int):
        """recv (count) on rank r = chunk r of the root's send (count x world)."""
        self._c.scatter(send_ptr, recv_ptr, count, int(dtype), root)

    def scan(self, ptr: int, count: int, dtype, op=ReduceOp.Sum):
        """In place: rank r holds op over ranks 0..r."""
        self._c.scan(ptr, count, int(dtype), int(ReduceOp.parse(op)))

    def exclusive_scan(self, ptr: int, count: int, dtype, op=ReduceOp.Sum):
        """In place: rank r holds op over ranks 0..r-1 (the identity on rank 0)."""
        self._c.exclusive_scan(ptr, count, int(dtype), int(ReduceOp.parse(op)))

    def barrier(self, timeout_s: Optional[float] = None):
        """Return once every rank of this communicator has entered the barrier."""
        if timeout_s is None:
            self._c.barrier()
        else:
            self._c.barrier_with_timeout(timeout_s)

    # ------------------------------------------------------------ non-blocking
    def all_reduce_nb(self, ptr: int, count: int, dtype, op=ReduceOp.Sum) -> CollectiveHandle:
        """Non-blocking ``all_reduce``: starts it on a worker thread and returns a CollectiveHandle."""
        return CollectiveHandle(self._c.all_reduce_nb(ptr, count, int(dtype), int(ReduceOp.parse(op))))

    def _nb(self, op: str, *args) -> CollectiveHandle:
        return CollectiveHandle(self._c.spawn_collective(op, tuple(int(a) for a in args)))

    def broadcast_nb(self, ptr, count, dtype, root):
        """Non-blocking ``broadcast``: starts it on a worker thread and returns a CollectiveHandle."""
        return self._nb("broadcast", ptr, count, dtype, root)

    def all_gather_nb(self, send_ptr, recv_ptr, count, dtype):
        """Non-blocking ``all_gather``: starts it on a worker thread and returns a CollectiveHandle."""
        return self._nb("all_gather", send_ptr, recv_ptr, count, dtype)

    def reduce_scatter_nb(self, send_ptr, recv_ptr, count, dtype, op=ReduceOp.Sum):
        """Non-blocking ``reduce_scatter``: starts it on a worker thread and returns a CollectiveHandle."""
        return self._nb("reduce_scatter", send_ptr, recv_ptr, count, dtype, ReduceOp.parse(op))

    def reduce_nb(self, ptr, count, dtype, op, root):
        """Non-blocking ``reduce``: starts it on a worker thread and returns a CollectiveHandle."""
        return self._nb("reduce", ptr, count, dtype, ReduceOp.parse(op), root)

    def all_to_all_nb(self, send_ptr, recv_ptr, count, dtype):
        """Non-blocking ``all_to_all``: starts it on a worker thread and returns a CollectiveHandle."""
        return self._nb("all_to_all", send_ptr, recv_ptr, count, dtype)

    def gather_nb(self, send_ptr, recv_ptr, count, dtype, root):
        """Non-blocking ``gather``: starts it on a worker thread and returns a CollectiveHandle."""
        return self._nb("gather", send_ptr, recv_ptr, count, dtype, root)

    def scatter_nb(self, send_ptr, recv_ptr, count, dtype, root):
        """Non-blocking ``scatter``: starts it on a worker thread and returns a CollectiveHandle."""
        return self._nb("scatter", send_ptr, recv_ptr, count, dtype, root)

    def scan_nb(self, ptr, count, dtype, op=ReduceOp.Sum):
        """Non-blocking ``scan``: starts it on a worker thread and returns a CollectiveHandle."""
        return self._nb("scan", ptr, count, dtype, ReduceOp.parse(op))

    def exclusive_scan_nb(self, ptr, count, dtype, op=ReduceOp.Sum):
        """Non-blocking ``exclusive_scan``: starts it on a worker thread and returns a CollectiveHandle."""
        return self._nb("exclusive_scan", ptr, count, dtype, ReduceOp.parse(op))

    def all_reduce_rs_ag_nb(self, ptr, count, dtype, op=ReduceOp.Sum):
        """Non-blocking ``all_reduce_rs_ag``: starts it on a worker thread and returns a CollectiveHandle."""
        return self._nb("all_reduce_rs_ag", ptr, count, dtype, ReduceOp.parse(op))

    def barrier_nb(self):
        """Non-blocking ``barrier``: starts it on a worker thread and returns a CollectiveHandle."""
        return self._nb("barrier")

    def all_reduce_bucketed_nb(self, entries: Sequence[Tuple[int, int]], dtype, op=ReduceOp.Sum):
        """Non-blocking ``all_reduce_bucketed``: starts it on a worker thread and returns a CollectiveHandle."""
        return CollectiveHandle(self._c.all_reduce_bucketed_nb(list(entries), int(dtype), int(ReduceOp.parse(op))))

    def all_reduce_compressed_nb(self, ptr: int, count: int, dtype, op, compressor, residual_ptr: int):
        """Non-blocking ``all_reduce_compressed``: starts it on a worker thread and returns a CollectiveHandle."""
        return CollectiveHandle(self._c.all_reduce_compressed_nb(ptr, count, int(dtype), int(ReduceOp.parse(op)),
                                                                 compressor, residual_ptr))

    # ------------------------------------------------------------ typed host helpers
    def all_reduce_host(self, buf, op=ReduceOp.Sum):
        """``all_reduce`` on host buffers (numpy arrays or CPU tensors); returns the result buffer."""
        p, n, dt = _host_buf(buf)
        self.all_reduce(p, n, dt, op)
        return buf

    def all_reduce_rs_ag_host(self, buf, op=ReduceOp.Sum):
        """``all_reduce_rs_ag`` on host buffers (numpy arrays or CPU tensors); returns the result buffer."""
        p, n, dt = _host_buf(buf)
        self.all_reduce_rs_ag(p, n, dt, op)
        return buf

    def broadcast_host(self, buf, root: int):
        """``broadcast`` on host buffers (numpy arrays or CPU tensors); returns the result buffer."""
        p, n, dt = _host_buf(buf)
        self.broadcast(p, n, dt, root)
        return buf

    def all_gather_host(self, send, recv):
        """``all_gather`` on host buffers (numpy arrays or CPU tensors); returns the result buffer."""
        ps, n, dt = _host_buf(send)
        pr, _, _ = _host_buf(recv)
        self.all_gather(ps, pr, n, dt)
        return recv

    def reduce_scatter_host(self, send, recv, op=ReduceOp.Sum):
        """``reduce_scatter`` on host buffers (numpy arrays or CPU tensors); returns the result buffer."""
        ps, _, dt = _host_buf(send)
        pr, n, _ = _host_buf(recv)
        self.reduce_scatter(ps, pr, n, dt, op)
        return recv

    def reduce_host(self, buf, op, root: int):
        """``reduce`` on host buffers (numpy arrays or CPU tensors); returns the result buffer."""
        p, n, dt = _host_buf(buf)
        self.reduce(p, n, dt, op, root)
        return buf

    def all_to_all_host(self, send, recv):
        """``all_to_all`` on host buffers (numpy arrays or CPU tensors); returns the result buffer."""
        ps, n, dt = _host_buf(send)
        pr, _, _ = _host_buf(recv)
        self.all_to_all(ps, pr, n // self.world_size, dt)
        return recv

    def gather_host(self, send, recv, root: int):
        """``gather`` on host buffers (numpy arrays or CPU tensors); returns the result buffer."""
        ps, n, dt = _host_buf(send)
        pr = _host_buf(recv)[0] if recv is not None else 0
        self.gather(ps, pr, n, dt, root)
        return recv

    def scatter_host(self, send, recv, root: int):
        """``scatter`` on host buffers (numpy arrays or CPU tensors); returns the result buffer."""
        pr, n, dt = _host_buf(recv)
        ps = _host_buf(send)[0] if send is not None else 0
        self.scatter(ps, pr, n, dt, root)
        return recv

    def scan_host(self, buf, op=ReduceOp.Sum):
        """``scan`` on host buffers (numpy arrays or CPU tensors); returns the result buffer."""
        p, n, dt = _host_buf(buf)
        self.scan(p, n, dt, op)
        return buf

    def exclusive_scan_host(self, buf, op=ReduceOp.Sum):
        """``exclusive_scan`` on host buffers (numpy arrays or CPU tensors); returns the result buffer."""
        p, n, dt = _host_buf(buf)
        self.exclusive_scan(p, n, dt, op)
        return buf

    def all_reduce_bucketed_host(self, bufs, op=ReduceOp.Sum):
        """``all_reduce_bucketed`` on host buffers (numpy arrays or CPU tensors); returns the result buffer."""
        entries = [_buf(b) for b in bufs]
        dts = {e[2] for e in entries}
        if len(dts) != 1:
            raise ValueError("all buffers of a bucket need one dtype")
        self.all_reduce_bucketed([(p, n) for p, n, _ in entries], dts.pop(), op)
        return bufs

    def all_reduce_compressed_host(self, buf, compressor, residual, op=ReduceOp.Sum):
        """``all_reduce_compressed`` on host buffers (numpy arrays or CPU tensors); returns the result buffer."""
        p, n, dt = _buf(buf)
        r, _, _ = _buf(residual)
        self.all_reduce_compressed(p, n, dt, op, compressor, r)
        return buf

    # ------------------------------------------------------------ device (CUDA adapter)
    def attach_device(self, device: Optional[int] = None, nccl: bool = False, **kw):
        """Attach the CUDA DeviceAdapter: maps the symmetric heaps of every rank
        (handles travel over this client's mesh) so ``*_device`` calls run the
        sm_100a peer-memory kernels. ``nccl=True`` also forms an NCCL
        communicator over this client (id sent by rank 0 over the mesh) that
        carries device ``send`` / ``recv`` without ``torch.distributed``."""
        from .device import DeviceCommunicator
        self._device = DeviceCommunicator.from_client(self, device=device, **kw)
        if nccl:
            from .device.nccl import nccl_group_for_client
            self._device.attach_nccl(nccl_group_for_client(self, device=self._device.device))
        return self._device

    def reattach_device(self, old=None, device: Optional[int] = None, nccl: Optional[bool] = None, **kw):
        """Device communicator for a rebuilt client (after ``rebuild_excluding``
        / ``rebuild_adding``, a recovery or an elastic resize): closes ``old``
        (the parent's DeviceCommunicator: its mappings of departed ranks go
        away) and maps the heaps of this client's ranks. Every rank of this
        client calls it together. ``device`` and ``nccl`` default to the old
        communicator's settings. A job that relies on recovery keeps NVLS off
        (``NEXAR_NVLS=0``): a multicast object whose member died cannot be
        unbound safely."""
        if old is not None:
            if device is None:
                device = old.device
            if nccl is None:
                nccl = old.nccl is not None
            old.close()
        return self.attach_device(device, nccl=bool(nccl), **kw)

    @property
    def device(self):
        if self._device is None:
            raise RuntimeError("no CUDA device attached; call attach_device()")
        return self._device

    def _staged(self, *tensors) -> bool:
        """True when ``*_device`` calls go through the adapter's host staging
        (no device communicator attached, an adapter that is not host memory):
        the cross-host path for device buffers. Pending work on the tensors is
        finished first; the results are on the device when the call returns."""
        if self._device is not None:
            return False
        if self._c.adapter().host_addressable():
            raise RuntimeError("no CUDA device attached; call attach_device() or set a CudaAdapter")
        import torch
        for t in tensors:
            if isinstance(t, torch.Tensor) and t.is_cuda:
                torch.cuda.synchronize(t.device)
        return True

    def _staged_done(self, *tensors):
        import torch
        for t in tensors:
            if isinstance(t, torch.Tensor) and t.is_cuda:
                torch.cuda.synchronize(t.device)

    def all_reduce_device(self, t, op=ReduceOp.Sum):
        """``all_reduce`` on CUDA tensors: the device communicator's kernels, or the adapter's host staging when none is attached."""
        if self._staged(t):
            p, n, dt = _buf(t)
            self.all_reduce(p, n, dt, op)
            self._staged_done(t)
            return t
        return self.device.all_reduce(t, op=str(ReduceOp.parse(op)))

    def all_reduce_rs_ag_device(self, t, op=ReduceOp.Sum):
        """Reduce-scatter then all-gather (nexar/src/collective/rs_ag_allreduce.rs):
        on the box that is the two-shot peer-memory kernel."""
        if self._staged(t):
            p, n, dt = _buf(t)
            self.all_reduce_rs_ag(p, n, dt, op)
            self._staged_done(t)
            return t
        return self.device.all_reduce(t, op=str(ReduceOp.parse(op)), algo="two_shot")

    def broadcast_device(self, t, root: int):
        """``broadcast`` on CUDA tensors: the device communicator's kernels, or the adapter's host staging when none is attached."""
        if self._staged(t):
            p, n, dt = _buf(t)
            self.broadcast(p, n, dt, root)
            self._staged_done(t)
            return t
        return self.device.broadcast(t, root)

    def all_gather_device(self, send, recv):
        """``all_gather`` on CUDA tensors: the device communicator's kernels, or the adapter's host staging when none is attached."""
        if self._staged(send, recv):
            ps, n, dt = _buf(send)
            self.all_gather(ps, _buf(recv)[0], n, dt)
            self._staged_done(recv)
            return recv
        return self.device.all_gather(send, recv)

    def reduce_scatter_device(self, send, recv, op=ReduceOp.Sum):
        """``reduce_scatter`` on CUDA tensors: the device communicator's kernels, or the adapter's host staging when none is attached."""
        if self._staged(send, recv):
            pr, n, dt = _buf(recv)
            self.reduce_scatter(_buf(send)[0], pr, n, dt, op)
            self._staged_done(recv)
            return recv
        return self.device.reduce_scatter(send, recv, op=str(ReduceOp.parse(op)))

    def reduce_device(self, t, op, root: int):
        """``reduce`` on CUDA tensors: the device communicator's kernels, or the adapter's host staging when none is attached."""
        if self._staged(t):
            p, n, dt = _buf(t)
            self.reduce(p, n, dt, op, root)
            self._staged_done(t)
            return t
        return self.device.reduce(t, root, op=str(ReduceOp.parse(op)))

    def all_to_all_device(self, send, recv):
        """``all_to_all`` on CUDA tensors: the device communicator's kernels, or the adapter's host staging when none is attached."""
        if self._staged(send, recv):
            ps, n, dt = _buf(send)
            self.all_to_all(ps, _buf(recv)[0], n // self.world_size, dt)
            self._staged_done(recv)
            return recv
        return self.device.all_to_all(send, recv)

    def gather_device(self, send, recv, root: int):
        """``gather`` on CUDA tensors: the device communicator's kernels, or the adapter's host staging when none is attached."""
        if self._staged(send, recv):
            ps, n, dt = _buf(send)
            self.gather(ps, _buf(recv)[0] if recv is not None else 0, n, dt, root)
            self._staged_done(recv)
            return recv
        return self.device.gather(send, root, recv)

    def scatter_device(self, send, recv, root: int):
        """``scatter`` on CUDA tensors: the device communicator's kernels, or the adapter's host staging when none is attached."""
        if self._staged(send, recv):
            pr, n, dt = _buf(recv)
            self.scatter(_buf(send)[0] if send is not None else 0, pr, n, dt, root)
            self._staged_done(recv)
            return recv
        return self.device.scatter(send, root, recv)

    def scan_device(self, t, op=ReduceOp.Sum):
        """``scan`` on CUDA tensors: the device communicator's kernels, or the adapter's host staging when none is attached."""
        if self._staged(t):
            p, n, dt = _buf(t)
            self.scan(p, n, dt, op)
            self._staged_done(t)
            return t
        return t.copy_(self.device.scan(t, op=str(ReduceOp.parse(op))))

    def exclusive_scan_device(self, t, op=ReduceOp.Sum):
        """``exclusive_scan`` on CUDA tensors: the device communicator's kernels, or the adapter's host staging when none is attached."""
        if self._staged(t):
            p, n, dt = _buf(t)
            self.exclusive_scan(p, n, dt, op)
            self._staged_done(t)
            return t
        return t.copy_(self.device.exclusive_scan(t, op=str(ReduceOp.parse(op))))

    # ------------------------------------------------------------ helpers for the device layer
    def all_gather_bytes(self, data: bytes) -> List[bytes]:
        """All-gather variable-length byte strings (used for handle exchange)."""
        import numpy as np
        n = np.array([len(data)], dtype=np.uint64)
        lens = np.zeros(self.world_size, dtype=np.uint64)
        self.all_gather_host(n, lens)
        m = int(lens.max())
        mine = np.zeros(m, dtype=np.uint8)
        mine[:len(data)] = np.frombuffer(data, dtype=np.uint8)
        out = np.zeros(m * self.world_size, dtype=np.uint8)
        self.all_gather_host(mine, out)
        return [out[i * m: i * m + int(lens[i])].tobytes() for i in range(self.world_size)]

    # ------------------------------------------------------------ communicators
    def split(self, color: int, key: int) -> "NexarClient":
        """Sub-communicator of the ranks with the same `color`, ordered by (`key`, rank)."""
        return NexarClient(self._c.split(color, key))

    def rebuild_excluding(self, dead_ranks: Iterable[int]) -> "NexarClient":
        """Communicator of the surviving ranks (renumbered in order) without `dead_ranks`."""
        return NexarClient(self._c.rebuild_excluding(sorted(set(dead_ranks))))

    def rebuild_adding(self, new_mesh_ranks: Iterable[int], comm_id: int = 0) -> "NexarClient":
        """Communicator grown by the given mesh ranks (appended after the current ranks)."""
        return NexarClient(self._c.rebuild_adding(list(new_mesh_ranks), comm_id))

    def failure_watch(self) -> List[int]:
        """Current dead ranks (communicator numbering)."""
        return self._c.dead_ranks()

    def wait_failure(self, timeout_s: float) -> List[int]:
        """Block until a peer is declared dead or `timeout_s` passes; returns the dead ranks."""
        return self._c.wait_failure(timeout_s)

    def close(self):
        """Shut every connection of this rank (fault injection)."""
        self._c.close()


# The C++ API is synchronous, so the blocking client is the same object.
class RpcDispatcher:
    """Serves the RPC handlers registered on a client (nexar's RpcDispatcher)."""

    def __init__(self, client: "NexarClient"):
        self._client = client

    def register(self, fn_id: int, handler):
        self._client.register_rpc(fn_id, handler)

    def serve_once(self, src: int, timeout_s: float = -1.0):
        self._client.serve_rpc_once(src, timeout_s)

    def start(self):
        self._client.start_rpc_server()

    def stop(self):
        self._client.stop_rpc_server()


class ElasticConfig:
    """Elastic membership bounds (nexar/src/cluster/elastic.rs:21-35):
    ``min_world_size`` (shrinks below it are refused), ``max_world_size``
    (0 = unbounded joins), ``checkpoint_timeout_s``."""

    def __init__(self, min_world_size: int = 1, max_world_size: int = 0, checkpoint_timeout_s: float = 60.0):
        self.min_world_size = int(min_world_size)
        self.max_world_size = int(max_world_size)
        self.checkpoint_timeout_s = float(checkpoint_timeout_s)

    def __repr__(self):
        return (f"ElasticConfig(min_world_size={self.min_world_size}, max_world_size={self.max_world_size}, "
                f"checkpoint_timeout_s={self.checkpoint_timeout_s})")


class ElasticBootstrap:
    """Result of ``NexarClient.bootstrap_elastic``: the seed, the initial clients, their managers."""

    def __init__(self, seed, clients, managers):
        self.seed = seed
        self.clients = clients
        self.managers = managers

    @property
    def seed_addr(self) -> str:
        return self.seed.local_addr()


SyncClient = NexarClient


class WorkerNode:
    """Joins a cluster through its seed (nexar/src/cluster/worker.rs:10-149)."""

    @staticmethod
    def connect(seed_addr: str, token: Optional[bytes] = None, bind_host: str = "127.0.0.1", tls: bool = False):
        """Bind this rank's mesh listener on ``bind_host`` (advertised to the
        others), send Hello with ``token`` (``NEXAR_CLUSTER_TOKEN`` if None),
        wait for Welcome. Returns a ``WorkerInfo`` (rank, world_size, peers,
        listen_addr) for ``NexarClient.from_worker``."""
        return _h().WorkerNode.connect(seed_addr, token, bind_host, tls)


def SeedNode(addr: str = "127.0.0.1:0", token: Optional[bytes] = None, local: bool = False):
    h = _h()
    return h.SeedNode.bind_local() if local else h.SeedNode.bind(addr, token)


def TopKCompressor(ratio: float):
    return _h().TopKCompressor(ratio)


def RandomKCompressor(ratio: float):
    return _h().RandomKCompressor(ratio)


def NoCompression():
    return _h().NoCompression()


class RecoveryPolicy:
    """Recovery policy codes (nexar/src/config.rs RecoveryPolicy)."""
    Automatic = 0
    Manual = 1
    Abort = 2


class RecoveryOrchestrator:
    """Failure watch + agreement + rebuild (nexar/src/cluster/recovery.rs:16-355),
    over the native orchestrator.

    ``new(client, policy)`` returns ``(orchestrator, receiver)`` like the
    reference; ``subscribe()`` adds broadcast receivers (``recv(timeout_s)``
    returns the next RecoveryEvent or None). ``run()`` blocks on the calling
    thread until ``shutdown()``; ``start()`` runs the same loop on a native
    thread."""

    def __init__(self, client: "NexarClient", policy: int = RecoveryPolicy.Automatic):
        self._o = _h().RecoveryOrchestrator(client.native, int(policy))

    @classmethod
    def new(cls, client: "NexarClient", policy: int = RecoveryPolicy.Automatic):
        o = cls(client, policy)
        return o, o.subscribe()

    @classmethod
    def from_config(cls, client: "NexarClient"):
        o = cls.__new__(cls)
        o._o = _h().RecoveryOrchestrator.from_config(client.native)
        return o, o.subscribe()

    def subscribe(self):
        return self._o.subscribe()

    def client(self) -> "NexarClient":
        return NexarClient(self._o.client())

    def start(self):
        self._o.start()

    def run(self):
        self._o.run()

    def shutdown(self):
        self._o.shutdown()

    def next_event(self, timeout_s: float):
        return self._o.next_event(timeout_s)

    def error(self) -> str:
        return self._o.error()

    @property
    def native(self):
        return self._o


class ElasticManager:
    """Elastic membership at training-step boundaries (nexar/src/cluster/elastic.rs),
    over the native manager: ``elastic_checkpoint()`` (collective), ``subscribe()``,
    ``client()``, ``remove_node(rank)`` (coordinator), ``events()``.
    Joiners call ``ElasticManager.join(seed_addr, token)``."""

    def __init__(self, client: "NexarClient", seed=None, min_world: int = 1, max_world: int = 0,
                 timeout_s: float = 60.0):
        self._m = _h().ElasticManager(client.native, seed, min_world, max_world, timeout_s)

    @classmethod
    def wrap(cls, native) -> "ElasticManager":
        m = cls.__new__(cls)
        m._m = native
        return m

    @staticmethod
    def join(seed_addr: str, token: Optional[bytes] = None, config=None, timeout_s: float = 60.0) -> "NexarClient":
        cfg = config if config is not None else _h().Config()
        return NexarClient(_h().ElasticManager.join(seed_addr, token, cfg, timeout_s))

    def elastic_checkpoint(self) -> bool:
        return self._m.elastic_checkpoint()

    def subscribe(self):
        return self._m.subscribe()

    def client(self) -> Optional["NexarClient"]:
        c = self._m.client()
        return None if c is None else NexarClient(c)

    def remove_node(self, rank: int):
        self._m.remove_node(rank)

    def events(self):
        return self._m.events()

    @property
    def epoch(self) -> int:
        return self._m.epoch

    @property
    def native(self):
        return self._m
