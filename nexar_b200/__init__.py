"""nexar_b200: a B200-native collectives runtime with the capabilities of nexar.

Layers:
  * ``nexar_b200.core``      DataType / ReduceOp wire codes, config, errors.
  * ``nexar_b200.client``    NexarClient / SyncClient over the C++ host runtime
                             (seed/worker bootstrap, tagged p2p, host collectives,
                             RPC, split, rebuild, recovery, elastic, sparse overlays).
  * ``nexar_b200.device``    DeviceCommunicator: symmetric heap over NVLink and the
                             sm_100a peer-memory collectives; NcclGroup (device
                             point-to-point over NCCL).
  * ``nexar_b200.ops``       model kernels (LayerNorm, GELU, SwiGLU, cross-entropy,
                             AdamW, tcgen05 GEMM, fused GEMM+collective kernels).
  * ``nexar_b200.models``    GPT-2, Llama MLP (TP) and MoE (EP) model definitions.
  * ``nexar_b200.parallel``  data, tensor, expert, sequence (Ulysses), context
                             (ring attention) and pipeline (1F1B) parallel
                             training steps; the hierarchical (node x
                             cross-node) communicator.
  * ``nexar_b200.memory``    BufferRef<Host|Device>, the tiered host buffer pool.
"""
from .core import DataType, ReduceOp, NexarError, Priority  # noqa: F401

__version__ = "0.1.0"

# The reference's crate-root exports (nexar/src/lib.rs:17-33, nexar-nccl/src/lib.rs:9-14),
# resolved on first use so that importing the package loads no extension.
_EXPORTS = {
    "NexarClient": "client", "SyncClient": "client", "CollectiveHandle": "client",
    "CollectiveGroup": "client", "SeedNode": "client", "WorkerNode": "client",
    "RecoveryOrchestrator": "client", "RecoveryPolicy": "client", "ElasticManager": "client",
    "ElasticBootstrap": "client", "ElasticConfig": "client", "Config": "client",
    "NexarConfig": ("client", "Config"), "CpuAdapter": "client", "CudaAdapter": "client",
    "DeviceAdapter": "client", "TopKCompressor": "client", "RandomKCompressor": "client",
    "NoCompression": "client", "RpcDispatcher": "client",
    "BufferPtr": "memory", "BufferRef": "memory", "MemorySpace": "memory", "Host": "memory",
    "Device": "memory", "BufferPool": "memory", "PoolBuilder": "memory", "PoolProfile": "memory",
    "TierConfig": "memory",
    "DeviceCommunicator": "device", "GlobalPtr": "device", "DeviceHandle": "device",
    "NcclGroup": ("device.nccl", "NcclGroup"),
    "HierarchicalComm": "parallel.hierarchical", "form_hierarchical_comm": "parallel.hierarchical",
    "NodeTopology": "parallel.hierarchical",
}

# Scalar aliases of the reference (nexar/src/types.rs): ranks and node ids are ints.
Rank = int
NodeId = int


def IoVec(ptr: int, len: int):  # noqa: A002  (field name of the reference's IoVec)
    """One scatter / gather region (nexar/src/types.rs:102-107): ``(ptr, len)``
    in bytes, the element type of ``send_iov`` / ``recv_iov``."""
    return (int(ptr), int(len))


def __getattr__(name):
    spec = _EXPORTS.get(name)
    if spec is None:
        if name in ("TopologyStrategy", "Compressor", "RecoveryEvent", "ElasticEvent", "ClusterMap"):
            from . import _native
            return getattr(_native.host(), name)
        raise AttributeError(f"module 'nexar_b200' has no attribute {name!r}")
    mod, attr = spec if isinstance(spec, tuple) else (spec, name)
    import importlib
    return getattr(importlib.import_module(f".{mod}", __name__), attr)
