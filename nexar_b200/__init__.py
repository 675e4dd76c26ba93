"""nexar_b200: a B200-native collectives runtime with the capabilities of nexar.

Layers:
  * ``nexar_b200.core``      DataType / ReduceOp wire codes, config, errors.
  * ``nexar_b200.client``    NexarClient / SyncClient over the C++ host runtime
                             (seed/worker bootstrap, tagged p2p, host collectives,
                             RPC, split, rebuild, recovery, elastic, sparse overlays).
  * ``nexar_b200.device``    DeviceCommunicator: symmetric heap over NVLink and the
                             sm_100a peer-memory collectives.
  * ``nexar_b200.ops``       model kernels (LayerNorm, GELU, SwiGLU, cross-entropy,
                             AdamW, tcgen05 GEMM, fused GEMM+collective kernels).
  * ``nexar_b200.models``    GPT-2, Llama MLP (TP) and MoE (EP) model definitions.
  * ``nexar_b200.parallel``  data-parallel, tensor-parallel and expert-parallel
                             training entry points; the hierarchical (node x
                             cross-node) communicator.
  * ``nexar_b200.memory``    BufferRef<Host|Device>, the tiered host buffer pool.
"""
from .core import DataType, ReduceOp, NexarError  # noqa: F401

__version__ = "0.1.0"
