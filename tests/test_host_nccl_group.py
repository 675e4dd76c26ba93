"""NCCL layer without a GPU: type mapping, id format and the id exchange over
the host control plane. Parity with nexar-nccl/tests/hierarchical.rs
(test_type_mappings, test_nccl_id_serialization, test_error_types) and
nexar-nccl/src/bootstrap.rs:79-118 (lead -> local ranks, tag 0xACC1_0000 | node)."""
import pytest
import torch

from helpers_host import bootstrap, run_collective
from nexar_b200.core import DataType, NexarError, ReduceOp
from nexar_b200.device import nccl
from nexar_b200.parallel.hierarchical import NodeTopology

# ncclDataType_t / ncclRedOp_t values from nccl.h
NCCL_TYPES = {
    DataType.F32: 7, DataType.F64: 8, DataType.F16: 6, DataType.BF16: 9,
    DataType.I8: 0, DataType.I32: 2, DataType.I64: 4, DataType.U8: 1,
    DataType.U32: 3, DataType.U64: 5, DataType.F8E4M3: 10, DataType.F8E5M2: 11,
}
NCCL_OPS = {ReduceOp.Sum: 0, ReduceOp.Prod: 1, ReduceOp.Max: 2, ReduceOp.Min: 3}


def test_type_mappings():
    for dt, v in NCCL_TYPES.items():
        assert nccl.to_nccl_dtype(dt) == v, dt
        assert nccl.to_nccl_dtype(dt.to_torch()) == v, dt
    for op, v in NCCL_OPS.items():
        assert nccl.to_nccl_op(op) == v, op
        assert nccl.to_nccl_op(op.name.lower()) == v, op
    with pytest.raises(NexarError):
        nccl._native_call(nccl._lib().nccl_dtype, 12)
    with pytest.raises(ValueError):
        nccl.to_nccl_dtype(99)


def test_nccl_id_serialization():
    a, b = nccl.unique_id(), nccl.unique_id()
    assert len(a) == nccl.UNIQUE_ID_BYTES == nccl._lib().UNIQUE_ID_BYTES == 128
    assert a != b
    assert nccl.id_from_bytes(nccl.id_to_bytes(a)) == a
    for bad in (b"", b"x" * 127, b"x" * 129):
        with pytest.raises(nccl.BootstrapError):
            nccl.id_from_bytes(bad)
    assert nccl.version() >= 22700


def test_error_types():
    for cls in (nccl.NcclError, nccl.CudaDriverError, nccl.TopologyError, nccl.InvalidRank,
                nccl.NotLeadRank, nccl.BootstrapError):
        assert issubclass(cls, nccl.NcclCommError) and issubclass(cls, NexarError)
    assert isinstance(nccl._translate(RuntimeError("nccl: ncclAllReduce failed: x")), nccl.NcclError)
    assert isinstance(nccl._translate(RuntimeError("cuda: cudaEventRecord failed")), nccl.CudaDriverError)
    e = nccl._translate(RuntimeError("usage: invalid rank 5: world size is 4"))
    assert isinstance(e, nccl.InvalidRank) and "world size is 4" in str(e)
    assert "hostname mismatch" in str(nccl.TopologyError("hostname mismatch"))


def test_group_rejects_bad_arguments_before_touching_a_device():
    uid = nccl.unique_id()
    with pytest.raises(nccl.InvalidRank):
        nccl._native_call(nccl._lib().NcclGroup, 4, 4, uid, 0, 0)
    with pytest.raises(nccl.NcclCommError, match="128 bytes"):
        nccl._native_call(nccl._lib().NcclGroup, 0, 2, b"short", 0, 0)


@pytest.mark.parametrize("names", [["a", "a", "b", "b"], ["a", "b", "a", "b"], ["a", "a", "a", "b"]])
def test_nccl_id_exchange_per_node(names):
    """Every rank of a node ends with its lead's id; nodes get distinct ids."""
    clients = bootstrap(len(names))
    try:
        def go(c):
            t = NodeTopology.from_hostnames(c.rank, names)
            return nccl.exchange_nccl_id(c, t.local_ranks, t.node_idx, t.lead)

        ids = run_collective(clients, go)
        topo = NodeTopology.from_hostnames(0, names)
        for node in topo.nodes:
            assert len({ids[r] for r in node}) == 1
            assert len(ids[node[0]]) == 128
        assert len({ids[n[0]] for n in topo.nodes}) == len(topo.nodes)
    finally:
        for c in clients:
            c.close()


def test_nccl_id_exchange_whole_client():
    clients = bootstrap(3)
    try:
        ids = run_collective(clients, lambda c: nccl.exchange_nccl_id(c, list(range(3)), 0, 0))
        assert ids[0] == ids[1] == ids[2]
    finally:
        for c in clients:
            c.close()


def test_tensor_ops_need_cuda_tensors():
    with pytest.raises(nccl.NcclCommError, match="CUDA"):
        nccl._ptr(torch.zeros(4))
