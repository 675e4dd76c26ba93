"""Wire codes and error hierarchy (mirrors nexar/src/types.rs and error.rs unit tests)."""
import pytest

from nexar_b200.core import DataType, ReduceOp, Priority, NexarError, CollectiveFailed, raise_for_code


def test_datatype_codes_match_reference():
    assert [int(d) for d in (DataType.F32, DataType.F64, DataType.F16, DataType.BF16, DataType.I8,
                             DataType.I32, DataType.I64, DataType.U8, DataType.U32, DataType.U64)] == list(range(10))
    assert int(DataType.F8E4M3) == 10 and int(DataType.F8E5M2) == 11


def test_datatype_sizes_and_names():
    sizes = {DataType.F32: 4, DataType.F64: 8, DataType.F16: 2, DataType.BF16: 2, DataType.I8: 1,
             DataType.I32: 4, DataType.I64: 8, DataType.U8: 1, DataType.U32: 4, DataType.U64: 8}
    for d, s in sizes.items():
        assert d.size_in_bytes == s
    assert str(DataType.BF16) == "bf16" and str(DataType.U64) == "u64"


def test_reduce_op_order_and_parse():
    assert [int(o) for o in (ReduceOp.Sum, ReduceOp.Prod, ReduceOp.Min, ReduceOp.Max)] == [0, 1, 2, 3]
    assert ReduceOp.parse("max") is ReduceOp.Max and str(ReduceOp.Sum) == "sum"
    assert int(Priority.Critical) == 0 and int(Priority.Bulk) == 2


def test_error_codes_roundtrip():
    with pytest.raises(CollectiveFailed):
        raise_for_code(CollectiveFailed.code, "x")
    assert issubclass(CollectiveFailed, NexarError)


def test_torch_dtype_mapping():
    import torch
    for d in DataType:
        assert DataType.from_torch(d.to_torch()) is d
