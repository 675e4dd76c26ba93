"""Wire-level enums and the error hierarchy.

``DataType`` keeps the reference's ``repr(u8)`` codes 0..9 exactly
(nexar/src/types.rs:13-24) and adds the two fp8 formats as 10 and 11.
``ReduceOp`` keeps the reference's order Sum, Prod, Min, Max
(nexar/src/types.rs:62-71). The error classes mirror ``NexarError``
(nexar/src/error.rs:6-105); the C++ runtime raises them by numeric code.
"""
from __future__ import annotations

import enum

PROTOCOL_VERSION = 1  # nexar/src/types.rs:110


class DataType(enum.IntEnum):
    F32 = 0
    F64 = 1
    F16 = 2
    BF16 = 3
    I8 = 4
    I32 = 5
    I64 = 6
    U8 = 7
    U32 = 8
    U64 = 9
    F8E4M3 = 10
    F8E5M2 = 11

    @property
    def size_in_bytes(self) -> int:
        return _DT_SIZE[self]

    @property
    def type_name(self) -> str:
        return self.name.lower().replace("f8e4m3", "f8e4m3").replace("f8e5m2", "f8e5m2")

    def __str__(self) -> str:  # matches the reference's Display ("f32", "bf16", ...)
        return self.type_name

    @staticmethod
    def from_torch(dtype) -> "DataType":
        import torch
        table = {
            torch.float32: DataType.F32, torch.float64: DataType.F64,
            torch.float16: DataType.F16, torch.bfloat16: DataType.BF16,
            torch.int8: DataType.I8, torch.int32: DataType.I32, torch.int64: DataType.I64,
            torch.uint8: DataType.U8, torch.uint32: DataType.U32, torch.uint64: DataType.U64,
            torch.float8_e4m3fn: DataType.F8E4M3, torch.float8_e5m2: DataType.F8E5M2,
        }
        if dtype not in table:
            raise UnsupportedDType(f"unsupported torch dtype {dtype}")
        return table[dtype]

    def to_torch(self):
        import torch
        return {
            DataType.F32: torch.float32, DataType.F64: torch.float64,
            DataType.F16: torch.float16, DataType.BF16: torch.bfloat16,
            DataType.I8: torch.int8, DataType.I32: torch.int32, DataType.I64: torch.int64,
            DataType.U8: torch.uint8, DataType.U32: torch.uint32, DataType.U64: torch.uint64,
            DataType.F8E4M3: torch.float8_e4m3fn, DataType.F8E5M2: torch.float8_e5m2,
        }[self]

    def to_numpy(self):
        import numpy as np
        table = {
            DataType.F32: np.float32, DataType.F64: np.float64, DataType.F16: np.float16,
            DataType.I8: np.int8, DataType.I32: np.int32, DataType.I64: np.int64,
            DataType.U8: np.uint8, DataType.U32: np.uint32, DataType.U64: np.uint64,
            DataType.BF16: np.uint16,  # raw bits; numpy has no bfloat16
        }
        return table[self]


_DT_SIZE = {
    DataType.F32: 4, DataType.I32: 4, DataType.U32: 4,
    DataType.F64: 8, DataType.I64: 8, DataType.U64: 8,
    DataType.F16: 2, DataType.BF16: 2,
    DataType.I8: 1, DataType.U8: 1, DataType.F8E4M3: 1, DataType.F8E5M2: 1,
}


class ReduceOp(enum.IntEnum):
    Sum = 0
    Prod = 1
    Min = 2
    Max = 3

    def __str__(self) -> str:
        return self.name.lower()

    @staticmethod
    def parse(op) -> "ReduceOp":
        if isinstance(op, ReduceOp):
            return op
        if isinstance(op, int):
            return ReduceOp(op)
        return {"sum": ReduceOp.Sum, "prod": ReduceOp.Prod, "min": ReduceOp.Min,
                "max": ReduceOp.Max}[str(op).lower()]


class Priority(enum.IntEnum):
    """Message priority (nexar/src/types.rs:91-98)."""
    Critical = 0
    Realtime = 1
    Bulk = 2


# ----------------------------------------------------------------- errors
class NexarError(RuntimeError):
    """Base class of every error raised by nexar_b200 (nexar/src/error.rs)."""
    code = 0


def _err(name, code, base=NexarError):
    cls = type(name, (base,), {"code": code})
    return cls


ConnectionFailed = _err("ConnectionFailed", 1)
PeerDisconnected = _err("PeerDisconnected", 2)
UnknownPeer = _err("UnknownPeer", 3)
ProtocolMismatch = _err("ProtocolMismatch", 4)
DecodeFailed = _err("DecodeFailed", 5)
EncodeFailed = _err("EncodeFailed", 6)
BarrierTimeout = _err("BarrierTimeout", 7)
ClusterFormationTimeout = _err("ClusterFormationTimeout", 8)
UnsupportedDType = _err("UnsupportedDType", 9)
BufferSizeMismatch = _err("BufferSizeMismatch", 10)
InvalidRank = _err("InvalidRank", 11)
Transport = _err("Transport", 12)
Tls = _err("Tls", 13)
Io = _err("Io", 14)
RpcNotRegistered = _err("RpcNotRegistered", 15)
RpcFailed = _err("RpcFailed", 16)
DeviceError = _err("DeviceError", 17)
CollectiveFailed = _err("CollectiveFailed", 18)
Cancelled = _err("Cancelled", 19)
ClusterTokenMismatch = _err("ClusterTokenMismatch", 20)
IndivisibleCount = _err("IndivisibleCount", 21)
LockPoisoned = _err("LockPoisoned", 22)
Recovery = _err("Recovery", 23)
ElasticTimeout = _err("ElasticTimeout", 24)
Elastic = _err("Elastic", 25)
Timeout = _err("Timeout", 26)

ERRORS_BY_CODE = {c.code: c for c in [
    ConnectionFailed, PeerDisconnected, UnknownPeer, ProtocolMismatch, DecodeFailed,
    EncodeFailed, BarrierTimeout, ClusterFormationTimeout, UnsupportedDType,
    BufferSizeMismatch, InvalidRank, Transport, Tls, Io, RpcNotRegistered, RpcFailed,
    DeviceError, CollectiveFailed, Cancelled, ClusterTokenMismatch, IndivisibleCount,
    LockPoisoned, Recovery, ElasticTimeout, Elastic, Timeout]}


def raise_for_code(code: int, message: str):
    raise ERRORS_BY_CODE.get(code, NexarError)(message)
