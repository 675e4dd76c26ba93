"""Typed buffer references and the tiered host buffer pool.

Parity:
  * ``BufferPtr`` / ``BufferRef`` with a memory-space marker (``Host`` /
    ``Device``): nexar/src/memory/buffer.rs:15-115. The reference uses the
    marker to pick the adapter at compile time; here it is checked when the
    reference is built (a CUDA tensor is ``Device``, everything else ``Host``)
    and ``NexarClient`` routes ``Device`` references to the sm_100a
    communicator.
  * ``GlobalPtr`` (nexar/src/memory/global_ptr.rs): ``nexar_b200.device.GlobalPtr``.
  * ``PoolProfile`` / ``TierConfig`` / ``PoolBuilder`` / ``BufferPool``:
    nexar/src/transport/buffer_pool.rs:28-354, implemented in C++
    (``csrc/host/buffer_pool.cc``); this module is the Python surface.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass
from typing import Optional

from . import _native
from .core import DataType

__all__ = ["MemorySpace", "Host", "Device", "BufferPtr", "BufferRef", "PoolProfile", "TierConfig",
           "PoolBuilder", "BufferPool", "GlobalPtr"]


class MemorySpace(enum.Enum):
    Host = "host"
    Device = "device"


Host = MemorySpace.Host
Device = MemorySpace.Device


@dataclass(frozen=True)
class BufferPtr:
    """A raw address in one memory space."""
    address: int
    space: MemorySpace

    def as_u64(self) -> int:
        return int(self.address)


class BufferRef:
    """A contiguous buffer (address, byte length, element type) in one memory space.

    Built from a torch tensor, a numpy array, or a raw (address, nbytes,
    dtype, space). Keeps the source object alive."""

    def __init__(self, obj=None, *, address: Optional[int] = None, nbytes: Optional[int] = None,
                 dtype: Optional[DataType] = None, space: Optional[MemorySpace] = None):
        self._obj = obj
        if obj is not None:
            from .client import _buf
            addr, numel, dt = _buf(obj)
            is_cuda = bool(getattr(obj, "is_cuda", False))
            self._ptr = BufferPtr(addr, Device if is_cuda else Host)
            self._dtype = dt
            self._nbytes = numel * dt.size_in_bytes
            if space is not None and space != self._ptr.space:
                raise ValueError(f"buffer lives in {self._ptr.space.value} memory, not {space.value}")
        else:
            if address is None or nbytes is None or dtype is None or space is None:
                raise ValueError("raw BufferRef needs address, nbytes, dtype and space")
            self._ptr = BufferPtr(int(address), space)
            self._dtype = DataType(dtype)
            self._nbytes = int(nbytes)

    @classmethod
    def host(cls, obj) -> "BufferRef":
        return cls(obj, space=Host)

    @classmethod
    def device(cls, obj) -> "BufferRef":
        return cls(obj, space=Device)

    def ptr(self) -> BufferPtr:
        return self._ptr

    @property
    def space(self) -> MemorySpace:
        return self._ptr.space

    @property
    def dtype(self) -> DataType:
        return self._dtype

    def len_bytes(self) -> int:
        return self._nbytes

    def count(self) -> int:
        return self._nbytes // self._dtype.size_in_bytes

    def is_empty(self) -> bool:
        return self._nbytes == 0

    def as_u64(self) -> int:
        return self._ptr.as_u64()

    @property
    def obj(self):
        return self._obj

    def __repr__(self):
        return f"BufferRef<{self.space.value}>(0x{self.as_u64():x}, {self._nbytes} B, {self._dtype.name})"


class PoolProfile(enum.IntEnum):
    """Buffer counts per tier: Training 256/32/16/4, Inference 256/16/4/0."""
    Training = 0
    Inference = 1


@dataclass
class TierConfig:
    count: int      # buffers kept on the tier's free list
    capacity: int   # bytes per buffer


class PoolBuilder:
    """Fluent tier configuration; defaults 1 small (64 KiB), 1 large (8 MiB),
    1 huge (64 MiB), 0 giant (256 MiB)."""

    def __init__(self):
        self._t = [TierConfig(1, 64 << 10), TierConfig(1, 8 << 20), TierConfig(1, 64 << 20), TierConfig(0, 256 << 20)]

    def small(self, c: TierConfig) -> "PoolBuilder":
        self._t[0] = c
        return self

    def large(self, c: TierConfig) -> "PoolBuilder":
        self._t[1] = c
        return self

    def huge(self, c: TierConfig) -> "PoolBuilder":
        self._t[2] = c
        return self

    def giant(self, c: TierConfig) -> "PoolBuilder":
        self._t[3] = c
        return self

    def build(self):
        return _native.host().BufferPool.from_tiers(*[(t.count, t.capacity) for t in self._t])


class BufferPool:
    """Constructors of the native tiered pool (``checkout(len)`` returns a
    zeroed ``PooledBuf`` that goes back to its tier when released)."""

    @staticmethod
    def new():
        return BufferPool.with_profile(PoolProfile.Training)

    @staticmethod
    def with_profile(profile: PoolProfile):
        return _native.host().BufferPool.with_profile(int(profile))

    @staticmethod
    def with_config(small_pool_size: int, small_buf_cap: int):
        return _native.host().BufferPool.with_config(small_pool_size, small_buf_cap)

    @staticmethod
    def builder() -> PoolBuilder:
        return PoolBuilder()


def __getattr__(name):
    if name == "GlobalPtr":
        from .device import GlobalPtr
        return GlobalPtr
    raise AttributeError(name)
