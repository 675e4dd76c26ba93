"""Data parallelism for any torch module: bucketed gradient all-reduce that
overlaps backward.

Parameters are grouped into buckets of about ``bucket_bytes`` in reverse
registration order (roughly the order backward produces their gradients).
A post-accumulate hook marks each gradient ready; when a bucket is complete
its gradients are packed into one flat buffer and a non-blocking all-reduce
of the bucket starts while backward continues. :meth:`finish` (call it
before the optimizer step) waits for every bucket and writes the averaged
gradients back. Gradient accumulation: run every backward pass but the last
of a step under :meth:`no_sync` (gradients only accumulate in ``.grad``); the
last pass starts the all-reduces of the accumulated sums. A second backward
outside ``no_sync`` before ``finish()`` raises instead of losing gradients.
Every rank must run the same model, so the buckets complete in the same
order everywhere and the collectives match.

Backends: :class:`DeviceBuckets` (the device communicator's all-reduce on its
side stream, with the 1/W mean fused into the kernel) and
:class:`HostBuckets` (a host client's non-blocking all-reduce on CPU
tensors). The GPT-2 trainer (``dp.DataParallelTrainer``) is the specialised
form with gradients written straight into symmetric memory. The reference
provides the primitives (all_reduce_nb and CollectiveGroup,
nexar/src/client/collectives_nb.rs:33-47; bucketed all-reduce,
nexar/src/collective/bucketed_allreduce.rs:23-75).
"""
from __future__ import annotations

import contextlib
from typing import List

import torch

from ..core import DataType


class HostBuckets:
    """Non-blocking host all-reduce of CPU tensors (mean over the ranks)."""

    def __init__(self, client):
        self.client = client
        self.world_size = client.world_size

    def start(self, flat: torch.Tensor):
        return self.client.all_reduce_nb(flat.data_ptr(), flat.numel(), DataType.from_torch(flat.dtype))

    def finish(self, handle, flat: torch.Tensor):
        handle.wait()
        flat.div_(self.world_size)


class DeviceBuckets:
    """The device communicator's all-reduce with the mean fused in (side stream)."""

    def __init__(self, comm):
        self.comm = comm
        self.world_size = comm.world_size

    def start(self, flat: torch.Tensor):
        return self.comm.all_reduce_nb(flat, scale=1.0 / self.world_size)

    def finish(self, handle, flat: torch.Tensor):
        handle.wait()


class DistributedDataParallel(torch.nn.Module):
    def __init__(self, module: torch.nn.Module, backend, bucket_bytes: int = 25 << 20):
        super().__init__()
        self.module = module
        self.backend = backend
        params = [p for p in module.parameters() if p.requires_grad]
        self.buckets: List[List[torch.nn.Parameter]] = []
        cur, size = [], 0
        for p in reversed(params):
            if cur and (size + p.numel() * p.element_size() > bucket_bytes or p.dtype != cur[0].dtype):
                self.buckets.append(cur)
                cur, size = [], 0
            cur.append(p)
            size += p.numel() * p.element_size()
        if cur:
            self.buckets.append(cur)
        self._bucket_of = {id(p): b for b, ps in enumerate(self.buckets) for p in ps}
        self._sync = True
        self._reset()
        for p in params:
            p.register_post_accumulate_grad_hook(self._hook)

    def _reset(self):
        self._left = [len(b) for b in self.buckets]
        self._inflight = {}

    @contextlib.contextmanager
    def no_sync(self):
        """Backward passes inside this context only accumulate gradients; the
        next backward outside it reduces the accumulated sums."""
        old, self._sync = self._sync, False
        try:
            yield
        finally:
            self._sync = old

    def _hook(self, p):
        if not self._sync:
            return
        b = self._bucket_of[id(p)]
        if b in self._inflight:
            raise RuntimeError(
                f"a gradient of bucket {b} arrived after its all-reduce had started: a second backward pass "
                "before finish(); run the accumulation passes under no_sync()")
        self._left[b] -= 1
        if self._left[b] == 0:
            flat = torch.cat([q.grad.reshape(-1) for q in self.buckets[b]])
            self._inflight[b] = (self.backend.start(flat), flat)

    def forward(self, *args, **kwargs):
        return self.module(*args, **kwargs)

    def finish(self):
        """Wait for every bucket's all-reduce and write the mean gradients back."""
        for b, ps in enumerate(self.buckets):
            if b not in self._inflight:  # parameters that received no gradient this step
                for q in ps:
                    if q.grad is None:
                        q.grad = torch.zeros_like(q)
                flat = torch.cat([q.grad.reshape(-1) for q in ps])
                self._inflight[b] = (self.backend.start(flat), flat)
        for b in range(len(self.buckets)):
            handle, flat = self._inflight[b]
            self.backend.finish(handle, flat)
            off = 0
            for q in self.buckets[b]:
                q.grad.copy_(flat[off:off + q.numel()].view_as(q))
                off += q.numel()
        self._reset()
