"""Sharded data parallelism (ZeRO stage 1: optimizer state sharded) for any torch module.

Every rank keeps the full parameters and the full gradients (for forward and
backward) but only 1/W of the optimizer state: after backward the flat
gradient is reduce-scattered (rank r receives the average over ranks of its
shard), AdamW updates the fp32 master copy of that shard, and the updated
shards are all-gathered back into every rank's parameters. Optimizer memory
(master weights and both moments) per rank drops by W; gradient memory does
not (ZeRO stage 2 would also shard the gradients). The bytes on the wire
equal one all-reduce. All parameters must share one dtype (they travel as
one flat tensor).

Backends: :class:`DeviceSharding` (a DeviceCommunicator: reduce-scatter and
all-gather kernels over NVLink peer memory, with the 1/W averaging fused into
the reduce-scatter) and :class:`HostSharding` (a host client on CPU tensors).
The reference's counterpart is the reduce-scatter + all-gather all-reduce
("ZeRO-style", nexar/src/collective/rs_ag_allreduce.rs:1-8); it has no
optimizer.
"""
from __future__ import annotations

from typing import Iterable

import torch


class HostSharding:
    """reduce_scatter / all_gather of flat CPU tensors over a host NexarClient."""

    def __init__(self, client):
        self.client = client
        self.rank = client.rank
        self.world_size = client.world_size

    def reduce_scatter_mean(self, flat: torch.Tensor) -> torch.Tensor:
        out = torch.empty(flat.numel() // self.world_size, dtype=flat.dtype)
        self.client.reduce_scatter_host(flat.contiguous(), out)
        return out / self.world_size

    def all_gather(self, shard: torch.Tensor) -> torch.Tensor:
        out = torch.empty(shard.numel() * self.world_size, dtype=shard.dtype)
        self.client.all_gather_host(shard.contiguous(), out)
        return out


class DeviceSharding:
    """The device communicator's reduce-scatter (with the 1/W scale fused) and all-gather."""

    def __init__(self, comm):
        self.comm = comm
        self.rank = comm.rank
        self.world_size = comm.world_size

    def reduce_scatter_mean(self, flat: torch.Tensor) -> torch.Tensor:
        out = torch.empty(flat.numel() // self.world_size, dtype=flat.dtype, device=flat.device)
        self.comm.reduce_scatter(flat.contiguous(), out, scale=1.0 / self.world_size)
        return out

    def all_gather(self, shard: torch.Tensor) -> torch.Tensor:
        out = torch.empty(shard.numel() * self.world_size, dtype=shard.dtype, device=shard.device)
        self.comm.all_gather(shard.contiguous(), out)
        return out


class ShardedAdamW:
    """AdamW whose state is sharded over the data-parallel ranks.

    Call :meth:`step` after ``loss.backward()`` on every rank (a collective);
    it averages the gradients over the ranks, updates this rank's shard and
    leaves every rank's parameters identical. Weight decay is decoupled
    (AdamW) and applies to all parameters."""

    def __init__(self, params: Iterable[torch.nn.Parameter], backend, lr: float = 1e-3, betas=(0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 0.0):
        self.params = [p for p in params if p.requires_grad]
        dtypes = {p.dtype for p in self.params}
        if len(dtypes) != 1:
            raise ValueError(f"ShardedAdamW needs parameters of one dtype (one flat tensor), got {sorted(map(str, dtypes))}")
        self.backend = backend
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        W, r = backend.world_size, backend.rank
        n = sum(p.numel() for p in self.params)
        self.numel = n
        self.padded = (n + W - 1) // W * W
        self.shard = self.padded // W
        self.lo = r * self.shard
        dev = self.params[0].device
        flat = self._flat(lambda p: p.detach())
        self.master = flat[self.lo:self.lo + self.shard].to(torch.float32 if flat.dtype != torch.float64
                                                             else torch.float64).clone()
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.t = 0
        self.device = dev

    def _flat(self, get) -> torch.Tensor:
        parts = [get(p).reshape(-1) for p in self.params]
        pad = self.padded - self.numel
        if pad:
            parts.append(torch.zeros(pad, dtype=parts[0].dtype, device=parts[0].device))
        return torch.cat(parts)

    def zero_grad(self):
        for p in self.params:
            p.grad = None

    @torch.no_grad()
    def step(self):
        b1, b2 = self.betas
        grads = self._flat(lambda p: p.grad if p.grad is not None else torch.zeros_like(p))
        g = self.backend.reduce_scatter_mean(grads).to(self.master.dtype)
        self.t += 1
        self.exp_avg.mul_(b1).add_(g, alpha=1 - b1)
        self.exp_avg_sq.mul_(b2).addcmul_(g, g, value=1 - b2)
        bc1 = 1 - b1 ** self.t
        bc2 = 1 - b2 ** self.t
        denom = (self.exp_avg_sq / bc2).sqrt_().add_(self.eps)
        self.master.mul_(1 - self.lr * self.wd)
        self.master.addcdiv_(self.exp_avg, denom, value=-self.lr / bc1)
        full = self.backend.all_gather(self.master.to(self.params[0].dtype))
        off = 0
        for p in self.params:
            p.copy_(full[off:off + p.numel()].view_as(p))
            off += p.numel()

    def state_bytes(self) -> int:
        """Optimizer state held by this rank (master weights and both moments)."""
        return 3 * self.master.numel() * self.master.element_size()
