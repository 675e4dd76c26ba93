"""Sequence parallelism (Ulysses-style) for self-attention.

Each of W ranks holds a contiguous shard of T/W tokens of every sequence. The
attention layer re-shards with one all-to-all so that each rank holds the
whole sequence for H/W of the heads, runs ordinary attention on those heads,
and re-shards the output back with a second all-to-all. The reference offers
only the primitive (all_to_all, nexar/src/collective/alltoall.rs:14-64); on
the box the all-to-all is the peer-memory kernel of
:class:`~nexar_b200.device.DeviceCommunicator`, on CPU tensors any client
with ``all_to_all_host`` (see :class:`HostAllToAll`).

Layouts (row-major):
  qkv_local  [B*T_loc, 3*C]   the QKV projection of this rank's tokens
                              ([B, T_loc, 3, H, D] flattened; C = H * D)
  y_local    [B*T_loc, C]     attention output for the same tokens
Rank r owns tokens [r*T_loc, (r+1)*T_loc) of each sequence and, between the
two all-to-alls, heads [r*H/W, (r+1)*H/W).

The all-to-all of equal chunks is its own adjoint (y_r[q] = x_q[r] gives
dx_q[r] = dy_r[q]), so the backward pass is the same exchange on the
gradients.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch


class HostAllToAll:
    """``all_to_all(inp, out)`` over a host ``NexarClient`` for CPU tensors."""

    def __init__(self, client):
        self.client = client
        self.world_size = client.world_size
        self.rank = client.rank

    def all_to_all(self, inp: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        self.client.all_to_all_host(inp.reshape(-1), out.reshape(-1))
        return out


class _AllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, comm):
        ctx.comm = comm
        x = x.contiguous()
        out = torch.empty_like(x)
        comm.all_to_all(x, out)
        return out

    @staticmethod
    def backward(ctx, dy):
        dy = dy.contiguous()
        dx = torch.empty_like(dy)
        ctx.comm.all_to_all(dy, dx)
        return dx, None


def all_to_all(x: torch.Tensor, comm) -> torch.Tensor:
    """Differentiable all-to-all of equal chunks: x is [W, ...] (chunk q goes
    to rank q); the result is [W, ...] (chunk q came from rank q)."""
    return _AllToAll.apply(x, comm)


def _default_attention(qkv: torch.Tensor, B: int, T: int, H: int, D: int, causal: bool) -> torch.Tensor:
    """The tcgen05 kernels where they apply (CUDA, head dim 64, T % 128 == 0),
    else torch SDPA on [B, H, T, D] views."""
    if qkv.is_cuda and D == 64:
        from .. import ops
        if ops.attention_supported(B, T, H, D):
            return ops.attention(qkv, B, T, H, causal=causal)
    x = qkv.view(B, T, 3, H, D)
    q, k, v = (t.transpose(1, 2) for t in x.unbind(2))
    y = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=causal)
    return y.transpose(1, 2).reshape(B * T, H * D)


def ulysses_attention(qkv_local: torch.Tensor, B: int, T_local: int, H: int, D: int, comm, causal: bool = True,
                      attention: Optional[Callable] = None) -> torch.Tensor:
    """Self-attention over sequences sharded across ``comm``'s ranks.

    ``qkv_local`` is [B*T_local, 3*H*D]; returns [B*T_local, H*D]. H must be a
    multiple of the world size. ``attention(qkv, B, T, H_local, D, causal)``
    computes attention for whole sequences on H_local heads (default: the
    tcgen05 kernels or torch SDPA)."""
    W = comm.world_size
    if H % W:
        raise ValueError(f"{H} heads do not split over {W} ranks")
    Hl = H // W
    T = T_local * W
    attn = attention or _default_attention
    # [B, T_loc, 3, W, Hl, D] -> [W (head group = destination), B, T_loc, 3, Hl, D]
    send = qkv_local.view(B, T_local, 3, W, Hl, D).permute(3, 0, 1, 2, 4, 5)
    recv = all_to_all(send, comm)                        # [W (source = token shard), B, T_loc, 3, Hl, D]
    qkv_full = recv.permute(1, 0, 2, 3, 4, 5).reshape(B * T, 3 * Hl * D)
    y = attn(qkv_full, B, T, Hl, D, causal)             # [B*T, Hl*D]
    back = y.view(B, W, T_local, Hl, D).permute(1, 0, 2, 3, 4)  # [W (token shard), B, T_loc, Hl, D]
    got = all_to_all(back, comm)                         # [W (head group), B, T_loc, Hl, D]
    return got.permute(1, 2, 0, 3, 4).reshape(B * T_local, H * D)
