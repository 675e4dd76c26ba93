"""Context parallelism: ring attention over sequence shards.

Each of W ranks holds a contiguous shard of T/W tokens (its Q, K and V). The
key / value blocks travel around the ring (rank r sends to r + 1, receives
from r - 1) while every rank attends its queries to the block it holds; the
partial outputs merge through their log-sum-exp. Under the causal mask a
rank skips blocks from later shards and masks its own block's diagonal.
The backward pass rotates each key / value block together with the gradient
accumulated for it, so after W steps every rank holds dK and dV of its own
shard; dQ stays local. The reference has no attention; the transfers are its
tagged send / recv (nexar/src/client/async_client.rs:312-379), here through
:class:`RingHost` (CPU ranks over a host client) or :class:`RingNccl`
(GPUs over an NcclGroup, one grouped send + receive per step).

Shapes: q, k, v [N, S, D] for one rank's S tokens and N = batch x heads.
"""
from __future__ import annotations

import math

import torch


class RingHost:
    """Ring shifts between CPU ranks over a host NexarClient (tagged messages)."""

    def __init__(self, client):
        self.client = client
        self.rank = client.rank
        self.world_size = client.world_size
        self._tag = 0

    def shift(self, t: torch.Tensor) -> torch.Tensor:
        """Send t to rank + 1, return the same-shaped tensor from rank - 1."""
        W = self.world_size
        self._tag += 1
        t = t.contiguous()
        self.client.send(t.data_ptr(), t.numel() * t.element_size(), (self.rank + 1) % W, self._tag)
        out = torch.empty_like(t)
        self.client.recv(out.data_ptr(), out.numel() * out.element_size(), (self.rank - 1) % W, self._tag)
        return out


class RingNccl:
    """Ring shifts between GPUs over an NcclGroup (send and receive as one group)."""

    def __init__(self, group):
        self.group = group
        self.rank = group.local_rank
        self.world_size = group.local_world

    def shift(self, t: torch.Tensor) -> torch.Tensor:
        W = self.world_size
        out = torch.empty_like(t)
        self.group.send_recv(t.contiguous(), (self.rank + 1) % W, out, (self.rank - 1) % W)
        return out


def _block_fwd(q, k, v, scale, diag):
    s = torch.einsum("nqd,nkd->nqk", q, k) * scale
    if diag:
        S = q.shape[1]
        s = s.masked_fill(torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    o = torch.einsum("nqk,nkd->nqd", torch.exp(s - lse[..., None]), v)
    return o, lse


def _merge(o, lse, o_b, lse_b):
    new = torch.logaddexp(lse, lse_b)
    return o * torch.exp(lse - new)[..., None] + o_b * torch.exp(lse_b - new)[..., None], new


class _RingAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, ring, causal):
        W, r = ring.world_size, ring.rank
        scale = 1.0 / math.sqrt(q.shape[-1])
        o = torch.zeros_like(q, dtype=torch.float32 if q.dtype != torch.float64 else q.dtype)
        lse = torch.full(q.shape[:2], float("-inf"), dtype=o.dtype, device=q.device)
        kv = torch.stack([k, v])
        for step in range(W):
            src = (r - step) % W
            if not (causal and src > r):
                o_b, lse_b = _block_fwd(q.to(o.dtype), kv[0].to(o.dtype), kv[1].to(o.dtype), scale,
                                        causal and src == r)
                o, lse = _merge(o, lse, o_b, lse_b)
            if step < W - 1:
                kv = ring.shift(kv)
        out = o.to(q.dtype)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.ring, ctx.causal, ctx.scale = ring, causal, scale
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse = ctx.saved_tensors
        ring, causal, scale = ctx.ring, ctx.causal, ctx.scale
        W, r = ring.world_size, ring.rank
        f = lse.dtype
        qf, dof = q.to(f), dout.to(f)
        delta = (dof * out.to(f)).sum(-1)
        dq = torch.zeros_like(qf)
        kv = torch.stack([k, v])
        dkv = torch.zeros_like(kv, dtype=f)
        S = q.shape[1]
        for step in range(W):
            src = (r - step) % W
            if not (causal and src > r):
                kf, vf = kv[0].to(f), kv[1].to(f)
                s = torch.einsum("nqd,nkd->nqk", qf, kf) * scale
                if causal and src == r:
                    s = s.masked_fill(torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
                p = torch.exp(s - lse[..., None])
                dp = torch.einsum("nqd,nkd->nqk", dof, vf)
                ds = p * (dp - delta[..., None])
                dq += torch.einsum("nqk,nkd->nqd", ds, kf) * scale
                dkv[0] += torch.einsum("nqk,nqd->nkd", ds, qf) * scale
                dkv[1] += torch.einsum("nqk,nqd->nkd", p, dof)
            # the gradient travels with its block; after W shifts it is home
            if step < W - 1:
                kv = ring.shift(kv)
            dkv = ring.shift(dkv) if W > 1 else dkv
        return dq.to(q.dtype), dkv[0].to(k.dtype), dkv[1].to(v.dtype), None, None


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, ring, causal: bool = True) -> torch.Tensor:
    """softmax(q K^T / sqrt(D)) V over the whole ring's sequence for this
    rank's queries; q, k, v are [N, S, D] shards (rank r holds tokens
    [r*S, (r+1)*S)). Differentiable in q, k and v."""
    return _RingAttention.apply(q, k, v, ring, causal)
