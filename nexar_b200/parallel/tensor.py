"""Tensor-parallel SwiGLU MLP training step (forward and backward).

Sequence-parallel layout over W ranks: every rank holds T/W tokens of the
block's input and output, its column slice of the gate / up projection
(w_gu = [gate_r; up_r], [2F/W, d]) and its row slice of the down projection
(w_down [d, F/W]).

  forward   gu = AG(x) w_gu^T        (fused all-gather -> GEMM)
            h  = silu(gate) * up
            y  = RS(h w_down^T)      (fused GEMM -> reduce-scatter)
  backward  dh = AG(dy) w_down       (fused all-gather -> GEMM, B = w_down^T)
            dw_down = AG(dy)^T h     (GEMM on MN-major operands, no transposes)
            dgu = swiglu'(gu) dh
            dx = RS(dgu w_gu)        (fused GEMM -> reduce-scatter, B = w_gu^T)
            dw_gu = dgu^T AG(x)

The collectives and GEMMs come from a backend: :class:`DeviceTP` runs the
tcgen05 fused kernels of a :class:`~nexar_b200.device.DeviceCommunicator`;
:class:`HostTP` runs the same schedule on CPU tensors over a host client
(all-gather / reduce-scatter on the host transport, torch matmuls), which is
how the schedule is tested without GPUs. The reference has no tensor
parallelism (its primitives are all_gather / reduce_scatter,
nexar/src/collective/{allgather,reduce_scatter}.rs).
"""
from __future__ import annotations

import torch

from .. import _native


class DeviceTP:
    """Fused kernels over a DeviceCommunicator (bf16 CUDA tensors)."""

    def __init__(self, comm):
        self.comm = comm
        self.world_size = comm.world_size
        self.rank = comm.rank

    def ag_gemm(self, x_shard, B):
        """(AG(x) B^T, AG(x)): the gathered input comes from the kernel's workspace."""
        out = self.comm.all_gather_gemm(x_shard, B)
        full = self.comm.gathered(x_shard.shape[0] * self.world_size, x_shard.shape[1]).clone()
        return out, full

    def gemm_rs(self, A, B):
        return self.comm.gemm_reduce_scatter(A, B)

    def matmul_tn(self, A, B):
        """A^T B for A [M, N1], B [M, N2] (both read MN-major)."""
        from .. import ops
        return ops.matmul_nt(A, B, a_t=True, b_t=True)

    def swiglu(self, gu):
        h = torch.empty(gu.shape[0], gu.shape[1] // 2, dtype=gu.dtype, device=gu.device)
        _native.cuda().swiglu_fwd(gu, h)
        return h

    def swiglu_bwd(self, gu, dh):
        dgu = torch.empty_like(gu)
        _native.cuda().swiglu_bwd(gu, dh, dgu)
        return dgu


class HostTP:
    """The same schedule on CPU tensors over a host NexarClient."""

    def __init__(self, client):
        self.client = client
        self.world_size = client.world_size
        self.rank = client.rank

    def _all_gather(self, x):
        full = torch.empty(x.shape[0] * self.world_size, *x.shape[1:], dtype=x.dtype)
        self.client.all_gather_host(x.contiguous().reshape(-1), full.reshape(-1))
        return full

    def ag_gemm(self, x_shard, B):
        full = self._all_gather(x_shard)
        return full @ B.t(), full

    def gemm_rs(self, A, B):
        part = (A @ B.t()).contiguous()
        out = torch.empty(part.shape[0] // self.world_size, part.shape[1], dtype=part.dtype)
        self.client.reduce_scatter_host(part.reshape(-1), out.reshape(-1))
        return out

    def matmul_tn(self, A, B):
        return A.t() @ B

    def swiglu(self, gu):
        F = gu.shape[1] // 2
        return torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]

    def swiglu_bwd(self, gu, dh):
        F = gu.shape[1] // 2
        g, u = gu[:, :F], gu[:, F:]
        sg = torch.sigmoid(g)
        silu = g * sg
        return torch.cat([dh * u * (sg * (1 + g * (1 - sg))), dh * silu], dim=1)


class _TPMLP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_shard, w_gu, w_down, tp):
        gu, x_full = tp.ag_gemm(x_shard.contiguous(), w_gu)
        h = tp.swiglu(gu)
        y = tp.gemm_rs(h, w_down)
        ctx.tp = tp
        ctx.save_for_backward(x_full, gu, h, w_gu, w_down)
        return y

    @staticmethod
    def backward(ctx, dy):
        x_full, gu, h, w_gu, w_down = ctx.saved_tensors
        tp = ctx.tp
        dh, dy_full = tp.ag_gemm(dy.contiguous(), w_down.t().contiguous())
        dw_down = tp.matmul_tn(dy_full, h)
        dgu = tp.swiglu_bwd(gu, dh)
        dx = tp.gemm_rs(dgu, w_gu.t().contiguous())
        dw_gu = tp.matmul_tn(dgu, x_full)
        return dx, dw_gu, dw_down, None


def tp_mlp(x_shard: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor, tp) -> torch.Tensor:
    """One tensor-parallel SwiGLU MLP block on this rank's token shard, differentiable
    in the input and both weight slices."""
    return _TPMLP.apply(x_shard, w_gu, w_down, tp)
