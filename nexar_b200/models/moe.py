"""Expert-parallel MoE layer (8 experts on 8 GPUs, top-2 router): one SwiGLU expert per GPU,
top-2 softmax routing, d=4096, expert ffn=14336, 16384 tokens per GPU, bf16.

forward():          route kernel -> device all-gather of the per-expert counts
                    -> fused dispatch (all-to-all + permutation, peer stores
                    into the expert's symmetric receive buffer) -> expert
                    SwiGLU MLP on tcgen05 GEMMs -> fused combine (peer loads,
                    gate scaling and top-2 sum).
forward_baseline(): the same layer with torch routing/permutation, NCCL
                    all_to_all_single and cuBLAS GEMMs (the comparator).
train_step():       forward and backward (nexar_b200.parallel.expert): the
                    output gradient goes to the experts with a gate-scaled
                    fused dispatch, input and gate gradients come back with
                    fused combines; train_step_baseline() is its comparator.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import _native, ops


@dataclass
class MoEConfig:
    d_model: int = 4096
    ffn: int = 14336
    tokens_per_gpu: int = 16384
    capacity_factor: float = 2.0  # receive rows = capacity_factor * 2 * tokens_per_gpu

    @staticmethod
    def small() -> "MoEConfig":
        return MoEConfig(d_model=256, ffn=512, tokens_per_gpu=512)


class ExpertParallelMoE:
    def __init__(self, cfg: MoEConfig, comm, seed: int = 0):
        self.cfg, self.comm = cfg, comm
        self.E = comm.world_size
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        g = torch.Generator(device=dev).manual_seed(seed + 7919 * comm.rank)
        F, d = cfg.ffn, cfg.d_model
        self.w_up = (0.02 * torch.randn(2 * F, d, device=dev, generator=g)).to(torch.bfloat16)   # [gate; up]
        self.w_down = (0.02 * torch.randn(d, F, device=dev, generator=g)).to(torch.bfloat16)
        T = cfg.tokens_per_gpu
        self.capacity = int(cfg.capacity_factor * 2 * T)
        self.recv = comm.symmetric_empty([self.capacity, d], torch.bfloat16)
        self.eout = comm.symmetric_empty([self.capacity, d], torch.bfloat16)
        self.slot_expert = torch.empty(2 * T, dtype=torch.int32, device=dev)
        self.slot_pos = torch.empty(2 * T, dtype=torch.int32, device=dev)
        self.slot_gate = torch.empty(2 * T, dtype=torch.float32, device=dev)
        self.counts = torch.zeros(self.E, dtype=torch.int32, device=dev)
        self.counts_all = torch.empty(self.E * self.E, dtype=torch.int32, device=dev)
        self.ticket = torch.zeros(1, dtype=torch.int32, device=dev)
        self.gu = torch.empty(self.capacity, 2 * F, dtype=torch.bfloat16, device=dev)
        self.h = torch.empty(self.capacity, F, dtype=torch.bfloat16, device=dev)
        self._C = _native.cuda()
        self.last_rows = 0

    def flops(self, rows: int) -> float:
        c = self.cfg
        return 2.0 * rows * c.d_model * 2 * c.ffn + 2.0 * rows * c.ffn * c.d_model

    def forward(self, x: torch.Tensor, logits: torch.Tensor) -> torch.Tensor:
        """x: [T, d] bf16 tokens of this rank; logits: [T, E] router logits."""
        C, comm = self._C, self.comm
        T, d = x.shape
        self.counts.zero_()
        C.moe_route(logits, self.slot_expert, self.slot_pos, self.slot_gate, self.counts)
        comm.all_gather(self.counts, self.counts_all)
        comm.order_launch()
        C.moe_dispatch(comm.native, x, self.slot_expert, self.slot_pos, self.counts_all, self.recv, self.ticket)
        # rows this expert received (host read of E*E ints: sizes the GEMM launches)
        rows = int(self.counts_all.view(self.E, self.E)[:, comm.rank].sum().item())
        rows = min(rows, self.capacity)
        self.last_rows = rows
        if rows > 0:
            gu, h = self.gu[:rows], self.h[:rows]
            C.gemm(self.recv[:rows], self.w_up, gu)
            C.swiglu_fwd(gu, h)
            C.gemm(h, self.w_down, self.eout[:rows])
        out = torch.empty_like(x)
        comm.order_launch()
        C.moe_combine(comm.native, out, self.slot_expert, self.slot_pos, self.slot_gate, self.eout)
        return out

    def train_step(self, x: torch.Tensor, logits: torch.Tensor, dout: torch.Tensor):
        """Forward and backward of the layer on the fused kernels
        (nexar_b200.parallel.expert): returns a dict with out, dx, dlogits,
        dw_up and dw_down. The first call allocates the gradient buffers in
        symmetric memory (every rank calls it together)."""
        from ..parallel.expert import DeviceEP, moe_train_step
        if getattr(self, "_ep", None) is None:
            self._ep = DeviceEP(self)
        return moe_train_step(x, logits, dout, self.w_up, self.w_down, self._ep)

    def train_step_baseline(self, x: torch.Tensor, logits: torch.Tensor, dout: torch.Tensor, group=None):
        """The same forward and backward with torch routing / permutation, NCCL
        all_to_all_single and cuBLAS GEMMs (the comparator)."""
        import torch.distributed as dist
        T, d = x.shape
        E, F = self.E, self.cfg.ffn
        top_v, top_i = torch.topk(logits.float(), 2, dim=-1)
        gates = torch.softmax(top_v, dim=-1)
        flat_e = top_i.reshape(-1)
        order = torch.argsort(flat_e, stable=True)
        send = x.repeat_interleave(2, dim=0)[order]
        send_counts = torch.bincount(flat_e, minlength=E)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()

        def a2a(t, out_rows, out_splits, in_splits):
            out = torch.empty(out_rows, d, dtype=t.dtype, device=t.device)
            dist.all_to_all_single(out, t.contiguous(), out_splits, in_splits, group=group)
            return out

        recv = a2a(send, sum(rc), rc, sc)
        gu = torch.matmul(recv, self.w_up.t())
        g, u = gu[:, :F], gu[:, F:]
        sg = torch.sigmoid(g)
        silu = g * sg
        hh = silu * u
        eo = torch.matmul(hh, self.w_down.t())
        back = a2a(eo, 2 * T, sc, rc)
        unperm = torch.empty_like(back)
        unperm[order] = back
        unperm = unperm.view(T, 2, d).float()
        out = (unperm * gates.unsqueeze(-1)).sum(1).to(x.dtype)
        # backward
        df = dout.float()
        dg = (unperm * df.unsqueeze(1)).sum(-1)                       # [T, 2]
        d_unperm = (gates.unsqueeze(-1) * df.unsqueeze(1)).to(x.dtype).view(2 * T, d)
        d_eo = a2a(d_unperm[order], sum(rc), rc, sc)
        dhh = torch.matmul(d_eo, self.w_down)
        dw_down = torch.matmul(d_eo.t(), hh)
        dgu = torch.cat([dhh * u * (sg * (1 + g * (1 - sg))), dhh * silu], dim=1)
        d_recv = torch.matmul(dgu, self.w_up)
        dw_up = torch.matmul(dgu.t(), recv)
        d_send = a2a(d_recv, 2 * T, sc, rc)
        d_rep = torch.empty_like(d_send)
        d_rep[order] = d_send
        dx = d_rep.view(T, 2, d).float().sum(1).to(x.dtype)
        c = gates[:, 0] * gates[:, 1] * (dg[:, 0] - dg[:, 1])
        dlogits = torch.zeros(T, E, dtype=torch.float32, device=x.device)
        ar = torch.arange(T, device=x.device)
        dlogits[ar, top_i[:, 0]] += c
        dlogits[ar, top_i[:, 1]] -= c
        return {"out": out, "dx": dx, "dlogits": dlogits, "dw_up": dw_up, "dw_down": dw_down}

    def forward_baseline(self, x: torch.Tensor, logits: torch.Tensor, group=None) -> torch.Tensor:
        import torch.distributed as dist
        T, d = x.shape
        E = self.E
        top_v, top_i = torch.topk(logits.float(), 2, dim=-1)
        gates = torch.softmax(top_v, dim=-1)
        flat_e = top_i.reshape(-1)
        order = torch.argsort(flat_e, stable=True)
        send = x.repeat_interleave(2, dim=0)[order]                       # permute
        send_counts = torch.bincount(flat_e, minlength=E)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        recv = torch.empty(sum(rc), d, dtype=x.dtype, device=x.device)
        dist.all_to_all_single(recv, send, rc, sc, group=group)
        gu = torch.matmul(recv, self.w_up.t())
        F = self.cfg.ffn
        hh = torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]
        eo = torch.matmul(hh, self.w_down.t())
        back = torch.empty_like(send)
        dist.all_to_all_single(back, eo, sc, rc, group=group)
        unperm = torch.empty_like(back)
        unperm[order] = back                                             # unpermute
        unperm = unperm.view(T, 2, d).float()
        return (unperm * gates.unsqueeze(-1)).sum(1).to(x.dtype)
