"""Expert-parallel MoE training step (forward and backward), one expert per rank.

Forward (top-2 routing, SwiGLU experts):
  route      slot (t, k) -> expert e_k(t), gate g_k(t) = softmax of the two logits
  dispatch   token rows into the experts' receive buffers        (fused all-to-all)
  experts    gu = recv w_up^T, h = swiglu(gu), eout = h w_down^T
  combine    out[t] = sum_k g_k eout[e_k][row_k]                  (fused all-to-all)
Backward (for a given dout):
  d_eout     rows g_k * dout[t] into the experts' gradient buffers (scaled dispatch)
  d_gate     dg_k(t) = <dout[t], eout[e_k][row_k]> (two combines with one-hot gates)
  experts    dh = d_eout w_down, dw_down = d_eout^T h, dgu = swiglu'(gu) dh,
             d_recv = dgu w_up, dw_up = dgu^T recv
  dx         dx[t] = sum_k d_recv[e_k][row_k]                   (combine, unit gates)
  dlogits    through the two-way softmax: d l_first = g1 g2 (dg1 - dg2) = -d l_second

Backends: :class:`DeviceEP` runs the sm_100a route / dispatch / combine kernels
of :class:`~nexar_b200.models.moe.ExpertParallelMoE` (peer stores and loads
over NVLink) and the tcgen05 GEMMs; :class:`HostEP` runs the same schedule on
CPU tensors over a host client (all-gathers stand in for the peer accesses),
which is how the schedule is tested without GPUs. The reference has no MoE;
its primitive is all_to_all (nexar/src/collective/alltoall.rs:14-64).
"""
from __future__ import annotations

from typing import Dict

import torch

from .. import _native


def _gate_masks(T: int, device):
    first = torch.zeros(2 * T, dtype=torch.float32, device=device)
    first[0::2] = 1.0
    second = 1.0 - first
    ones = torch.ones(2 * T, dtype=torch.float32, device=device)
    return first, second, ones


def moe_train_step(x: torch.Tensor, logits: torch.Tensor, dout: torch.Tensor, w_up: torch.Tensor,
                   w_down: torch.Tensor, ep) -> Dict[str, torch.Tensor]:
    """One forward + backward of the MoE layer on this rank's T tokens.

    x [T, d], logits [T, E] (E = number of ranks), dout [T, d]; w_up [2F, d]
    ([gate; up]) and w_down [d, F] are this rank's expert. Returns out, dx,
    dlogits, dw_up, dw_down."""
    T, d = x.shape
    slots = ep.route(logits)
    rows = slots["rows"]
    recv = ep.dispatch(x, slots)
    eout = ep.expert_buffer()
    if rows > 0:
        gu = ep.nt(recv, w_up)
        h = ep.swiglu(gu)
        ep.nt(h, w_down, out=eout[:rows])
    out = ep.combine(eout, slots, slots["gate"], T, d)

    first, second, ones = _gate_masks(T, x.device)
    d_eout = ep.dispatch_rows(dout, slots, slots["gate"])
    r1 = ep.combine(eout, slots, first, T, d).float()
    r2 = ep.combine(eout, slots, second, T, d).float()
    df = dout.float()
    dg1, dg2 = (df * r1).sum(1), (df * r2).sum(1)
    d_recv = ep.grad_buffer()
    if rows > 0:
        dh = ep.nn(d_eout, w_down)
        dw_down = ep.tn(d_eout, h)
        dgu = ep.swiglu_bwd(gu, dh)
        ep.nn(dgu, w_up, out=d_recv[:rows])
        dw_up = ep.tn(dgu, recv)
    else:  # no token chose this expert
        dw_down, dw_up = torch.zeros_like(w_down), torch.zeros_like(w_up)
    dx = ep.combine(d_recv, slots, ones, T, d)

    gate = slots["gate"].float()
    g1, g2 = gate[0::2], gate[1::2]
    c = g1 * g2 * (dg1 - dg2)
    experts = slots["expert"].long()
    dlogits = torch.zeros(T, logits.shape[1], dtype=torch.float32, device=x.device)
    ar = torch.arange(T, device=x.device)
    dlogits[ar, experts[0::2]] += c
    dlogits[ar, experts[1::2]] -= c
    return {"out": out, "dx": dx, "dlogits": dlogits, "dw_up": dw_up, "dw_down": dw_down}


class DeviceEP:
    """The fused kernels and buffers of an ExpertParallelMoE layer (bf16, CUDA)."""

    def __init__(self, layer):
        self.layer = layer
        self.comm = layer.comm
        self.world_size = self.comm.world_size
        self.rank = self.comm.rank
        self._C = _native.cuda()
        d = layer.cfg.d_model
        # gradient buffers the peers store into: symmetric, allocated in the same
        # order on every rank
        self.d_eout = self.comm.symmetric_empty([layer.capacity, d], torch.bfloat16)
        self.d_recv = self.comm.symmetric_empty([layer.capacity, d], torch.bfloat16)

    def route(self, logits):
        L, C = self.layer, self._C
        L.counts.zero_()
        C.moe_route(logits.contiguous(), L.slot_expert, L.slot_pos, L.slot_gate, L.counts)
        self.comm.all_gather(L.counts, L.counts_all)
        rows = int(L.counts_all.view(self.world_size, self.world_size)[:, self.rank].sum().item())
        return {"expert": L.slot_expert, "pos": L.slot_pos, "gate": L.slot_gate, "rows": min(rows, L.capacity)}

    def dispatch(self, x, slots):
        L = self.layer
        self.comm.order_launch()
        self._C.moe_dispatch(self.comm.native, x.contiguous(), L.slot_expert, L.slot_pos, L.counts_all, L.recv,
                             L.ticket)
        return L.recv[:slots["rows"]]

    def dispatch_rows(self, g, slots, scale):
        L = self.layer
        self.comm.order_launch()
        self._C.moe_dispatch_rows(self.comm.native, g.contiguous(), L.slot_expert, L.slot_pos, scale, self.d_eout,
                                  L.ticket)
        return self.d_eout[:slots["rows"]]

    def combine(self, buf, slots, gates, T, d):
        L = self.layer
        out = torch.empty(T, d, dtype=torch.bfloat16, device=buf.device)
        self.comm.order_launch()
        self._C.moe_combine(self.comm.native, out, L.slot_expert, L.slot_pos, gates, buf)
        return out

    def expert_buffer(self):
        return self.layer.eout

    def grad_buffer(self):
        return self.d_recv

    @staticmethod
    def nt(a, b, out=None):
        from .. import ops
        return ops.matmul_nt(a, b, out=out)

    @staticmethod
    def nn(a, b, out=None):
        from .. import ops
        return ops.matmul_nt(a, b, out=out, b_t=True)

    @staticmethod
    def tn(a, b):
        from .. import ops
        return ops.matmul_nt(a, b, a_t=True, b_t=True)

    def swiglu(self, gu):
        h = torch.empty(gu.shape[0], gu.shape[1] // 2, dtype=gu.dtype, device=gu.device)
        self._C.swiglu_fwd(gu, h)
        return h

    def swiglu_bwd(self, gu, dh):
        dgu = torch.empty_like(gu)
        self._C.swiglu_bwd(gu, dh.contiguous(), dgu)
        return dgu


class HostEP:
    """The same schedule on CPU tensors over a host NexarClient: routing by the
    kernel's rule (top two logits, softmax over them), positions in slot order
    within each (source rank, expert), expert buffers of `capacity` rows; the
    peer stores and loads of the fused kernels become all-gathers."""

    def __init__(self, client, capacity: int, d: int, dtype=torch.float64):
        self.client = client
        self.world_size = client.world_size
        self.rank = client.rank
        self.capacity = capacity
        self.eout = torch.zeros(capacity, d, dtype=dtype)
        self.d_eout = torch.zeros(capacity, d, dtype=dtype)
        self.d_recv = torch.zeros(capacity, d, dtype=dtype)

    def _all_gather(self, t):
        out = torch.empty(self.world_size, *t.shape, dtype=t.dtype)
        self.client.all_gather_host(t.contiguous().reshape(-1), out.reshape(-1))
        return out

    def route(self, logits):
        T, E = logits.shape
        top = torch.topk(logits, 2, dim=1)
        g2 = torch.sigmoid(top.values[:, 1] - top.values[:, 0])
        gate = torch.stack([1.0 - g2, g2], dim=1).reshape(-1)
        expert = top.indices.reshape(-1).to(torch.int32)
        local = torch.empty(2 * T, dtype=torch.int32)
        counts = torch.zeros(E, dtype=torch.int32)
        for s in range(2 * T):
            e = int(expert[s])
            local[s] = counts[e]
            counts[e] += 1
        counts_all = self._all_gather(counts)                       # [W, E]
        base = counts_all[:self.rank].sum(0)                        # rows of earlier sources first
        pos = (base[expert.long()] + local).to(torch.int32)
        pos[pos >= self.capacity] = -1
        rows = min(int(counts_all[:, self.rank].sum()), self.capacity)
        return {"expert": expert, "pos": pos, "gate": gate, "rows": rows}

    def _scatter_rows(self, rows_src, slots, dst):
        """dst[pos] = rows_src[slot] for every rank's slots that target this rank's expert."""
        all_rows = self._all_gather(rows_src)
        all_e = self._all_gather(slots["expert"])
        all_p = self._all_gather(slots["pos"])
        for q in range(self.world_size):
            for s in range(all_e.shape[1]):
                if int(all_e[q, s]) == self.rank and int(all_p[q, s]) >= 0:
                    dst[int(all_p[q, s])] = all_rows[q, s]
        return dst[:slots["rows"]]

    def dispatch(self, x, slots):
        self.recv = torch.zeros(self.capacity, x.shape[1], dtype=x.dtype)
        return self._scatter_rows(x.repeat_interleave(2, dim=0), slots, self.recv)

    def dispatch_rows(self, g, slots, scale):
        return self._scatter_rows(g.repeat_interleave(2, dim=0) * scale.to(g.dtype)[:, None], slots, self.d_eout)

    def combine(self, buf, slots, gates, T, d):
        bufs = self._all_gather(buf)
        out = torch.zeros(T, d, dtype=buf.dtype)
        for s in range(2 * T):
            p = int(slots["pos"][s])
            if p >= 0:
                out[s // 2] += float(gates[s]) * bufs[int(slots["expert"][s]), p]
        return out

    def expert_buffer(self):
        return self.eout

    def grad_buffer(self):
        return self.d_recv

    @staticmethod
    def nt(a, b, out=None):
        r = a @ b.t()
        if out is not None:
            out.copy_(r)
            return out
        return r

    @staticmethod
    def nn(a, b, out=None):
        r = a @ b
        if out is not None:
            out.copy_(r)
            return out
        return r

    @staticmethod
    def tn(a, b):
        return a.t() @ b

    @staticmethod
    def swiglu(gu):
        F = gu.shape[1] // 2
        return torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]

    @staticmethod
    def swiglu_bwd(gu, dh):
        F = gu.shape[1] // 2
        g, u = gu[:, :F], gu[:, F:]
        sg = torch.sigmoid(g)
        return torch.cat([dh * u * (sg * (1 + g * (1 - sg))), dh * g * sg], dim=1)
