"""Llama-style SwiGLU MLP block, tensor parallel over the GPUs of one box
(benchmark configuration: d=4096, ffn=14336, TP=8, 8192 tokens, bf16).

Sequence-parallel layout: each rank holds T/W tokens of the input and of the
output. Column-parallel up projection (gate|up, [2F/W, d] per rank) runs as
one fused all-gather->GEMM kernel; SwiGLU is one elementwise kernel; the
row-parallel down projection ([d, F/W] per rank) runs as one fused
GEMM->reduce-scatter kernel. `forward_baseline` is the same block with NCCL
collectives and cuBLAS GEMMs (the comparator).

`train_step` runs forward and backward (nexar_b200.parallel.tensor): the
backward reuses the fused kernels (all-gather -> GEMM for the input
gradient of the down projection, GEMM -> reduce-scatter for the block's input
gradient) and reads the weight-gradient GEMM operands MN-major;
`train_step_baseline` is its NCCL + cuBLAS comparator.

`forward_fp8` is the block-scaled fp8 variant of config 4: weights are kept
as e4m3 with 128x128 block scales; the input shard is quantised per 1x128
block, all-gathered as fp8 bytes + fp32 scales (half the NVLink bytes of
bf16), multiplied on the fp8 promotion GEMM, SwiGLU is fused with the
re-quantisation, and the down projection runs as one fused fp8
GEMM->reduce-scatter kernel (bf16 output).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .. import ops


@dataclass
class LlamaMLPConfig:
    d_model: int = 4096
    ffn: int = 14336
    tokens: int = 8192

    @staticmethod
    def small() -> "LlamaMLPConfig":
        return LlamaMLPConfig(d_model=512, ffn=1024, tokens=1024)


class TPLlamaMLP:
    def __init__(self, cfg: LlamaMLPConfig, comm, seed: int = 0):
        self.cfg = cfg
        self.comm = comm
        W = comm.world_size if comm is not None else 1
        self.W = W
        assert cfg.ffn % W == 0 and cfg.tokens % (W * 128) == 0
        F = cfg.ffn // W
        dev = torch.device("cuda", torch.cuda.current_device())
        g = torch.Generator(device=dev).manual_seed(seed + 1000 * (comm.rank if comm is not None else 0))
        # N(0, 0.02) weights; [gate_r ; up_r] rows for this rank's ffn slice
        self.w_up = (0.02 * torch.randn(2 * F, cfg.d_model, device=dev, generator=g)).to(torch.bfloat16)
        self.w_down = (0.02 * torch.randn(cfg.d_model, F, device=dev, generator=g)).to(torch.bfloat16)
        self.F = F
        self._fp8 = None

    def fp8_weights(self):
        """e4m3 weights with 128x128 block scales (quantised once, cached)."""
        if self._fp8 is None:
            self._fp8 = (ops.quant_fp8_128x128(self.w_up), ops.quant_fp8_128x128(self.w_down))
        return self._fp8

    def flops(self) -> float:
        """Forward FLOPs of the whole block (all ranks)."""
        c = self.cfg
        return 2.0 * c.tokens * c.d_model * (2 * c.ffn) + 2.0 * c.tokens * c.ffn * c.d_model

    def forward(self, x_shard: torch.Tensor) -> torch.Tensor:
        """x_shard: [T/W, d] -> y_shard: [T/W, d] (fused kernels)."""
        gu = self.comm.all_gather_gemm(x_shard, self.w_up)          # [T, 2F/W]
        h = ops.swiglu(gu)                                          # [T, F/W]
        return self.comm.gemm_reduce_scatter(h, self.w_down)        # [T/W, d]

    def forward_fp8(self, x_shard: torch.Tensor) -> torch.Tensor:
        """x_shard: [T/W, d] bf16 -> y_shard: [T/W, d] bf16 through the block-scaled fp8 kernels."""
        T, d = self.cfg.tokens, self.cfg.d_model
        (wuq, wus), (wdq, wds) = self.fp8_weights()
        xq, xs = ops.quant_fp8_1x128(x_shard)
        xq_full = self.comm.all_gather(xq.view(torch.uint8).reshape(-1)).view(torch.float8_e4m3fn).view(T, d)
        xs_full = self.comm.all_gather(xs.reshape(-1)).view(T, -1)
        gu = ops.matmul_fp8(xq_full, xs_full, wuq, wus)             # [T, 2F/W]
        hq, hs = ops.swiglu_quant_fp8(gu)                          # [T, F/W] e4m3
        return self.comm.gemm_fp8_reduce_scatter(hq, hs, wdq, wds)  # [T/W, d]

    def train_step(self, x_shard: torch.Tensor, dy_shard: torch.Tensor):
        """Forward and backward of the block on the fused kernels
        (nexar_b200.parallel.tensor): returns (y_shard, dx_shard, dw_gu, dw_down)."""
        from ..parallel.tensor import DeviceTP, tp_mlp
        xs = x_shard.detach().requires_grad_(True)
        wg = self.w_up.detach().requires_grad_(True)
        wd = self.w_down.detach().requires_grad_(True)
        y = tp_mlp(xs, wg, wd, DeviceTP(self.comm))
        y.backward(dy_shard)
        return y.detach(), xs.grad, wg.grad, wd.grad

    def train_step_baseline(self, x_shard: torch.Tensor, dy_shard: torch.Tensor, group=None):
        """The same forward and backward with NCCL all-gather / reduce-scatter and cuBLAS GEMMs."""
        import torch.distributed as dist
        T, d, F = self.cfg.tokens, self.cfg.d_model, self.F

        def ag(t):
            full = torch.empty(T, t.shape[1], dtype=t.dtype, device=t.device)
            dist.all_gather_into_tensor(full, t.contiguous(), group=group)
            return full

        def rs(t):
            out = torch.empty(T // self.W, t.shape[1], dtype=t.dtype, device=t.device)
            dist.reduce_scatter_tensor(out, t.contiguous(), group=group)
            return out

        xf = ag(x_shard)
        gu = torch.matmul(xf, self.w_up.t())
        g, u = gu[:, :F], gu[:, F:]
        sg = torch.sigmoid(g)
        silu = g * sg
        h = silu * u
        y = rs(torch.matmul(h, self.w_down.t()))
        dyf = ag(dy_shard)
        dh = torch.matmul(dyf, self.w_down)
        dw_down = torch.matmul(dyf.t(), h)
        dgu = torch.cat([dh * u * (sg * (1 + g * (1 - sg))), dh * silu], dim=1)
        dx = rs(torch.matmul(dgu, self.w_up))
        dw_gu = torch.matmul(dgu.t(), xf)
        return y, dx, dw_gu, dw_down

    def forward_baseline(self, x_shard: torch.Tensor, group=None) -> torch.Tensor:
        """Same block with NCCL all_gather / reduce_scatter and cuBLAS GEMMs."""
        import torch.distributed as dist
        T, d = self.cfg.tokens, self.cfg.d_model
        xf = torch.empty(T, d, dtype=x_shard.dtype, device=x_shard.device)
        dist.all_gather_into_tensor(xf, x_shard, group=group)
        gu = torch.matmul(xf, self.w_up.t())
        gate, up = gu[:, :self.F], gu[:, self.F:]
        h = torch.nn.functional.silu(gate) * up
        yp = torch.matmul(h, self.w_down.t())
        y = torch.empty(T // self.W, d, dtype=x_shard.dtype, device=x_shard.device)
        dist.reduce_scatter_tensor(y, yp, group=group)
        return y
