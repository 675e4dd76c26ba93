"""GPT-2 decoder built on the nexar_b200 sm_100a kernels.

Benchmark configuration: 12 layers, d=768, 12 heads, vocab 50257 (padded to 50304
for 16-byte aligned rows), context 1024, bf16 compute, N(0, 0.02) init with
residual projections scaled by 1/sqrt(2*n_layer).

Kernels per layer: fused residual-add (+ the residual branch's bias) +
LayerNorm (its backward also yields that bias's gradient), QKV / proj / FC /
FC-proj GEMMs on the tcgen05 kernel (forward K-major; backward reads dY^T,
X^T and W as MN-major operands, split-K for the weight gradients; bias and
GELU fused into the FC epilogue), causal flash attention: torch SDPA by
default, the tcgen05 attention kernels of nexar_b200 with
NEXAR_ATTENTION=nexar (or own_attention=True; T a multiple of 128). The
head is the tied embedding GEMM followed by the fused softmax-cross-entropy
kernel that writes its gradient in place of the logits. Weight gradients
are stored straight into the flat gradient buffer (no zero-fill, no
per-parameter accumulation).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F

from .. import ops
from ..utils.flat import FlatParams


@dataclass
class GPT2Config:
    n_layer: int = 12
    n_head: int = 12
    n_embd: int = 768
    vocab_size: int = 50257
    padded_vocab: int = 50304
    block_size: int = 1024
    ln_eps: float = 1e-5

    @staticmethod
    def small() -> "GPT2Config":
        return GPT2Config()

    @staticmethod
    def tiny() -> "GPT2Config":
        return GPT2Config(n_layer=2, n_head=4, n_embd=128, vocab_size=1000, padded_vocab=1024, block_size=64)


def param_specs(cfg: GPT2Config) -> List[Tuple[str, Tuple[int, ...], bool]]:
    """(name, shape, weight_decay) in forward-use order."""
    C, Vp = cfg.n_embd, cfg.padded_vocab
    specs = [("wte", (Vp, C), True), ("wpe", (cfg.block_size, C), True)]
    for l in range(cfg.n_layer):
        p = f"h{l}."
        specs += [
            (p + "ln1.w", (C,), False), (p + "ln1.b", (C,), False),
            (p + "attn.w", (3 * C, C), True), (p + "attn.b", (3 * C,), False),
            (p + "proj.w", (C, C), True), (p + "proj.b", (C,), False),
            (p + "ln2.w", (C,), False), (p + "ln2.b", (C,), False),
            (p + "fc.w", (4 * C, C), True), (p + "fc.b", (4 * C,), False),
            (p + "fcproj.w", (C, 4 * C), True), (p + "fcproj.b", (C,), False),
        ]
    specs += [("lnf.w", (C,), False), ("lnf.b", (C,), False)]
    return specs


class GPT2(torch.nn.Module):
    def __init__(self, cfg: GPT2Config, device, grad_alloc=None, seed: int = 0,
                 own_attention: Optional[bool] = None):
        super().__init__()
        self.cfg = cfg
        if own_attention is None:
            own_attention = os.environ.get("NEXAR_ATTENTION", "sdpa") == "nexar"
        self.own_attention = bool(own_attention)
        self.flat = FlatParams(param_specs(cfg), device, grad_alloc=grad_alloc)
        self._init_weights(seed)
        self.p: Dict[str, torch.nn.Parameter] = self.flat.params()
        for i, (name, par) in enumerate(self.p.items()):
            self.register_parameter(name.replace(".", "_"), par)

    @torch.no_grad()
    def _init_weights(self, seed: int):
        cfg = self.cfg
        g = torch.Generator(device=self.flat.device)
        g.manual_seed(seed)
        std = 0.02
        proj_std = 0.02 / math.sqrt(2 * cfg.n_layer)
        for e in self.flat.entries:
            v = self.flat.view(self.flat.master, e.name)
            if e.name.endswith(".b"):
                v.zero_()
            elif e.name.endswith("ln1.w") or e.name.endswith("ln2.w") or e.name == "lnf.w":
                v.fill_(1.0)
            elif e.name.endswith("proj.w"):
                v.normal_(0.0, proj_std, generator=g)
            else:
                v.normal_(0.0, std, generator=g)
        # padded vocab rows never receive gradient; keep them zero
        self.flat.view(self.flat.master, "wte")[cfg.vocab_size:].zero_()
        self.flat.param_bf16.copy_(self.flat.master)

    def forward(self, idx: torch.Tensor, targets: Optional[torch.Tensor] = None, unit_grad: bool = False):
        cfg, p = self.cfg, self.p
        B, T = idx.shape
        C, H = cfg.n_embd, cfg.n_head
        hd = C // H
        x = ops.embedding(idx, p["wte"], p["wpe"]).view(B * T, C)
        h = ops.layer_norm(x, p["h0.ln1.w"], p["h0.ln1.b"], cfg.ln_eps)
        for l in range(cfg.n_layer):
            q = f"h{l}."
            qkv = ops.linear(h, p[q + "attn.w"], p[q + "attn.b"])
            if self.own_attention and ops.attention_supported(B, T, H, hd):
                y = ops.attention(qkv, B, T, H, causal=True)
            else:
                qkv = qkv.view(B, T, 3, H, hd)
                qh, kh, vh = qkv.unbind(2)
                y = F.scaled_dot_product_attention(qh.transpose(1, 2), kh.transpose(1, 2), vh.transpose(1, 2),
                                                   is_causal=True)
                y = y.transpose(1, 2).reshape(B * T, C)
            # projection bias is folded into the residual add of the next LayerNorm
            a = ops.linear(y, p[q + "proj.w"])
            x, h = ops.residual_layer_norm(x, a, p[q + "ln2.w"], p[q + "ln2.b"], cfg.ln_eps, rbias=p[q + "proj.b"])
            f = ops.linear(h, p[q + "fc.w"], p[q + "fc.b"], act="gelu")
            m = ops.linear(f, p[q + "fcproj.w"])
            if l + 1 < cfg.n_layer:
                nq = f"h{l + 1}."
                x, h = ops.residual_layer_norm(x, m, p[nq + "ln1.w"], p[nq + "ln1.b"], cfg.ln_eps,
                                               rbias=p[q + "fcproj.b"])
            else:
                x, h = ops.residual_layer_norm(x, m, p["lnf.w"], p["lnf.b"], cfg.ln_eps, rbias=p[q + "fcproj.b"])
        # tied head: its weight gradient is completed by the embedding backward
        logits = ops.linear(h, p["wte"], ready=False)  # [B*T, Vp]
        if targets is None:
            return logits.view(B, T, -1)
        return ops.cross_entropy(logits, targets, cfg.vocab_size, unit_grad=unit_grad)

    def flops_per_token(self, T: int) -> float:
        """Training FLOPs per token: 6*N (dense) + 6*L*T*C (causal attention, halved)."""
        cfg = self.cfg
        C, L = cfg.n_embd, cfg.n_layer
        n_dense = L * 12 * C * C + cfg.padded_vocab * C
        return 6.0 * n_dense + 6.0 * L * T * C
