"""Plain PyTorch comparator for the flagship step (``bench.py --impl torch``).

The same GPT-2-small training step written the way a PyTorch user would:
``nn.Linear`` / ``F.layer_norm`` / ``F.scaled_dot_product_attention``
(cuDNN / flash) under bf16 autocast with fp32 parameters, the tied LM head,
``F.cross_entropy``, ``torch.nn.utils.clip_grad_norm_`` and the fused
``torch.optim.AdamW``; for N > 1 ``torch.nn.parallel.DistributedDataParallel``
(NCCL, 25 MB buckets). Eager mode, no CUDA graph (torch.compile is not
used). Timed like the nexar_b200 arm: W warm-up steps, K steps between CUDA
events with a barrier and a synchronize on both sides, max over ranks; the
end-to-end figure adds each step's pinned H2D copy of the batch and the D2H
read of the loss.

This is not the reference (ml-rust/nexar has no model or trainer); it is
the NCCL + cuBLAS baseline the data-parallel configuration is measured
against.
"""
from __future__ import annotations

import json
import math
import os
import time

import torch
import torch.nn as nn
import torch.nn.functional as F


class _Block(nn.Module):
    def __init__(self, C: int, H: int):
        super().__init__()
        self.H = H
        self.ln1 = nn.LayerNorm(C)
        self.attn = nn.Linear(C, 3 * C)
        self.proj = nn.Linear(C, C)
        self.ln2 = nn.LayerNorm(C)
        self.fc = nn.Linear(C, 4 * C)
        self.fcproj = nn.Linear(4 * C, C)

    def forward(self, x):
        B, T, C = x.shape
        q, k, v = self.attn(self.ln1(x)).view(B, T, 3, self.H, C // self.H).unbind(2)
        y = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True)
        x = x + self.proj(y.transpose(1, 2).reshape(B, T, C))
        return x + self.fcproj(F.gelu(self.fc(self.ln2(x)), approximate="tanh"))


class TorchGPT2(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        C = cfg.n_embd
        self.wte = nn.Embedding(cfg.padded_vocab, C)
        self.wpe = nn.Embedding(cfg.block_size, C)
        self.blocks = nn.ModuleList(_Block(C, cfg.n_head) for _ in range(cfg.n_layer))
        self.lnf = nn.LayerNorm(C)
        proj_std = 0.02 / math.sqrt(2 * cfg.n_layer)
        for name, p in self.named_parameters():
            if name.endswith("bias"):
                nn.init.zeros_(p)
            elif p.dim() >= 2:
                nn.init.normal_(p, 0.0, proj_std if name.endswith("proj.weight") else 0.02)

    def forward(self, idx, tgt):
        T = idx.shape[1]
        x = self.wte(idx) + self.wpe.weight[:T]
        for blk in self.blocks:
            x = blk(x)
        logits = F.linear(self.lnf(x), self.wte.weight)  # tied head, padded vocab
        return F.cross_entropy(logits.float().view(-1, logits.shape[-1]), tgt.view(-1))


def run(args, metric: str) -> int:
    import torch.distributed as dist
    from ..models.gpt2 import GPT2Config
    from ..utils.clocks import ClockSampler, device_uuids

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=dev)
    cfg = GPT2Config.small() if args.model == "small" else GPT2Config.tiny()
    B, T = args.micro_batch, min(args.seq_len, cfg.block_size)
    torch.manual_seed(0)
    model = TorchGPT2(cfg).to(dev)
    if world > 1:
        model = nn.parallel.DistributedDataParallel(model, device_ids=[local_rank], bucket_cap_mb=25,
                                                    gradient_as_bucket_view=True)
    decay = [p for n, p in model.named_parameters() if p.dim() >= 2]
    no_decay = [p for n, p in model.named_parameters() if p.dim() < 2]
    opt = torch.optim.AdamW([{"params": decay, "weight_decay": 0.1}, {"params": no_decay, "weight_decay": 0.0}],
                            lr=6e-4, betas=(0.9, 0.95), eps=1e-8, fused=True)
    g = torch.Generator().manual_seed(1234 + rank)
    nb = 4
    host_idx = [torch.randint(0, cfg.vocab_size, (B, T), generator=g).pin_memory() for _ in range(nb)]
    host_tgt = [torch.randint(0, cfg.vocab_size, (B, T), generator=g).pin_memory() for _ in range(nb)]
    idx = host_idx[0].to(dev)
    tgt = host_tgt[0].to(dev)

    def step(i, t):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model(i, t)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss

    for _ in range(max(3, args.warmup)):
        step(idx, tgt)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device_uuids([local_rank]), period_ms=100) as clk:
        start.record()
        for _ in range(args.steps):
            step(idx, tgt)
        end.record()
        barrier()
    t = torch.tensor([start.elapsed_time(end)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item()) / args.steps
    tokens = B * T * world

    barrier()
    t0 = time.perf_counter()
    loss_v = None
    for i in range(args.steps):
        idx.copy_(host_idx[i % nb], non_blocking=True)
        tgt.copy_(host_tgt[i % nb], non_blocking=True)
        loss_v = float(step(idx, tgt).item())
    barrier()
    te = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    if rank == 0:
        print(json.dumps({
            "impl": "torch", "metric": metric, "value": round(tokens / (ms_per_step / 1e3), 1), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 autocast (fp32 params)",
            "data": "synthetic (uniform random token ids, seeded per rank; random N(0,0.02) init)",
            "config": {"model": "gpt2-small (12L, d768, 12H, vocab 50257 padded to 50304)", "global_batch": B * world,
                       "micro_batch_per_gpu": B, "seq_len": T, "parallelism": f"dp{world}", "grad_bucket_mb": 25,
                       "stack": "torch eager: nn.Linear (cuBLAS), SDPA, fused AdamW, DDP over NCCL",
                       "l2": "no flush: per-step working set exceeds the 126 MB L2"},
            "clocks": clk.summary(),
            "e2e": {"value": round(tokens * args.steps / float(te.item()), 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": 2 * B * T * 8, "d2h_bytes_per_step": 4, "last_loss": loss_v},
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main() -> int:
    """``python -m nexar_b200.bench.torch_gpt2`` (same flags as ``bench.py --impl torch``)."""
    import argparse
    ap = argparse.ArgumentParser(description="plain PyTorch GPT-2 data-parallel step (NCCL + cuBLAS comparator)")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--micro-batch", type=int, default=8)
    ap.add_argument("--seq-len", type=int, default=1024)
    ap.add_argument("--model", default="small", choices=["small", "tiny"])
    return run(ap.parse_args(), "dp_gpt2_small_train_tokens_per_sec")


if __name__ == "__main__":
    raise SystemExit(main())
