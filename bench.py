"""Flagship benchmark: data-parallel GPT-2-small training step (GPT-2-small, micro-batch 8 x 1024 tokens per GPU, bf16).

    python bench.py --gpus N --steps K --warmup W            # nexar_b200 (this repo)
    python bench.py --impl reference ...                     # the reference (unavailable here)
    python bench.py --impl torch ...                         # plain PyTorch + cuBLAS + NCCL comparator

For N > 1 launch with torchrun (one rank per GPU). Per GPU: micro-batch 8 x
1024 tokens, bf16, synthetic uniform token ids, random N(0, 0.02) init. The
timed step is the whole training step: forward, backward, bucketed gradient
all-reduce over NVLink (overlapped with backward), global-norm clip and
AdamW, replayed from one CUDA graph. `value` is whole-job tokens/s from CUDA
events (max over ranks); `e2e` re-times the same step through the public
`DataParallelTrainer.step()` API, including the pinned-host H2D copy of each
batch and the D2H read of the loss.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

METRIC = "dp_gpt2_small_train_tokens_per_sec"
MICRO_BATCH = 8
SEQ_LEN = 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="nexar", choices=["nexar", "reference", "torch"])
    ap.add_argument("--micro-batch", type=int, default=MICRO_BATCH)
    ap.add_argument("--seq-len", type=int, default=SEQ_LEN)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--model", default="small", choices=["small", "tiny"])
    ap.add_argument("--attention", default="sdpa", choices=["sdpa", "nexar"],
                    help="attention kernels: torch SDPA (default) or this package's tcgen05 kernels")
    return ap.parse_args()


def reference_unavailable(args):
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "n_gpus": args.gpus,
        "unavailable": "the reference (ml-rust/nexar) is a Rust workspace with no Python package and "
                       "no cargo/rustc on this image: pip install of the reference fails "
                       "('Neither setup.py nor pyproject.toml found'), and it has no model or trainer",
    }), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        reference_unavailable(args)
        return 0
    if args.impl == "torch":
        from nexar_b200.bench.torch_gpt2 import run
        return run(args, METRIC)
    if args.warmup < 3:
        args.warmup = 3
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if args.attention == "nexar":
        os.environ["NEXAR_ATTENTION"] = "nexar"
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=dev)

    from nexar_b200 import _native
    from nexar_b200.models.gpt2 import GPT2Config
    from nexar_b200.parallel.dp import DataParallelTrainer
    from nexar_b200.utils.clocks import ClockSampler, device_uuids

    cfg = GPT2Config.small() if args.model == "small" else GPT2Config.tiny()
    B, T = args.micro_batch, min(args.seq_len, cfg.block_size)
    comm = None
    if world > 1:
        from nexar_b200.device import DeviceCommunicator
        comm = DeviceCommunicator.from_torch()
    trainer = DataParallelTrainer(cfg, B, T, comm=comm, use_cuda_graph=not args.no_graph, seed=0)

    # synthetic data: uniform random token ids, seeded per rank
    g = torch.Generator().manual_seed(1234 + rank)
    nbatches = 4
    host_idx = [torch.randint(0, cfg.vocab_size, (B, T), generator=g).pin_memory() for _ in range(nbatches)]
    host_tgt = [torch.randint(0, cfg.vocab_size, (B, T), generator=g).pin_memory() for _ in range(nbatches)]
    trainer.set_batch(host_idx[0], host_tgt[0])
    torch.cuda.synchronize()
    trainer.capture(warmup=args.warmup)   # W untimed warm-up steps (+ graph capture)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ---------------- device-timed region: exactly K steps
    trainer.set_batch(host_idx[1], host_tgt[1])
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _native.launch_count()
    with ClockSampler(device_uuids([local_rank]), period_ms=100) as clk:
        start.record()
        for _ in range(args.steps):
            trainer.run_step()
        end.record()
        barrier()
    ms = start.elapsed_time(end)
    tl = trainer.timeline()  # NEXAR_DP_TIMELINE=1: per-bucket all-reduce timeline of the last step
    if tl is not None:
        tl["rank"] = rank
        print("timeline " + json.dumps(tl), file=sys.stderr, flush=True)
    eager_launches = _native.launch_count() - launches0
    gpu_launches = trainer.graph_launches * args.steps if trainer.graph is not None else eager_launches
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_per_step = ms_max / args.steps
    tokens_per_step = B * T * world
    value = tokens_per_step / (ms_per_step / 1e3)

    # ---------------- end-to-end through the public API: H2D batch + step + D2H loss
    barrier()
    t0 = time.perf_counter()
    loss = None
    for i in range(args.steps):
        loss = trainer.step(host_idx[i % nbatches], host_tgt[i % nbatches])
    barrier()
    e2e_s = time.perf_counter() - t0
    te = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = tokens_per_step * args.steps / float(te.item())
    h2d = 2 * B * T * 8
    d2h = 4

    clocks = clk.summary()
    if rank == 0:
        flops = trainer.model.flops_per_token(T) * tokens_per_step / (ms_per_step / 1e3)
        print(json.dumps({
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (uniform random token ids, seeded per rank; random N(0,0.02) init)",
            "impl": "nexar_b200",
            "config": {"model": "gpt2-small (12L, d768, 12H, vocab 50257 padded to 50304)",
                       "global_batch": B * world, "micro_batch_per_gpu": B, "seq_len": T,
                       "parallelism": f"dp{world}", "grad_bucket_mb": 25,
                       "cuda_graph": trainer.graph is not None,
                       "attention": "nexar tcgen05" if trainer.model.own_attention else "torch sdpa",
                       "l2": "no flush: per-step working set (weights+grads+optimizer 2 GB, activations ~5 GB) "
                             "exceeds the 126 MB L2"},
            "model_tflops_per_gpu": round(flops / world / 1e12, 1),
            "clocks": clocks,
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "api": "DataParallelTrainer.step", "last_loss": loss},
            "gpu_launches": int(gpu_launches),
        }), flush=True)
    trainer.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
