"""Expert-parallel MoE layer forward: fused dispatch/combine kernels vs
NCCL all_to_all_single + torch permutation + cuBLAS (the MoE benchmark configuration).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m nexar_b200.bench.moe [--tokens 16384] [--train]
"""
from __future__ import annotations

import argparse
import json
import os


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--d", type=int, default=4096)
    ap.add_argument("--ffn", type=int, default=14336)
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--train", action="store_true", help="also time forward + backward (train_step)")
    args = ap.parse_args()
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    os.environ.setdefault("NEXAR_SYMM_USER_BYTES", str(3 << 30))
    from nexar_b200.device import DeviceCommunicator
    from nexar_b200.models.moe import ExpertParallelMoE, MoEConfig
    nbuf = 4 if args.train else 2  # receive / expert-output buffers (+ their gradients when training)
    comm = DeviceCommunicator.from_torch(slot_bytes=64 << 20,
                                         heap_bytes=(1 << 20) + (128 << 20) + nbuf * (2 * args.tokens * 2) * args.d * 2
                                         + (64 << 20))
    cfg = MoEConfig(args.d, args.ffn, args.tokens)
    moe = ExpertParallelMoE(cfg, comm)
    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.randn(cfg.tokens_per_gpu, cfg.d_model, device=dev, generator=g).to(torch.bfloat16)
    logits = torch.randn(cfg.tokens_per_gpu, world, device=dev, generator=g)

    def timeit(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / args.iters], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms_fused = timeit(lambda: moe.forward(x, logits))
    ms_base = timeit(lambda: moe.forward_baseline(x, logits))
    ms_train = ms_train_base = None
    if args.train:
        dout = torch.randn(cfg.tokens_per_gpu, cfg.d_model, device=dev, generator=g).to(torch.bfloat16)
        ms_train = timeit(lambda: moe.train_step(x, logits, dout))
        ms_train_base = timeit(lambda: moe.train_step_baseline(x, logits, dout))
    rows = torch.tensor([float(moe.last_rows)], device=dev)
    dist.all_reduce(rows)
    comm.check()
    if rank == 0:
        T = cfg.tokens_per_gpu * world
        print(json.dumps({
            "bench": "moe_ep_layer_fwd", "n_gpus": world, "experts": world, "tokens_per_gpu": cfg.tokens_per_gpu,
            "d": cfg.d_model, "ffn": cfg.ffn, "top_k": 2, "dtype": "bf16",
            "ms_fused": round(ms_fused, 4), "ms_nccl_torch": round(ms_base, 4),
            "speedup": round(ms_base / ms_fused, 3),
            "tokens_per_s_fused": round(T / (ms_fused / 1e3), 1),
            "expert_tflops_per_gpu": round(moe.flops(rows.item() / world) / (ms_fused / 1e3) / 1e12, 1),
        }), flush=True)
    if rank == 0 and args.train:
        T = cfg.tokens_per_gpu * world
        print(json.dumps({
            "bench": "moe_ep_layer_train_step", "n_gpus": world, "experts": world,
            "tokens_per_gpu": cfg.tokens_per_gpu, "d": cfg.d_model, "ffn": cfg.ffn, "top_k": 2, "dtype": "bf16",
            "ms_fused": round(ms_train, 4), "ms_nccl_torch": round(ms_train_base, 4),
            "speedup": round(ms_train_base / ms_train, 3),
            "tokens_per_s_fused": round(T / (ms_train / 1e3), 1),
        }), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
