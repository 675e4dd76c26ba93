"""Top-k + fp8 compressed all-reduce vs uncompressed all-reduce (1 GiB bf16 gradient, top-1 %).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m nexar_b200.bench.compress \
        [--numel 536870912] [--ratio 0.01] [--iters 10] [--warmup 3]

A 1 GiB bf16 gradient (512 Mi elements, N(0,1), seeded per rank) is reduced
three ways, each timed with CUDA events over back-to-back iterations, max over
ranks: the compressed path (error-feedback residual, top-1 % selection, e4m3
values + u32 indices, all-gather of the blobs, rank-ordered decompress-add),
this package's uncompressed all-reduce, and NCCL's all_reduce. Bytes per rank
on the wire: blob = k * 5 bytes (+ 16) for the compressed path.
"""
from __future__ import annotations

import argparse
import json
import os


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--numel", type=int, default=1 << 29)
    ap.add_argument("--ratio", type=float, default=0.01)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args()
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    from nexar_b200.device import DeviceCommunicator
    comm = DeviceCommunicator.from_torch()
    n = args.numel
    g = torch.Generator(device=dev).manual_seed(rank)
    grad = torch.randn(n, device=dev, generator=g).to(torch.bfloat16)
    residual = torch.zeros(n, dtype=torch.float32, device=dev)
    out = torch.empty_like(grad)
    work = grad.clone()

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

    ms_cmp = timeit(lambda: comm.all_reduce_compressed(grad, args.ratio, residual, out=out, scale=1.0 / world))
    ms_nexar = timeit(lambda: comm.all_reduce(work, scale=1.0 / world))
    ms_nccl = timeit(lambda: dist.all_reduce(work))
    comm.check()
    k = -(-n * args.ratio // 1)
    if rank == 0:
        print(json.dumps({
            "bench": "compressed_all_reduce", "n_gpus": world, "numel": n, "dtype": "bf16",
            "dense_bytes": n * 2, "ratio": args.ratio, "blob_bytes_per_rank": int(k * 5 + 16),
            "ms_compressed": round(ms_cmp, 3), "ms_nexar_allreduce": round(ms_nexar, 3),
            "ms_nccl_allreduce": round(ms_nccl, 3),
            "speedup_vs_nccl": round(ms_nccl / ms_cmp, 2),
        }), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
