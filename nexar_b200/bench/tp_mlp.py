"""TP Llama-MLP block step: fused all-gather->GEMM / GEMM->reduce-scatter kernels
vs NCCL + cuBLAS (TP=8, d=4096, ffn=14336, 8192 tokens).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m nexar_b200.bench.tp_mlp [--tokens 8192] [--train]

Also times each fused kernel alone against its roofline: the slower of
(FLOPs at the measured bf16 GEMM peak) and (bytes that must cross NVLink at
770 GB/s per direction).
"""
from __future__ import annotations

import argparse
import json
import os


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--d", type=int, default=4096)
    ap.add_argument("--ffn", type=int, default=14336)
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--iters", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--train", action="store_true", help="also time forward + backward (train_step)")
    args = ap.parse_args()
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from nexar_b200.device import DeviceCommunicator
    from nexar_b200.models.llama_mlp import LlamaMLPConfig, TPLlamaMLP
    comm = DeviceCommunicator.from_torch()
    cfg = LlamaMLPConfig(args.d, args.ffn, args.tokens)
    mlp = TPLlamaMLP(cfg, comm)
    x = (torch.randn(cfg.tokens // world, cfg.d_model, device=dev)).to(torch.bfloat16)

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

    peaks = {"bf16_tflops": 1663.5}
    try:
        peaks.update(json.load(open("MEASURED_PEAKS.json")))
    except Exception:
        pass
    link = 770e9
    T, d, F, W = cfg.tokens, cfg.d_model, cfg.ffn, world
    ms_fused = timeit(lambda: mlp.forward(x))
    ms_base = timeit(lambda: mlp.forward_baseline(x))
    ms_fp8 = timeit(lambda: mlp.forward_fp8(x))
    # per-kernel rooflines
    xf_shard = x
    gu = comm.all_gather_gemm(xf_shard, mlp.w_up)
    h = torch.empty(T, F // W, dtype=torch.bfloat16, device=dev)
    ms_ag = timeit(lambda: comm.all_gather_gemm(xf_shard, mlp.w_up, out=gu))
    ms_rs = timeit(lambda: comm.gemm_reduce_scatter(h, mlp.w_down))
    flops_ag = 2.0 * T * d * (2 * F // W)
    flops_rs = 2.0 * T * (F // W) * d
    bytes_ag = (W - 1) / W * T * d * 2      # received per rank
    bytes_rs = (W - 1) / W * T * d * 2      # sent per rank
    peak = peaks["bf16_tflops"] * 1e12
    roof_ag = max(flops_ag / peak, bytes_ag / link if W > 1 else 0) * 1e3
    roof_rs = max(flops_rs / peak, bytes_rs / link if W > 1 else 0) * 1e3
    ms_train = ms_train_base = None
    if args.train:
        dy = torch.randn_like(x)
        ms_train = timeit(lambda: mlp.train_step(x, dy))
        ms_train_base = timeit(lambda: mlp.train_step_baseline(x, dy))
    comm.check()
    if rank == 0 and args.train:
        print(json.dumps({
            "bench": "tp_llama_mlp_train_step", "n_gpus": W, "tokens": T, "d": d, "ffn": F, "dtype": "bf16",
            "ms_fused": round(ms_train, 4), "ms_nccl_cublas": round(ms_train_base, 4),
            "speedup": round(ms_train_base / ms_train, 3),
            "tokens_per_s_fused": round(T / (ms_train / 1e3), 1),
            "tflops_fused": round(3 * mlp.flops() / (ms_train / 1e3) / 1e12, 1),
        }), flush=True)
    if rank == 0:
        print(json.dumps({
            "bench": "tp_llama_mlp_fwd", "n_gpus": W, "tokens": T, "d": d, "ffn": F, "dtype": "bf16",
            "ms_fused": round(ms_fused, 4), "ms_nccl_cublas": round(ms_base, 4),
            "speedup": round(ms_base / ms_fused, 3),
            "tokens_per_s_fused": round(T / (ms_fused / 1e3), 1),
            "tflops_fused": round(mlp.flops() / (ms_fused / 1e3) / 1e12, 1),
            "ag_gemm": {"ms": round(ms_ag, 4), "roofline_ms": round(roof_ag, 4), "frac": round(roof_ag / ms_ag, 3)},
            "gemm_rs": {"ms": round(ms_rs, 4), "roofline_ms": round(roof_rs, 4), "frac": round(roof_rs / ms_rs, 3)},
        }), flush=True)
        print(json.dumps({
            "bench": "tp_llama_mlp_fwd", "n_gpus": W, "tokens": T, "d": d, "ffn": F,
            "dtype": "fp8 e4m3 block-scaled (1x128 activations, 128x128 weights)",
            "ms_fp8": round(ms_fp8, 4), "ms_bf16_fused": round(ms_fused, 4), "ms_bf16_nccl_cublas": round(ms_base, 4),
            "speedup_vs_bf16_nccl_cublas": round(ms_base / ms_fp8, 3),
            "tokens_per_s_fp8": round(T / (ms_fp8 / 1e3), 1),
            "tflops_fp8": round(mlp.flops() / (ms_fp8 / 1e3) / 1e12, 1),
        }), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
