"""One small single-GPU workload per kernel, for profiling (ncu) and quick timing.

    python -m nexar_b200.bench.kernels <name> [--iters 3]

names:
  gemm2sm      bf16 8192 x 4096 x 4096 on the CTA-pair tcgen05 kernel
  gemm1sm      the same shape on the 1-SM kernel
  fp8          block-scaled e4m3 8192 x 3584 x 4096 (promotion kernel)
  gemm_rs      fused GEMM -> reduce-scatter with a one-rank communicator
               (8192 x 4096 x 1792: the epilogue stores into the rank's
               staging slot and the kernel reduces it, as on W ranks)
  ag_gemm      fused all-gather -> GEMM with a one-rank communicator
               (8192 x 3584 x 4096 bf16, the TP=8 gate + up projection per GPU:
               the copy warps stage the local shard, the MMA waits on it)
  attn         causal self-attention of one GPT-2 layer (B 8, T 1024, 12
               heads of 64): forward (k_attn_fwd) and backward (k_attn_delta,
               k_attn_bwd, k_attn_dq_out) timed apart on the tcgen05 kernels,
               and torch SDPA (cuDNN) forward and forward + backward
  compress     top-1 % + e4m3 compression of 64 Mi bf16 values
  ln_bwd       LayerNorm backward, 8192 x 768 with the bias-gradient sums

Each run prints one JSON line with the CUDA-event time per launch (after two
warm-up launches). Inputs are a few hundred MB at most.
"""
from __future__ import annotations

import argparse
import json

import torch


def _time(fn, iters):
    fn()
    fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("name")
    ap.add_argument("--iters", type=int, default=3)
    args = ap.parse_args()
    from nexar_b200 import _native, ops
    C = _native.cuda()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    rec = {"kernel": args.name}
    if args.name in ("gemm2sm", "gemm1sm"):
        M, N, K = 8192, 4096, 4096
        A = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        B = torch.randn(N, K, device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        C.gemm_set_2sm(1 if args.name == "gemm2sm" else 0)
        ms = _time(lambda: ops.matmul_nt(A, B, out=out, splits=1), args.iters)
        rec.update(M=M, N=N, K=K, us=round(ms * 1e3, 1), tflops=round(2 * M * N * K / ms / 1e9, 1))
    elif args.name == "fp8":
        M, N, K = 8192, 3584, 4096
        xq, xs = ops.quant_fp8_1x128(torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16))
        wq, ws = ops.quant_fp8_128x128((0.05 * torch.randn(N, K, device=dev, generator=g)).to(torch.bfloat16))
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        ms = _time(lambda: ops.matmul_fp8(xq, xs, wq, ws, out=out), args.iters)
        rec.update(M=M, N=N, K=K, us=round(ms * 1e3, 1), tflops=round(2 * M * N * K / ms / 1e9, 1))
    elif args.name == "gemm_rs":
        from nexar_b200.device import DeviceCommunicator
        comm = DeviceCommunicator(0, 1, 0, exchange=lambda h: [h])
        M, N, K = 8192, 4096, 1792
        A = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        B = (0.05 * torch.randn(N, K, device=dev, generator=g)).to(torch.bfloat16)
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        ms = _time(lambda: comm.gemm_reduce_scatter(A, B, out=out), args.iters)
        comm.check()
        rec.update(M=M, N=N, K=K, us=round(ms * 1e3, 1), tflops=round(2 * M * N * K / ms / 1e9, 1))
    elif args.name == "ag_gemm":
        from nexar_b200.device import DeviceCommunicator
        comm = DeviceCommunicator(0, 1, 0, exchange=lambda h: [h])
        M, N, K = 8192, 14336 // 8 * 2, 4096
        x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        B = (0.05 * torch.randn(N, K, device=dev, generator=g)).to(torch.bfloat16)
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        ms = _time(lambda: comm.all_gather_gemm(x, B, out=out), args.iters)
        comm.check()
        rec.update(M=M, N=N, K=K, us=round(ms * 1e3, 1), tflops=round(2 * M * N * K / ms / 1e9, 1))
    elif args.name == "attn":
        Bn, T, Hn = 8, 1024, 12
        Cn = Hn * 64
        qkv = torch.randn(Bn * T, 3 * Cn, device=dev, generator=g).to(torch.bfloat16)
        dy = torch.randn(Bn * T, Cn, device=dev, generator=g).to(torch.bfloat16)
        y = torch.empty(Bn * T, Cn, device=dev, dtype=torch.bfloat16)
        lse = torch.empty(Bn * Hn * T, device=dev, dtype=torch.float32)
        dqkv = torch.empty_like(qkv)
        ws = torch.empty(C.attn_bwd_workspace_floats(Bn, T, Hn), device=dev, dtype=torch.float32)
        fwd_ms = _time(lambda: C.attn_fwd(qkv, y, lse, Bn, T, Hn, True), args.iters)
        bwd_ms = _time(lambda: C.attn_bwd(qkv, y, dy, lse, dqkv, ws, Bn, T, Hn, True), args.iters)
        qkv_r = qkv.clone().requires_grad_(True)

        def sdpa_fwd():
            x = qkv_r.view(Bn, T, 3, Hn, 64)
            q, k, v = (t.transpose(1, 2) for t in x.unbind(2))
            return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)

        def sdpa_both():
            sdpa_fwd().transpose(1, 2).reshape(Bn * T, Cn).backward(dy)

        with torch.no_grad():
            sdpa_fwd_ms = _time(sdpa_fwd, args.iters)
        sdpa_ms = _time(sdpa_both, args.iters)
        ffl = 4 * Bn * Hn * T * T * 64 / 2  # causal: half of the T x T scores
        rec.update(B=Bn, T=T, H=Hn, fwd_us=round(fwd_ms * 1e3, 1), bwd_us=round(bwd_ms * 1e3, 1),
                   fwd_tflops=round(ffl / fwd_ms / 1e9, 1), bwd_tflops=round(2.5 * ffl / bwd_ms / 1e9, 1),
                   sdpa_fwd_us=round(sdpa_fwd_ms * 1e3, 1), sdpa_fwd_bwd_us=round(sdpa_ms * 1e3, 1),
                   sdpa_bwd_us_incl_autograd=round((sdpa_ms - sdpa_fwd_ms) * 1e3, 1))
    elif args.name == "compress":
        n = 64 << 20
        grad = torch.randn(n, device=dev, generator=g).to(torch.bfloat16)
        res = torch.zeros(n, device=dev)
        k = n // 100
        blob = torch.empty(C.compress_blob_bytes(k), dtype=torch.uint8, device=dev)
        work = torch.empty(C.compress_workspace_bytes(n), dtype=torch.uint8, device=dev)
        ms = _time(lambda: C.topk_fp8_compress(grad, res, k, blob, work), args.iters)
        rec.update(numel=n, k=k, us=round(ms * 1e3, 1), gbs_of_residual_traffic=round(n * 10 / ms / 1e6, 1))
    elif args.name == "ln_bwd":
        R, Cn = 8192, 768
        x = torch.randn(R, Cn, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
        r = torch.randn(R, Cn, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
        w = torch.ones(Cn, device=dev, dtype=torch.bfloat16, requires_grad=True)
        b = torch.zeros(Cn, device=dev, dtype=torch.bfloat16, requires_grad=True)
        rb = torch.zeros(Cn, device=dev, dtype=torch.bfloat16, requires_grad=True)
        s, y = ops.residual_layer_norm(x, r, w, b, 1e-5, rbias=rb)
        dy = torch.randn_like(y)
        ds = torch.randn_like(s)
        ms = _time(lambda: torch.autograd.grad([s, y], [x, w, b, rb], [ds, dy], retain_graph=True), args.iters)
        rec.update(R=R, C=Cn, us=round(ms * 1e3, 1), gbs=round(R * Cn * 2 * 4 / ms / 1e6, 1))
    else:
        raise SystemExit(f"unknown kernel workload {args.name}")
    rec["err_flag"] = int(C.gemm_error_flag())
    print(json.dumps(rec), flush=True)


if __name__ == "__main__":
    main()
