"""tcgen05 GEMM throughput vs cuBLAS (torch.matmul) on one GPU.

    python -m nexar_b200.bench.gemm [--shapes 8192x8192x8192,8192x2304x768,...] [--iters 50]

Each point: 5 warm-up launches, then `iters` back-to-back launches between
CUDA events. Inputs are larger than L2 for the big shapes; reported TFLOP/s =
2*M*N*K / time.
"""
import argparse
import json

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="8192x8192x8192,8192x2304x768,8192x768x768,8192x3072x768,8192x768x3072,"
                                        "8192x50304x768,8192x3584x4096,8192x4096x1792")
    ap.add_argument("--iters", type=int, default=30)
    args = ap.parse_args()
    from nexar_b200 import _native
    C = _native.cuda()
    dev = torch.device("cuda", 0)
    for s in args.shapes.split(","):
        M, N, K = (int(x) for x in s.split("x"))
        A = torch.randn(M, K, device=dev).to(torch.bfloat16)
        B = torch.randn(N, K, device=dev).to(torch.bfloat16)
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        res = {}
        for name, fn in (("nexar", lambda: C.gemm(A, B, out)), ("cublas", lambda: torch.matmul(A, B.t(), out=out))):
            for _ in range(5):
                fn()
            torch.cuda.synchronize()
            st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            st.record()
            for _ in range(args.iters):
                fn()
            en.record()
            torch.cuda.synchronize()
            ms = st.elapsed_time(en) / args.iters
            res[name] = {"us": round(ms * 1e3, 1), "tflops": round(2 * M * N * K / (ms / 1e3) / 1e12, 1)}
        print(json.dumps({"M": M, "N": N, "K": K, **res, "err_flag": int(C.gemm_error_flag())}), flush=True)


if __name__ == "__main__":
    main()
