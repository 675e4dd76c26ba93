"""tcgen05 GEMM throughput vs cuBLAS (torch.matmul) on one GPU.

    python -m nexar_b200.bench.gemm [--shapes 8192x8192x8192,...] [--majors nt,nn,tn,tt] [--iters 30]

C[M, N] = opA . opB^T. Major code: first letter for A, second for B; "n" =
stored as the logical operand (K-major: A [M, K], B [N, K]), "t" = stored
transposed (MN-major: A as [K, M], B as [K, N]). The backward pass of a
linear layer uses "nt" (dX = dY . W) and "tt" (dW = dY^T . X). Split-K is
chosen by the kernel's cost model. Each point: 5 warm-up launches, then
`iters` back-to-back launches between CUDA events; TFLOP/s = 2*M*N*K / time.
"""
import argparse
import json

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="8192x8192x8192,8192x2304x768,8192x768x768,8192x3072x768,8192x768x3072,"
                                        "8192x50304x768,8192x3584x4096,8192x4096x1792")
    ap.add_argument("--majors", default="nn")
    ap.add_argument("--iters", type=int, default=30)
    ap.add_argument("--pair", action="store_true", help="also time the 2-SM (CTA pair) kernel")
    ap.add_argument("--fp8", action="store_true",
                    help="block-scaled e4m3 GEMM (1x128 / 128x128 scales) vs torch._scaled_mm and bf16 cuBLAS")
    args = ap.parse_args()
    if args.fp8:
        return bench_fp8(args)
    from nexar_b200 import _native, ops
    C = _native.cuda()
    dev = torch.device("cuda", 0)
    for s in args.shapes.split(","):
        M, N, K = (int(x) for x in s.split("x"))
        for mj in args.majors.split(","):
            a_t, b_t = mj[0] == "t", mj[1] == "t"
            A = torch.randn(K, M, device=dev).to(torch.bfloat16) if a_t else torch.randn(M, K, device=dev).to(torch.bfloat16)
            B = torch.randn(K, N, device=dev).to(torch.bfloat16) if b_t else torch.randn(N, K, device=dev).to(torch.bfloat16)
            out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
            opA = A.t() if a_t else A
            opBt = B if b_t else B.t()
            splits = C.gemm_choose_splits(M, N, K)
            res = {}
            arms = [("nexar", lambda: ops.matmul_nt(A, B, out=out, a_t=a_t, b_t=b_t)),
                    ("cublas", lambda: torch.matmul(opA, opBt, out=out))]
            if args.pair:
                def pair_fn():
                    C.gemm_set_2sm(1)
                    try:
                        ops.matmul_nt(A, B, out=out, a_t=a_t, b_t=b_t)
                    finally:
                        C.gemm_set_2sm(0)
                arms.insert(1, ("nexar_2sm", pair_fn))
            for name, fn in arms:
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
            print(json.dumps({"M": M, "N": N, "K": K, "majors": mj, "splits": splits, **res,
                              "err_flag": int(C.gemm_error_flag())}), flush=True)


def _time(fn, iters):
    for _ in range(5):
        fn()
    torch.cuda.synchronize()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(iters):
        fn()
    en.record()
    torch.cuda.synchronize()
    return st.elapsed_time(en) / iters


def bench_fp8(args):
    from nexar_b200 import _native, ops
    dev = torch.device("cuda", 0)
    for s in args.shapes.split(","):
        M, N, K = (int(x) for x in s.split("x"))
        x = torch.randn(M, K, device=dev).to(torch.bfloat16)
        w = (0.05 * torch.randn(N, K, device=dev)).to(torch.bfloat16)
        xq, xs = ops.quant_fp8_1x128(x)
        wq, ws = ops.quant_fp8_128x128(w)
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        res = {}
        ms = _time(lambda: ops.matmul_fp8(xq, xs, wq, ws, out=out), args.iters)
        res["nexar_fp8_blockscaled"] = {"us": round(ms * 1e3, 1), "tflops": round(2 * M * N * K / ms / 1e9, 1)}
        ms = _time(lambda: torch.matmul(x, w.t(), out=out), args.iters)
        res["cublas_bf16"] = {"us": round(ms * 1e3, 1), "tflops": round(2 * M * N * K / ms / 1e9, 1)}
        try:  # library fp8 with row-wise scales (the closest scaled-mm recipe torch exposes)
            sa = torch.ones(M, 1, device=dev)
            sb = torch.ones(1, N, device=dev)
            ms = _time(lambda: torch._scaled_mm(xq, wq.t(), scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16),
                       args.iters)
            res["torch_scaled_mm_rowwise"] = {"us": round(ms * 1e3, 1), "tflops": round(2 * M * N * K / ms / 1e9, 1)}
        except Exception as e:  # noqa: BLE001
            res["torch_scaled_mm_rowwise"] = f"unavailable: {str(e)[:80]}"
        print(json.dumps({"M": M, "N": N, "K": K, **res, "err_flag": int(_native.cuda().gemm_error_flag())}),
              flush=True)


if __name__ == "__main__":
    main()
