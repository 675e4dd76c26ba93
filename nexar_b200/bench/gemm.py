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
    args = ap.parse_args()
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
            for name, fn in (("nexar", lambda: ops.matmul_nt(A, B, out=out, a_t=a_t, b_t=b_t)),
                             ("cublas", lambda: torch.matmul(opA, opBt, out=out))):
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


if __name__ == "__main__":
    main()
