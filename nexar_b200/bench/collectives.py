"""Device collective sweep: nexar_b200 peer-memory kernels vs NCCL (1 KB - 1 GB, 2/4/8 GPUs).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m nexar_b200.bench.collectives \
        [--ops all_reduce,reduce_scatter,all_gather,all_to_all,broadcast] [--dtype bf16]
        [--min-bytes 1024] [--max-bytes 1073741824] [--iters 100] [--warmup 20] [--out file.jsonl]

The NCCL arm issues the same call sequence as the reference's nexar-nccl
single-node path (ncclAllReduce / ncclReduceScatter / ncclAllGather /
ncclBroadcast in place on one stream; all_to_all as grouped send/recv),
through torch.distributed's NCCL backend. The ``nccl_group`` arm issues it through
``nexar_b200.device.nccl.NcclGroup`` (raw ncclAllReduce / ncclReduceScatter /
ncclAllGather / ncclBroadcast on device pointers, in place where the reference
is, on the timed stream; nexar-nccl has no device all_to_all, so that arm
skips it). The ``nexar_sym`` arm runs the same
calls on buffers allocated in symmetric memory (the NVSwitch multicast region
when NVLS is the preferred path, else the peer-mapped heap), the equivalent of NCCL's
registered buffers: no staging copies. Both arms are timed the same way:
warm-up iterations, then `reps` windows of `iters` back-to-back launches
between CUDA events, max over ranks per window, median window reported. Bus bandwidth follows the nccl-tests convention.
"""
from __future__ import annotations

import argparse
import json
import os
import sys


def busbw_factor(op: str, n: int) -> float:
    if op == "all_reduce":
        return 2.0 * (n - 1) / n
    if op in ("reduce_scatter", "all_gather", "all_to_all"):
        return (n - 1) / n
    return 1.0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--ops", default="all_reduce,reduce_scatter,all_gather,all_to_all,broadcast")
    ap.add_argument("--dtype", default="bf16")
    ap.add_argument("--min-bytes", type=int, default=1024)
    ap.add_argument("--max-bytes", type=int, default=1 << 30)
    ap.add_argument("--step", type=int, default=2, help="size multiplier between points")
    ap.add_argument("--iters", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--reps", type=int, default=3,
                    help="timing windows of `iters` calls each; the median window (max over ranks) is reported")
    ap.add_argument("--impls", default="nexar,nexar_sym,nccl",
                    help="comma list of nexar, nexar_sym, nccl, nccl_group")
    ap.add_argument("--algo", default="auto")
    ap.add_argument("--out", default=None)
    args = ap.parse_args(argv)

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    # Every arm runs on (and is timed on) one non-default stream: the raw
    # NcclGroup calls go to the stream it was given, which must have a handle.
    torch.cuda.set_stream(torch.cuda.Stream(dev))
    from nexar_b200.device import DeviceCommunicator
    comm = DeviceCommunicator.from_torch()
    dtype = {"bf16": torch.bfloat16, "f32": torch.float32, "f16": torch.float16}[args.dtype]
    es = torch.empty((), dtype=dtype).element_size()
    out_f = open(args.out, "a") if (args.out and rank == 0) else None
    g = torch.Generator(device=dev).manual_seed(rank)

    def time_it(fn):
        for _ in range(args.warmup):
            fn()
        windows = []
        for _ in range(max(1, args.reps)):
            torch.cuda.synchronize()
            dist.barrier()
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(args.iters):
                fn()
            e.record()
            torch.cuda.synchronize()
            t = torch.tensor([s.elapsed_time(e) / args.iters], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            windows.append(float(t.item()))
        # A single late launch on one rank (host scheduling) stalls every
        # rank's spinning kernels for that window; the median window is the
        # steady-state figure, and every arm is measured the same way.
        return sorted(windows)[len(windows) // 2]

    ops = args.ops.split(",")
    impls = args.impls.split(",")
    group = None
    if "nccl_group" in impls:
        from nexar_b200.core import DataType
        from nexar_b200.device import nccl as nccl_mod
        uid = [nccl_mod.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        group = nccl_mod.NcclGroup(rank, world, uid[0], device=local, stream=torch.cuda.current_stream(dev))
        gdt = DataType.from_torch(dtype)

    def pick(impl, ours, torch_nccl, raw=None):
        if impl == "nexar":
            return ours
        if impl == "nccl":
            return torch_nccl
        return raw

    def sym_buf(numel):
        return comm.symmetric_empty([numel], dtype, nvls=comm.nvls_preferred)

    def sym_reset():
        if comm.nvls_preferred:
            comm.native.nvls_reset()
        else:
            comm.native.reset_symmetric()
    size = args.min_bytes
    while size <= args.max_bytes:
        n = max(world, size // es)
        n = (n // world) * world
        big = torch.randn(n, device=dev, generator=g).to(dtype)
        for op in ops:
            for impl in impls:
                if impl == "nexar_sym":
                    if op == "all_to_all":
                        continue
                    if op == "all_reduce":
                        t = sym_buf(n)
                        t.copy_(big)
                        fn = lambda: comm.all_reduce(t)  # noqa: E731
                    elif op == "reduce_scatter":
                        inp = sym_buf(n)
                        inp.copy_(big)
                        out = torch.empty(n // world, dtype=dtype, device=dev)
                        fn = lambda: comm.reduce_scatter(inp, out)  # noqa: E731
                    elif op == "all_gather":
                        inp = big[: n // world].clone()
                        out = sym_buf(n)
                        fn = lambda: comm.all_gather(inp, out)  # noqa: E731
                    else:
                        t = sym_buf(n)
                        t.copy_(big)
                        fn = lambda: comm.broadcast(t, 0)  # noqa: E731
                    nbytes = n * es
                elif op == "all_reduce":
                    t = big.clone()
                    fn = pick(impl, lambda: comm.all_reduce(t, algo=args.algo), lambda: dist.all_reduce(t),
                              lambda: group.allreduce_inplace(t.data_ptr(), n, gdt))
                    nbytes = n * es
                elif op == "reduce_scatter":
                    out = torch.empty(n // world, dtype=dtype, device=dev)
                    fn = pick(impl, lambda: comm.reduce_scatter(big, out), lambda: dist.reduce_scatter_tensor(out, big),
                              lambda: group.reduce_scatter_ptr(big.data_ptr(), out.data_ptr(), n // world, gdt))
                    nbytes = n * es
                elif op == "all_gather":
                    inp = big[: n // world].clone()
                    out = torch.empty(n, dtype=dtype, device=dev)
                    fn = pick(impl, lambda: comm.all_gather(inp, out), lambda: dist.all_gather_into_tensor(out, inp),
                              lambda: group.allgather(inp.data_ptr(), out.data_ptr(), n // world, gdt))
                    nbytes = n * es
                elif op == "all_to_all":
                    out = torch.empty_like(big)
                    fn = pick(impl, lambda: comm.all_to_all(big, out), lambda: dist.all_to_all_single(out, big))
                    nbytes = n * es
                elif op == "broadcast":
                    t = big.clone()
                    fn = pick(impl, lambda: comm.broadcast(t, 0), lambda: dist.broadcast(t, 0),
                              lambda: group.broadcast_inplace(t.data_ptr(), n, gdt, 0))
                    nbytes = n * es
                else:
                    raise SystemExit(f"unknown op {op}")
                if fn is None:
                    continue
                ms = time_it(fn)
                if impl == "nexar_sym":
                    torch.cuda.synchronize()
                    sym_reset()
                algbw = nbytes / (ms / 1e3) / 1e9
                rec = {"op": op, "impl": impl, "dtype": args.dtype, "bytes": nbytes, "n_gpus": world,
                       "us": round(ms * 1e3, 2), "algbw_gbs": round(algbw, 2),
                       "busbw_gbs": round(algbw * busbw_factor(op, world), 2)}
                if rank == 0:
                    print(json.dumps(rec), flush=True)
                    if out_f:
                        out_f.write(json.dumps(rec) + "\n")
        del big
        size *= args.step
    comm.check()
    if group is not None:
        group.destroy()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
