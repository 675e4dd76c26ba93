"""Device collectives against a CPU fp64/exact oracle.

Multi-rank cases run one process per GPU (never two ranks on one GPU: the
kernels wait on each other and must be co-resident). Data is rank- and
index-dependent so chunk-placement errors are caught (e.g. reduce_scatter
must give rank r chunk r).
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import gpu_count

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data(rank, n, dtype, seed=0):
    g = torch.Generator().manual_seed(seed * 1000 + rank)
    if dtype.is_floating_point:
        return (torch.randn(n, generator=g, dtype=torch.float64) + rank * 0.25).to(dtype)
    return torch.randint(-50, 50, (n,), generator=g, dtype=torch.int64).to(dtype)


def _oracle_reduce(xs, op):
    acc = xs[0].double() if xs[0].is_floating_point() else xs[0].long()
    for x in xs[1:]:
        y = x.double() if x.is_floating_point() else x.long()
        if op == "sum":
            acc = acc + y
        elif op == "prod":
            acc = acc * y
        elif op == "min":
            acc = torch.minimum(acc, y)
        else:
            acc = torch.maximum(acc, y)
    return acc


def _tol(dtype, world):
    if dtype == torch.bfloat16:
        return dict(atol=3e-2 * world, rtol=2e-2)
    if dtype == torch.float16:
        return dict(atol=5e-3 * world, rtol=5e-3)
    return dict(atol=1e-5 * world, rtol=1e-5)


def _worker(rank, world, port, results):
    import torch.distributed as dist
    from nexar_b200.device import DeviceCommunicator
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    dev = torch.device("cuda", rank)
    comm = DeviceCommunicator.from_torch(timeout_us=5_000_000, slot_bytes=8 << 20)
    errors = []

    def check(name, got, want, **tol):
        try:
            torch.testing.assert_close(got.cpu().double() if got.is_floating_point() else got.cpu().long(),
                                       want.double() if want.is_floating_point() else want.long(), **tol)
        except AssertionError as e:
            errors.append(f"{name}: {str(e)[:300]}")

    for dtype in (torch.float32, torch.bfloat16, torch.float16, torch.int32):
        for n in (1, 7, 4095, 1 << 16, 3 * (1 << 20) + 5):
            xs = [_data(r, n, dtype) for r in range(world)]
            ops_ = ("sum", "max") if dtype != torch.int32 else ("sum", "min", "prod")
            for op in ops_:
                for algo in ("oneshot", "twoshot"):
                    t = xs[rank].to(dev)
                    comm.all_reduce(t, op=op, algo=algo)
                    want = _oracle_reduce(xs, op)
                    if dtype == torch.int32 and op == "prod":
                        want = want.to(torch.int32)  # wrapping semantics
                    check(f"all_reduce {dtype} n={n} {op} {algo}", t, want, **_tol(dtype, world))
        # fused scale + cast (bf16 in, fp32 out)
    n = 100003
    xs = [_data(r, n, torch.bfloat16) for r in range(world)]
    out = torch.empty(n, dtype=torch.float32, device=dev)
    comm.all_reduce(xs[rank].to(dev), out=out, scale=1.0 / world)
    check("all_reduce bf16->f32 scaled", out, _oracle_reduce(xs, "sum") / world, atol=2e-2, rtol=1e-2)
    # symmetric in-place two-shot
    sym = comm.symmetric_empty([n], torch.bfloat16)
    sym.copy_(xs[rank].to(dev))
    comm.all_reduce(sym, scale=0.5, algo="twoshot")
    check("all_reduce symmetric twoshot", sym, _oracle_reduce(xs, "sum") * 0.5, **_tol(torch.bfloat16, world))
    sym.copy_(xs[rank].to(dev))
    comm.all_reduce(sym, algo="oneshot")
    check("all_reduce symmetric oneshot", sym, _oracle_reduce(xs, "sum"), **_tol(torch.bfloat16, world))

    for dtype in (torch.float32, torch.bfloat16, torch.int64, torch.uint8):
        for count in (1, 5, 1000, 1 << 18):
            xs = [_data(r, count * world, dtype, seed=3) for r in range(world)]
            # reduce_scatter: rank r gets chunk r
            if dtype != torch.uint8:
                out = comm.reduce_scatter(xs[rank].to(dev))
                want = _oracle_reduce(xs, "sum")[rank * count:(rank + 1) * count]
                check(f"reduce_scatter {dtype} {count}", out, want, **_tol(dtype, world))
            # all_gather
            mine = xs[rank][:count]
            out = comm.all_gather(mine.to(dev))
            want = torch.cat([xs[r][:count] for r in range(world)])
            check(f"all_gather {dtype} {count}", out, want, atol=0, rtol=0)
            # all_to_all: out[p] = in_p[rank]
            out = comm.all_to_all(xs[rank].to(dev))
            want = torch.cat([xs[p][rank * count:(rank + 1) * count] for p in range(world)])
            check(f"all_to_all {dtype} {count}", out, want, atol=0, rtol=0)
            for root in (0, world - 1):
                # broadcast
                t = xs[rank][:count].clone().to(dev)
                comm.broadcast(t, root=root)
                check(f"broadcast {dtype} {count} root{root}", t, xs[root][:count], atol=0, rtol=0)
                # gather
                out = comm.gather(xs[rank][:count].to(dev), root=root)
                if rank == root:
                    check(f"gather {dtype} {count}", out, torch.cat([xs[r][:count] for r in range(world)]), atol=0, rtol=0)
                # scatter
                out = comm.scatter(xs[rank].to(dev), root=root)
                check(f"scatter {dtype} {count}", out, xs[root][rank * count:(rank + 1) * count], atol=0, rtol=0)
                # reduce
                if dtype != torch.uint8:
                    t = xs[rank][:count].clone().to(dev)
                    comm.reduce(t, root=root)
                    if rank == root:
                        check(f"reduce {dtype} {count}", t, _oracle_reduce([x[:count] for x in xs], "sum"), **_tol(dtype, world))
            if dtype in (torch.float32, torch.int64):
                out = comm.scan(xs[rank][:count].to(dev))
                check(f"scan {dtype} {count}", out, _oracle_reduce([x[:count] for x in xs[:rank + 1]], "sum"), **_tol(dtype, world))
                out = comm.exclusive_scan(xs[rank][:count].to(dev))
                zero = torch.zeros(count, dtype=torch.float64 if dtype.is_floating_point else torch.int64)
                want = zero if rank == 0 else _oracle_reduce([x[:count] for x in xs[:rank]], "sum")
                check(f"exscan {dtype} {count}", out, want, **_tol(dtype, world))
    comm.barrier()
    # non-blocking handle
    t = xs[rank][:1000].clone().to(dev) if xs[rank].is_floating_point() else torch.ones(1000, device=dev)
    h = comm.all_reduce_nb(t)
    h.wait()
    torch.cuda.synchronize()
    # non-blocking and blocking collectives in flight together: an all_reduce_nb
    # (side stream), then a blocking all_reduce (current stream) before wait(),
    # then two overlapping non-blocking ones; each against the fp64 oracle
    n = 4 << 20
    xa = [_data(r, n, torch.float32, seed=7) for r in range(world)]
    xb = [_data(r, n, torch.float32, seed=8) for r in range(world)]
    xc = [_data(r, n, torch.float32, seed=9) for r in range(world)]
    xd = [_data(r, n, torch.float32, seed=10) for r in range(world)]
    a, b, c, d = (v[rank].to(dev) for v in (xa, xb, xc, xd))
    d_out = torch.empty(n // world, device=dev)
    ha = comm.all_reduce_nb(a)
    comm.all_reduce(b, scale=0.5)
    hc = comm.all_reduce_nb(c, op="max")
    hd = comm.reduce_scatter_nb(d, d_out)
    for hh in (ha, hc, hd):
        hh.wait()
    torch.cuda.synchronize()
    check("nb all_reduce (then blocking)", a, _oracle_reduce(xa, "sum"), **_tol(torch.float32, world))
    check("blocking all_reduce while nb in flight", b, _oracle_reduce(xb, "sum") * 0.5, **_tol(torch.float32, world))
    check("overlapping nb all_reduce max", c, _oracle_reduce(xc, "max"), atol=0, rtol=0)
    check("overlapping nb reduce_scatter", d_out, _oracle_reduce(xd, "sum")[rank * (n // world):(rank + 1) * (n // world)],
          **_tol(torch.float32, world))
    try:
        comm.check()
    except Exception as e:  # noqa: BLE001
        errors.append(f"status: {e}")
    results[rank] = errors
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.multigpu
@pytest.mark.skipif(gpu_count() < 2, reason="needs >= 2 GPUs")
def test_device_collectives_multi_gpu():
    world = min(gpu_count(), 4)
    port = _free_port()
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    mp.start_processes(_worker, args=(world, port, results), nprocs=world, start_method="spawn", join=True)
    for r in range(world):
        assert results.get(r) == [], f"rank {r}: {results.get(r)}"


def test_world1_allreduce_scale_cast(cuda0):
    from nexar_b200.device import DeviceCommunicator
    comm = DeviceCommunicator(0, 1, 0, exchange=lambda h: [h], slot_bytes=1 << 20)
    x = torch.randn(4097, device=cuda0).to(torch.bfloat16)
    out = torch.empty(4097, device=cuda0, dtype=torch.float32)
    comm.all_reduce(x, out=out, scale=0.5)
    torch.testing.assert_close(out, x.float() * 0.5)
    comm.check()
    st = comm.stats()
    assert st["all_reduce"] == {"calls": 1, "bytes": 4097 * 2}
    assert st["all_reduce_algorithms"] == {"local": 1}
    sym = comm.symmetric_empty([1024], torch.float32)
    gp = comm.global_ptr(sym, 0)
    assert gp.address() == sym.data_ptr() and gp.nbytes == 4096


def test_device_wait_timeout_reports_error(cuda0):
    """A barrier whose peer flag is never written gives up after the bounded
    wait, records the failure in the status word and leaves the context usable.

    Rank 1 is this process's own heap, and nothing ever writes the flag that
    rank 0 waits for, so exactly one kernel runs and its wait times out.
    """
    from nexar_b200.core import CollectiveFailed
    from nexar_b200.device import DeviceCommunicator
    holder = {}

    def exchange(h):
        holder["h"] = h
        return [h, h]

    comm = DeviceCommunicator(0, 2, 0, exchange=exchange, slot_bytes=1 << 20, timeout_us=300_000)
    comm.barrier()
    torch.cuda.synchronize()
    with pytest.raises(CollectiveFailed):
        comm.check()
    st = comm.status()
    assert st["code"] == 1 and st["rank"] == 1
    # the context still works
    y = torch.ones(10, device=cuda0) * 2
    assert float(y.sum()) == 20.0


def _nvls_worker(rank, world, port, results):
    """NVLS paths forced for every 16-byte-aligned message (nvls_min_bytes = 0)."""
    import torch.distributed as dist
    from nexar_b200.device import DeviceCommunicator
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    dev = torch.device("cuda", rank)
    comm = DeviceCommunicator.from_torch(timeout_us=5_000_000, slot_bytes=8 << 20)
    errors = []
    if not comm.nvls:
        results[rank] = ("no-nvls", [comm.nvls_reason])
        dist.barrier()
        dist.destroy_process_group()
        return
    for k in ("nvls_min_bytes", "nvls_min_rs_bytes", "nvls_min_ag_bytes", "nvls_min_bcast_bytes"):
        setattr(comm.native, k, 0)

    def check(name, got, want, **tol):
        try:
            torch.testing.assert_close(got.cpu().double(), want.double(), **tol)
        except AssertionError as e:
            errors.append(f"{name}: {str(e)[:300]}")

    # staged all-reduce, several sizes in a row (round counters, slot reuse across calls)
    for rep in range(2):
        for dtype in (torch.float32, torch.bfloat16, torch.float16):
            for n in (8, 4096, 1 << 20, 3 * (1 << 20) + 64, 40 << 20 if dtype != torch.float32 else 24 << 20):
                xs = [_data(r, n, dtype, seed=rep) for r in range(world)]
                t = xs[rank].to(dev)
                out = torch.empty_like(t)
                comm.all_reduce(t, out=out, scale=1.0 / world)
                check(f"nvls all_reduce {dtype} n={n}", out, _oracle_reduce(xs, "sum") / world, **_tol(dtype, world))
    # in place on an NVLS-resident tensor (no staging)
    n = 5 * (1 << 20) + 8
    xs = [_data(r, n, torch.bfloat16, seed=7) for r in range(world)]
    sym = comm.symmetric_empty([n], torch.bfloat16, nvls=True)
    assert comm.native.nvls_offset(sym) >= 0
    for _ in range(3):
        sym.copy_(xs[rank].to(dev))
        comm.all_reduce(sym, scale=0.5)
        check("nvls all_reduce in place", sym, _oracle_reduce(xs, "sum") * 0.5, **_tol(torch.bfloat16, world))
    # CUDA graph replay of an in-place NVLS all-reduce
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        comm.all_reduce(sym)
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(g):
        comm.all_reduce(sym)
    for _ in range(3):
        sym.copy_(xs[rank].to(dev))
        g.replay()
        torch.cuda.synchronize()
        check("nvls all_reduce graph replay", sym, _oracle_reduce(xs, "sum"), **_tol(torch.bfloat16, world))
    del g
    # reduce-scatter / all-gather / broadcast
    for dtype in (torch.float32, torch.bfloat16):
        for count in (8, 1 << 16, (1 << 20) + 8):
            xs = [_data(r, count * world, dtype, seed=3) for r in range(world)]
            out = comm.reduce_scatter(xs[rank].to(dev))
            check(f"nvls reduce_scatter {dtype} {count}", out,
                  _oracle_reduce(xs, "sum")[rank * count:(rank + 1) * count], **_tol(dtype, world))
            out = comm.all_gather(xs[rank][:count].to(dev))
            check(f"nvls all_gather {dtype} {count}", out, torch.cat([xs[r][:count] for r in range(world)]),
                  atol=0, rtol=0)
            for root in (0, world - 1):
                t = xs[rank][:count].clone().to(dev)
                comm.broadcast(t, root=root)
                check(f"nvls broadcast {dtype} {count} root{root}", t, xs[root][:count], atol=0, rtol=0)
    # zero-copy variants: NVLS-resident RS input, AG output, broadcast buffer
    count = (1 << 19) + 8
    xs = [_data(r, count * world, torch.bfloat16, seed=5) for r in range(world)]
    rin = comm.symmetric_empty([count * world], torch.bfloat16, nvls=True)
    agout = comm.symmetric_empty([count * world], torch.bfloat16, nvls=True)
    bbuf = comm.symmetric_empty([count], torch.bfloat16, nvls=True)
    for _ in range(2):
        rin.copy_(xs[rank].to(dev))
        out = comm.reduce_scatter(rin)
        check("nvls reduce_scatter resident", out, _oracle_reduce(xs, "sum")[rank * count:(rank + 1) * count],
              **_tol(torch.bfloat16, world))
        comm.all_gather(xs[rank][:count].to(dev), agout)
        check("nvls all_gather resident", agout, torch.cat([xs[r][:count] for r in range(world)]), atol=0, rtol=0)
        for root in (0, world - 1):
            bbuf.copy_(xs[rank][:count].to(dev))
            comm.broadcast(bbuf, root=root)
            check(f"nvls broadcast resident root{root}", bbuf, xs[root][:count], atol=0, rtol=0)
    torch.cuda.synchronize()
    try:
        comm.check()
    except Exception as e:  # noqa: BLE001
        errors.append(f"status: {e}")
    results[rank] = ("nvls", errors)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.multigpu
@pytest.mark.skipif(gpu_count() < 2, reason="needs >= 2 GPUs")
def test_nvls_collectives_multi_gpu():
    world = gpu_count()
    port = _free_port()
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_nvls_worker, args=(world, port, results), nprocs=world, start_method="spawn", join=True)
    modes = {results[r][0] for r in range(world)}
    assert len(modes) == 1, modes
    if modes == {"no-nvls"}:
        pytest.skip(f"NVSwitch multicast not available on this box: {results[0][1]}")
    for r in range(world):
        assert results[r][1] == [], f"rank {r}: {results[r][1]}"
