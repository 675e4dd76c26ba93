"""Top-k + fp8 compressed all-reduce against a torch fp32 reference."""
import math
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import gpu_count

pytestmark = pytest.mark.gpu


def _reference(xs, ress, ratio):
    """Per rank: r = res + x; keep the k largest |r|, fp8-quantised with scale max|r|/448."""
    total = None
    new_res = []
    for x, res in zip(xs, ress):
        r = res + x.float()
        n = r.numel()
        k = max(1, math.ceil(n * ratio))
        idx = torch.topk(r.abs(), k).indices
        scale = r.abs().max() / 448.0
        q = (r[idx] / scale).to(torch.float8_e4m3fn).float() * scale
        sent = torch.zeros_like(r)
        sent[idx] = q
        new_res.append(r - sent)
        total = sent if total is None else total + sent
    return total, new_res


def test_compressed_single_rank(cuda0):
    from nexar_b200.device import DeviceCommunicator
    comm = DeviceCommunicator(0, 1, 0, exchange=lambda h: [h], slot_bytes=1 << 20)
    g = torch.Generator(device=cuda0).manual_seed(0)
    n, ratio = 1 << 20, 0.01
    res = torch.zeros(n, device=cuda0)
    for step in range(3):
        x = torch.randn(n, device=cuda0, generator=g).to(torch.bfloat16)
        want, new_res = _reference([x], [res.clone()], ratio)
        out = comm.all_reduce_compressed(x, ratio, res)
        torch.cuda.synchronize()
        # selection is exact up to magnitudes equal in the top 24 bits: allow a few swaps
        mism = (out.float() - want).abs() > 1e-2 * want.abs().max()
        assert mism.sum().item() <= 4, mism.sum().item()
        assert (out != 0).sum().item() <= math.ceil(n * ratio)
        torch.testing.assert_close(res, new_res[0], atol=1e-2, rtol=0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, results):
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    from nexar_b200.device import DeviceCommunicator
    comm = DeviceCommunicator.from_torch(timeout_us=5_000_000, slot_bytes=16 << 20)
    n, ratio = 300_001, 0.02
    xs = [torch.randn(n, device=dev, generator=torch.Generator(device=dev).manual_seed(p)).to(torch.bfloat16)
          for p in range(world)]
    res = torch.zeros(n, device=dev)
    want, _ = _reference(xs, [torch.zeros(n, device=dev) for _ in range(world)], ratio)
    out = comm.all_reduce_compressed(xs[rank], ratio, res, scale=1.0 / world)
    torch.cuda.synchronize()
    err = []
    mism = (out.float() - want / world).abs() > 2e-2 * (want / world).abs().max()
    if mism.sum().item() > 4 * world:
        err.append(f"{mism.sum().item()} mismatches")
    results[rank] = (err, out.float().sum().item())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.multigpu
@pytest.mark.skipif(gpu_count() < 2, reason="needs >= 2 GPUs")
def test_compressed_multi_gpu_identical_on_all_ranks():
    world = min(gpu_count(), 4)
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, start_method="spawn", join=True)
    sums = set()
    for r in range(world):
        err, s = results[r]
        assert err == [], f"rank {r}: {err}"
        sums.add(s)
    assert len(sums) == 1  # bitwise-identical results on every rank


def _distinct_magnitudes(n, device, seed):
    """n values whose |v| differ in the top 24 bits of the fp32 pattern, in random order and sign."""
    i = torch.arange(n, device=device)
    v = torch.ldexp(1.0 + (i % 32768).float() / 32768.0, (i // 32768 - 5).int())
    g = torch.Generator(device=device).manual_seed(seed)
    perm = torch.randperm(n, device=device, generator=g)
    sign = torch.where(torch.rand(n, device=device, generator=g) < 0.5, -1.0, 1.0)
    return v[perm] * sign


def _run_compress(C, grad, res, k):
    dev = grad.device
    blob = torch.zeros(C.compress_blob_bytes(k), dtype=torch.uint8, device=dev)
    work = torch.empty(C.compress_workspace_bytes(grad.numel()), dtype=torch.uint8, device=dev)
    C.topk_fp8_compress(grad, res, k, blob, work)
    torch.cuda.synchronize()
    scale = blob[:4].view(torch.float32).item()
    idx = blob[16:16 + 4 * k].view(torch.int32).long()
    val = blob[16 + 4 * k:16 + 5 * k].view(torch.float8_e4m3fn).float() * scale
    return idx, val, scale


@pytest.mark.parametrize("n,offset", [(1 << 20, 0), (300_007, 0), (300_007, 1), (4097, 3)])
def test_topk_blob_exact_order_and_residual(cuda0, n, offset):
    """Exact selection when magnitudes are distinct: ascending indices, e4m3 values, residual.

    offset > 0 passes views that are not 16-byte aligned (the scalar load path)."""
    from nexar_b200 import _native
    C = _native.cuda()
    k = max(1, n // 50)
    store = torch.zeros(n + offset, device=cuda0)
    store[offset:] = _distinct_magnitudes(n, cuda0, seed=n)
    gstore = torch.zeros(n + offset, device=cuda0, dtype=torch.bfloat16)
    res, grad = store[offset:], gstore[offset:]
    r = res.clone()
    idx, val, scale = _run_compress(C, grad, res, k)
    want_idx = torch.topk(r.abs(), k).indices.sort().values
    assert torch.equal(idx, want_idx)
    want_scale = r.abs().max().item() / 448.0
    assert abs(scale - want_scale) <= 1e-6 * want_scale
    q = (r[want_idx] / scale).to(torch.float8_e4m3fn).float() * scale
    # r * (1/scale) on the device may round to the neighbouring e4m3 value at a
    # rounding boundary: allow a few one-step differences.
    off = (val - q).abs() > 1e-6 * q.abs()
    assert off.sum().item() <= 2 + k // 1000
    assert ((val - q).abs() <= 0.13 * q.abs()).all()
    want_res = r.clone()
    want_res[want_idx] -= val
    # the device fuses r - q * scale (one rounding); torch rounds q * scale
    # first: they differ by at most an ulp of |r| (magnitudes reach 2^26 here)
    assert ((res - want_res).abs() <= 2.0 ** -22 * r.abs() + 1e-6).all()


def test_topk_ties_taken_in_index_order(cuda0):
    """Mostly-zero input (an embedding gradient's unused rows): the k-th value is a tie
    shared by ~all elements; the lowest indices among the ties are taken."""
    from nexar_b200 import _native
    C = _native.cuda()
    n, k = 1 << 20, 1000
    g = torch.Generator(device=cuda0).manual_seed(3)
    nz = torch.randperm(n, device=cuda0, generator=g)[:100]
    res = torch.zeros(n, device=cuda0)
    res[nz] = torch.rand(100, device=cuda0, generator=g) + 1.0
    grad = torch.zeros(n, device=cuda0, dtype=torch.bfloat16)
    idx, val, _ = _run_compress(C, grad, res.clone(), k)
    zero_mask = torch.ones(n, dtype=torch.bool, device=cuda0)
    zero_mask[nz] = False
    first_zeros = torch.nonzero(zero_mask).flatten()[:k - 100]
    want = torch.cat([nz, first_zeros]).sort().values
    assert torch.equal(idx, want)
    assert (val[torch.isin(idx, nz)] > 0).all()
