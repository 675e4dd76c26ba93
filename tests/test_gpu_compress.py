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
