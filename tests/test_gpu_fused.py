"""Fused GEMM + collective kernels (GEMM->reduce-scatter, all-gather->GEMM)
and the TP Llama MLP block, against fp32 references, on >= 2 GPUs."""
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import gpu_count

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rand(shape, seed, dev, scale=1.0):
    g = torch.Generator(device=dev).manual_seed(seed)
    return (scale * torch.randn(*shape, device=dev, generator=g)).to(torch.bfloat16)


def _worker(rank, world, port, results):
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    from nexar_b200.device import DeviceCommunicator
    from nexar_b200 import _native
    comm = DeviceCommunicator.from_torch(timeout_us=5_000_000, slot_bytes=64 << 20)
    errs = []

    def check(name, got, want, atol, rtol=2e-2):
        try:
            torch.testing.assert_close(got.float(), want.float(), atol=atol, rtol=rtol)
        except AssertionError as e:
            errs.append(f"{name}: {str(e)[:400]}")

    for (M, N, K) in [(world * 128, 256, 128), (world * 256, 768, 512), (world * 384, 640, 1024)]:
        # GEMM -> RS: rank r gets rows [r*M/W, (r+1)*M/W) of sum_p A_p @ B_p^T
        for rep in range(2):
            A = _rand((M, K), 100 + rank + rep, dev)
            B = _rand((N, K), 200 + rank + rep, dev, 0.1)
            bias = _rand((N,), 7, dev)
            out = comm.gemm_reduce_scatter(A, B, bias=bias)
            torch.cuda.synchronize()
            ref = torch.zeros(M, N, device=dev)
            for p in range(world):
                ref += _rand((M, K), 100 + p + rep, dev).float() @ _rand((N, K), 200 + p + rep, dev, 0.1).float().t()
            rpr = M // world
            ref = ref[rank * rpr:(rank + 1) * rpr] + bias.float()
            check(f"gemm_rs {M}x{N}x{K} rep{rep}", out, ref, atol=0.05 * world)
        # AG -> GEMM: out = cat_p(x_p) @ B^T
        for rep in range(2):
            x = _rand((M // world, K), 300 + rank + rep, dev)
            B = _rand((N, K), 400 + rep, dev, 0.1)
            out = comm.all_gather_gemm(x, B)
            torch.cuda.synchronize()
            xf = torch.cat([_rand((M // world, K), 300 + p + rep, dev) for p in range(world)]).float()
            check(f"ag_gemm {M}x{N}x{K} rep{rep}", out, xf @ B.float().t(), atol=0.08)
    # TP MLP block vs the NCCL + cuBLAS formulation
    from nexar_b200.models.llama_mlp import LlamaMLPConfig, TPLlamaMLP
    cfg = LlamaMLPConfig(d_model=512, ffn=1024 * world, tokens=256 * world)
    mlp = TPLlamaMLP(cfg, comm, seed=3)
    x = _rand((cfg.tokens // world, cfg.d_model), 900 + rank, dev)
    y = mlp.forward(x)
    yb = mlp.forward_baseline(x)
    torch.cuda.synchronize()
    check("tp_mlp fused vs baseline", y, yb, atol=2e-2, rtol=5e-2)
    # fp8 block-scaled block: against an fp32 evaluation of the same quantised math
    from nexar_b200 import ops
    import torch.distributed as dist
    yf8 = mlp.forward_fp8(x)
    torch.cuda.synchronize()
    (wuq, wus), (wdq, wds) = mlp.fp8_weights()

    def deq(q, s, bm):
        R, K = q.shape
        f = q.float()
        sr = s.repeat_interleave(bm, 0)[:R] if bm > 1 else s
        return f * sr.repeat_interleave(128, 1)[:, :K]

    xs_all = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(xs_all, x)
    xfull = torch.cat(xs_all)
    xq, xsc = ops.quant_fp8_1x128(xfull)
    gu = deq(xq, xsc, 1) @ deq(wuq, wus, 128).t()
    F = mlp.F
    h = torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]
    hq, hs = ops.quant_fp8_1x128(h.to(torch.bfloat16))
    yp = deq(hq, hs, 1) @ deq(wdq, wds, 128).t()
    yp_all = [torch.empty_like(yp) for _ in range(world)]
    dist.all_gather(yp_all, yp.contiguous())
    rpr = cfg.tokens // world
    yref = sum(yp_all)[rank * rpr:(rank + 1) * rpr]
    check("tp_mlp fp8 vs fp32 of the quantised math", yf8, yref, atol=3e-2, rtol=5e-2)
    rel = ((yf8.float() - yb.float()).norm() / yb.float().norm()).item()
    if rel > 0.08:
        errs.append(f"tp_mlp fp8 vs bf16 baseline: relative error {rel:.3f}")
    try:
        comm.check()
    except Exception as e:  # noqa: BLE001
        errs.append(f"status: {e}")
    if _native.cuda().gemm_error_flag():
        errs.append("gemm error flag set")
    results[rank] = errs
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(gpu_count() < 2, reason="needs >= 2 GPUs")
def test_fused_gemm_collectives():
    world = min(gpu_count(), 8)
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, start_method="spawn", join=True)
    for r in range(world):
        assert results.get(r) == [], f"rank {r}: {results.get(r)}"
