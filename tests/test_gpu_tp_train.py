"""TP Llama-MLP training step (forward + backward on the fused kernels)
against the NCCL + cuBLAS formulation of the same step, on >= 2 GPUs."""
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


def _worker(rank, world, port, results):
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    from nexar_b200.device import DeviceCommunicator
    from nexar_b200.models.llama_mlp import LlamaMLPConfig, TPLlamaMLP
    comm = DeviceCommunicator.from_torch(timeout_us=5_000_000, slot_bytes=64 << 20)
    cfg = LlamaMLPConfig(d_model=512, ffn=1024 * world, tokens=256 * world)
    mlp = TPLlamaMLP(cfg, comm, seed=3)
    g = torch.Generator(device=dev).manual_seed(900 + rank)
    x = torch.randn(cfg.tokens // world, cfg.d_model, device=dev, generator=g).to(torch.bfloat16)
    dy = torch.randn(cfg.tokens // world, cfg.d_model, device=dev, generator=g).to(torch.bfloat16)
    errs = []
    for rep in range(2):
        got = mlp.train_step(x, dy)
        want = mlp.train_step_baseline(x, dy)
        torch.cuda.synchronize()
        for name, a, b in zip(("y", "dx", "dw_gu", "dw_down"), got, want):
            scale = b.float().abs().max().item()
            try:
                torch.testing.assert_close(a.float(), b.float(), rtol=5e-2, atol=3e-2 * max(scale, 1e-3))
            except AssertionError as e:
                errs.append(f"rep{rep} {name}: {str(e)[:300]}")
    comm.check()
    results[rank] = errs
    dist.barrier()
    dist.destroy_process_group()


def test_tp_train_step_matches_nccl_cublas():
    if gpu_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    results = mp.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, start_method="spawn", join=True)
    for r in range(world):
        assert results[r] == [], results[r]
