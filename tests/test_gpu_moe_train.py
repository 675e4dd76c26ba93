"""Expert-parallel MoE training step on the fused kernels against the NCCL +
cuBLAS formulation of the same forward and backward, on >= 2 GPUs."""
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
    from nexar_b200.models.moe import ExpertParallelMoE, MoEConfig
    comm = DeviceCommunicator.from_torch(timeout_us=5_000_000, slot_bytes=16 << 20)
    cfg = MoEConfig.small()
    moe = ExpertParallelMoE(cfg, comm, seed=1)
    errs = []
    for rep in range(2):
        g = torch.Generator(device=dev).manual_seed(100 * rep + rank)
        x = torch.randn(cfg.tokens_per_gpu, cfg.d_model, device=dev, generator=g).to(torch.bfloat16)
        logits = torch.randn(cfg.tokens_per_gpu, world, device=dev, generator=g)
        dout = torch.randn(cfg.tokens_per_gpu, cfg.d_model, device=dev, generator=g).to(torch.bfloat16)
        got = moe.train_step(x, logits, dout)
        want = moe.train_step_baseline(x, logits, dout)
        torch.cuda.synchronize()
        for k in ("out", "dx", "dlogits", "dw_up", "dw_down"):
            scale = want[k].float().abs().max().item()
            try:
                torch.testing.assert_close(got[k].float(), want[k].float(), rtol=5e-2, atol=3e-2 * max(scale, 1e-3))
            except AssertionError as e:
                errs.append(f"rep {rep} {k}: {str(e)[:300]}")
    try:
        comm.check()
    except Exception as e:  # noqa: BLE001
        errs.append(str(e))
    results[rank] = errs
    dist.barrier()
    dist.destroy_process_group()


def test_moe_train_step_matches_baseline():
    if gpu_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    results = mp.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, start_method="spawn", join=True)
    for r in range(world):
        assert results[r] == [], results[r]
