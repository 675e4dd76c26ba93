"""Expert-parallel MoE: fused dispatch/combine path vs the NCCL + torch formulation."""
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
    errs = []
    cfg = MoEConfig.small()
    moe = ExpertParallelMoE(cfg, comm, seed=1)
    for rep in range(3):
        g = torch.Generator(device=dev).manual_seed(100 * rep + rank)
        x = torch.randn(cfg.tokens_per_gpu, cfg.d_model, device=dev, generator=g).to(torch.bfloat16)
        logits = torch.randn(cfg.tokens_per_gpu, world, device=dev, generator=g)
        y = moe.forward(x, logits)
        yb = moe.forward_baseline(x, logits)
        torch.cuda.synchronize()
        try:
            torch.testing.assert_close(y.float(), yb.float(), atol=2e-2, rtol=5e-2)
        except AssertionError as e:
            errs.append(f"rep {rep}: {str(e)[:400]}")
    # routing alone: gates sum to 1, two distinct experts per token
    assert torch.allclose(moe.slot_gate.view(-1, 2).sum(1), torch.ones(cfg.tokens_per_gpu, device=dev))
    assert (moe.slot_expert.view(-1, 2)[:, 0] != moe.slot_expert.view(-1, 2)[:, 1]).all()
    try:
        comm.check()
    except Exception as e:  # noqa: BLE001
        errs.append(str(e))
    results[rank] = errs
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(gpu_count() < 2, reason="needs >= 2 GPUs")
def test_moe_fused_matches_baseline():
    world = min(gpu_count(), 8)
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, start_method="spawn", join=True)
    for r in range(world):
        assert results.get(r) == [], f"rank {r}: {results.get(r)}"
