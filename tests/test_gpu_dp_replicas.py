"""Data-parallel GPT-2 training on 2 GPUs keeps its replicas identical.

Each rank trains on different tokens; the bucketed gradient all-reduce
(launched from the backward hooks, overlapped with backward) must leave
every rank with the same averaged gradient, so after every step the bf16
parameters agree bit for bit across ranks. A bucket reduced before all of
its gradients were written would leave those parameters rank-local and the
replicas would drift apart. Also checks that every bucket launched after the
last of its parameters reported ready, in the order backward produced them.
"""
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import gpu_count

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _worker(rank, world, port, results, graph):
    import torch.distributed as dist
    from nexar_b200.device import DeviceCommunicator
    from nexar_b200.models.gpt2 import GPT2Config
    from nexar_b200.parallel.dp import DataParallelTrainer
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    errs = []
    try:
        comm = DeviceCommunicator.from_torch(timeout_us=5_000_000)
        cfg = GPT2Config(n_layer=4, n_head=4, n_embd=256, vocab_size=1000, padded_vocab=1024, block_size=256)
        tr = DataParallelTrainer(cfg, micro_batch=2, seq_len=256, comm=comm, use_cuda_graph=graph, seed=0,
                                 bucket_bytes=1 << 20)
        # Record, per step, which parameters had reported ready when each bucket launched.
        launched = []
        orig = tr._launch_bucket

        def spy(bi):
            launched.append((bi, set(tr._seen)))
            orig(bi)
        tr._launch_bucket = spy
        if graph:
            tr.capture()  # warm-up steps on the (identical, zero) static batch, then one captured step
        g = torch.Generator().manual_seed(100 + rank)
        for step in range(3):
            idx = torch.randint(0, cfg.vocab_size, (2, 256), generator=g)
            tgt = torch.randint(0, cfg.vocab_size, (2, 256), generator=g)
            tr.step(idx, tgt)
            torch.cuda.synchronize()
            p = tr.model.flat.param_bf16.view(torch.int32).cpu()  # bit patterns (gloo has no 16-bit ints)
            gathered = [torch.empty_like(p) for _ in range(world)]
            dist.all_gather(gathered, p)
            if not torch.equal(gathered[0], gathered[1]):
                diff = (gathered[0] != gathered[1]).nonzero().flatten() * 2  # bf16 index of each differing pair
                names = sorted({e.name for e in tr.model.flat.entries
                                for i in diff[:64].tolist() if e.offset <= i < e.offset + e.numel})
                errs.append(f"step {step}: {diff.numel()} parameters differ across ranks, e.g. in {names[:8]}")
                break
        for bi, seen in launched:
            start, end, names = tr.buckets[bi]
            missing = [n for n in names if n not in seen]
            if missing:
                errs.append(f"bucket {bi} launched before {missing[:4]} reported ready")
                break
        tr.release()
        comm.close()
    except Exception as e:  # noqa: BLE001
        errs.append(f"{type(e).__name__}: {e}")
    results[rank] = errs
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("graph", [False, True])
def test_dp_replicas_stay_identical(graph):
    if gpu_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_worker, args=(world, port, results, graph), nprocs=world, start_method="spawn", join=True)
    for r in range(world):
        assert results[r] == [], results[r]
