"""The CUDA staging adapter on the GPU (nexar-rdma/src/cuda_adapter.rs): with no
device communicator attached, ``*_device`` calls and raw-pointer collectives
on CUDA buffers go device -> host -> host collective -> device. Two ranks in
one process share cuda:0; expected values are PyTorch fp32 sums."""

import pytest
import torch

from helpers_host import run_collective
from nexar_b200.client import NexarClient
from nexar_b200.core import DataType, ReduceOp

pytestmark = pytest.mark.gpu

def test_cuda_adapter_stages_device_buffers(cuda0):
    cs = NexarClient.bootstrap_local(2, adapter="cuda")
    try:
        gens = [torch.Generator(device="cuda").manual_seed(20 + r) for r in range(2)]
        xs = [torch.randn(1000, device=cuda0, generator=gens[r]) for r in range(2)]
        ref = xs[0] + xs[1]
        run_collective(cs, lambda c: c.all_reduce_device(xs[c.rank]))
        for x in xs:
            torch.testing.assert_close(x, ref, rtol=1e-6, atol=1e-6)

        shards = [torch.full((8,), float(r + 1), device=cuda0) for r in range(2)]
        outs = [torch.zeros(16, device=cuda0) for _ in range(2)]
        run_collective(cs, lambda c: c.all_gather_device(shards[c.rank], outs[c.rank]))
        want = torch.cat([shards[0], shards[1]])
        for o in outs:
            torch.testing.assert_close(o, want, rtol=0, atol=0)

        b = [torch.arange(6, device=cuda0, dtype=torch.float32) * (r + 1) for r in range(2)]
        run_collective(cs, lambda c: c.broadcast_device(b[c.rank], 1))
        torch.testing.assert_close(b[0], torch.arange(6, device=cuda0, dtype=torch.float32) * 2, rtol=0, atol=0)

        # raw pointers (the reference's API) and p2p through the adapter
        y = [torch.full((5,), float(r + 1), device=cuda0, dtype=torch.bfloat16) for r in range(2)]
        run_collective(cs, lambda c: c.all_reduce(y[c.rank].data_ptr(), 5, DataType.BF16, ReduceOp.Max))
        torch.cuda.synchronize()
        assert all((t.float() == 2).all() for t in y)
        src = torch.arange(10, device=cuda0, dtype=torch.float32)
        dst = torch.zeros(10, device=cuda0)
        torch.cuda.synchronize()
        run_collective(cs, lambda c: c.send(src.data_ptr(), 40, 1, 3) if c.rank == 0
                       else c.recv(dst.data_ptr(), 40, 0, 3))
        torch.cuda.synchronize()
        torch.testing.assert_close(dst, src, rtol=0, atol=0)
    finally:
        for c in cs:
            c.close()
