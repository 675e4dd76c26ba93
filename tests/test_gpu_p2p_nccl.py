"""NcclGroup on the GPU: every call of the reference's NcclGroup
(nexar-nccl/src/group.rs) plus grouped send / recv, on one GPU (a
one-rank communicator: results equal the inputs, self send / recv is a copy),
and ring send / recv plus all-reduce over two GPUs when the box has them.
The expected values are plain PyTorch fp32 computations."""

import pytest
import torch

from conftest import gpu_count
from nexar_b200.core import DataType, ReduceOp
from nexar_b200.device import DeviceCommunicator
from nexar_b200.device import nccl

pytestmark = pytest.mark.gpu


def test_nccl_group_one_gpu(cuda0):
    g = nccl.NcclGroup(0, 1, nccl.unique_id(), device=0)
    assert (g.local_rank, g.local_world, g.device) == (0, 1, 0) and not g.closed
    gen = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(4097, device=cuda0, generator=gen)
    ref = x.clone()

    out = torch.empty_like(x)
    assert g.all_reduce(x, "sum", out=out) is out
    torch.testing.assert_close(out, ref, rtol=0, atol=0)
    g.all_reduce(x, "max")
    g.broadcast(x, root=0)
    g.reduce(x, root=0, op="sum")
    ag = torch.empty_like(x)
    g.all_gather(x, ag)
    rs = torch.empty_like(x)
    g.reduce_scatter(x, rs)
    torch.testing.assert_close(x, ref, rtol=0, atol=0)
    torch.testing.assert_close(ag, ref, rtol=0, atol=0)
    torch.testing.assert_close(rs, ref, rtol=0, atol=0)

    xb = x.to(torch.bfloat16)
    yb = torch.zeros_like(xb)
    g.send_recv(xb, 0, yb, 0)
    torch.testing.assert_close(yb.float(), ref.to(torch.bfloat16).float(), rtol=0, atol=0)

    y = torch.zeros_like(x)
    h = g.send_recv_nb(x, 0, y, 0)
    assert h.wait() is y
    h.synchronize()
    assert h.is_finished()
    torch.testing.assert_close(y, ref, rtol=0, atol=0)

    # raw-pointer calls on the group's stream, ordered by events
    z = ref.clone()
    torch.cuda.synchronize()
    g.allreduce_inplace(z.data_ptr(), z.numel(), DataType.F32, ReduceOp.Sum)
    ev = g.create_event()
    g.record_event(ev)
    g.stream_wait_event(ev, torch.cuda.current_stream())
    g.synchronize()
    assert g.event_query(ev)
    g.destroy_event(ev)
    torch.testing.assert_close(z, ref, rtol=0, atol=0)
    assert g.async_error() == 0

    comm = DeviceCommunicator(0, 1, 0, exchange=lambda h_: [h_], slot_bytes=1 << 20)
    comm.attach_nccl(g)
    assert comm.nccl is g
    g.destroy()
    assert g.closed
    with pytest.raises(nccl.NcclCommError, match="destroyed"):
        g.all_reduce(x)


# Two-GPU cases: one process per GPU (the deployment model), each joining the
# host mesh through a seed in this process. Two ranks as threads of one
# process are avoided: NCCL communicators of one clique inside one process
# share intra-process state, and tearing them down from two threads at once
# crashed the process on a B200 box.
def _spawn_ranks(target, world=2, timeout=180):
    import multiprocessing as mp

    from nexar_b200 import _host as H
    seed = H.SeedNode.bind("127.0.0.1:0", b"nccl-test")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank_main, args=(target, seed.local_addr(), q)) for _ in range(world)]
    try:
        for p_ in ps:
            p_.start()
        seed.with_formation_timeout(60.0).form_cluster(world)
        res = {}
        for _ in range(world):
            rank, out, err = q.get(timeout=timeout)
            if err:
                raise AssertionError(f"rank {rank}: {err}")
            res[rank] = _tensors(out)
    finally:
        for p_ in ps:
            p_.join(30)
            if p_.is_alive():
                p_.kill()
        seed.close()
    return [res[r] for r in range(world)]


def _plain(obj):
    """Tensors as numpy arrays (pickled by value: a shared-memory tensor would
    need this process alive when the parent unpickles it)."""
    if isinstance(obj, torch.Tensor):
        return obj.detach().cpu().numpy()
    if isinstance(obj, (list, tuple)):
        return type(obj)(_plain(o) for o in obj)
    return obj


def _tensors(obj):
    import numpy as np
    if isinstance(obj, np.ndarray):
        return torch.from_numpy(obj)
    if isinstance(obj, (list, tuple)):
        return type(obj)(_tensors(o) for o in obj)
    return obj


def _rank_main(target, seed_addr, q):
    import traceback

    from nexar_b200.client import NexarClient
    c = NexarClient.bootstrap(seed_addr, b"nccl-test")
    try:
        if torch.cuda.is_available():
            torch.cuda.set_device(c.rank)
        q.put((c.rank, _plain(target(c)), None))
    except BaseException:  # noqa: BLE001
        q.put((c.rank, None, traceback.format_exc()[-2000:]))
    finally:
        c.close()


def _ring_rank(c):
    g = nccl.nccl_group_for_client(c, device=c.rank)
    dev = torch.device("cuda", c.rank)
    n = 1 << 16
    xs = [torch.randn(n, generator=torch.Generator().manual_seed(10 + r)) for r in range(2)]
    x = xs[c.rank].to(dev)
    got = torch.empty_like(x)
    peer = 1 - c.rank
    g.send_recv(x, peer, got, peer)
    s = x.clone()
    g.all_reduce(s)
    torch.cuda.synchronize(dev)
    g.destroy()
    return got.cpu(), s.cpu(), xs[peer], xs[0] + xs[1]


def test_nccl_group_two_gpus_ring():
    if gpu_count() < 2:
        pytest.skip("needs two GPUs")
    for got, s, want_got, want_s in _spawn_ranks(_ring_rank):
        torch.testing.assert_close(got, want_got, rtol=0, atol=0)
        torch.testing.assert_close(s, want_s, rtol=1e-6, atol=1e-6)


_D, _ROWS, _M = 64, 16, 5


def _pipeline_setup():
    torch.manual_seed(0)
    stages = [torch.nn.Sequential(torch.nn.Linear(_D, _D), torch.nn.Tanh()) for _ in range(2)]
    g = torch.Generator().manual_seed(1)
    mbs = [torch.randn(_ROWS, _D, generator=g) for _ in range(_M)]
    tgts = [torch.randn(_ROWS, _D, generator=g) for _ in range(_M)]
    return stages, mbs, tgts


def _pipeline_rank(c):
    from nexar_b200.parallel.pipeline import NcclP2P, run_1f1b
    stages, mbs, tgts = _pipeline_setup()
    dev = torch.device("cuda", c.rank)
    grp = nccl.nccl_group_for_client(c, device=c.rank)
    mod = stages[c.rank].to(dev)
    inputs = [x.to(dev) for x in mbs] if c.rank == 0 else [None] * _M
    tg = [t.to(dev) for t in tgts]
    losses = run_1f1b(mod, NcclP2P(grp), inputs, (_ROWS, _D), torch.float32,
                      loss_fn=lambda y, i: ((y - tg[i]) ** 2).mean())
    torch.cuda.synchronize(dev)
    grads = [p.grad.cpu() for p in mod.parameters()]
    grp.destroy()
    return losses, grads


def test_pipeline_1f1b_two_gpus():
    """Two pipeline stages on two GPUs, activations and gradients over NCCL p2p,
    against the whole model on the CPU (fp32)."""
    if gpu_count() < 2:
        pytest.skip("needs two GPUs")
    ref, mbs, tgts = _pipeline_setup()
    whole = torch.nn.Sequential(*ref)
    ref_losses = []
    for x, t in zip(mbs, tgts):
        loss = ((whole(x) - t) ** 2).mean()
        loss.backward()
        ref_losses.append(float(loss.detach()))
    out = _spawn_ranks(_pipeline_rank)
    assert out[1][0] == pytest.approx(ref_losses, rel=1e-4, abs=1e-5)
    for s in range(2):
        for got, p in zip(out[s][1], ref[s].parameters()):
            torch.testing.assert_close(got, p.grad, rtol=1e-4, atol=1e-5)
