"""Device communicator lifecycle on one GPU: device-time histograms of the
collective calls, close(), and a client's reattach_device() after close.

A one-rank client: its device communicator reduces over one rank, so the
results equal the (scaled) inputs, computed here in fp32 with PyTorch."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_device_time_histogram_counts_every_call(cuda0):
    from nexar_b200.device import DeviceCommunicator
    comm = DeviceCommunicator(0, 1, 0, exchange=lambda h: [h], slot_bytes=1 << 20)
    comm.enable_timing()
    x = torch.randn(1 << 16, device=cuda0)
    for _ in range(5):
        comm.all_reduce(x, scale=0.5)
    out = torch.empty(1 << 16, device=cuda0)
    comm.all_gather(x, out)
    torch.cuda.synchronize()
    dt = comm.stats()["device_time"]
    assert dt["all_reduce"]["count"] == 5 and dt["all_gather"]["count"] == 1
    h = dt["all_reduce"]
    assert sum(h["buckets"]) == 5 and 0 < h["min_us"] <= h["mean_us"] <= h["max_us"]
    assert len(h["buckets"]) == len(h["bucket_edges_us"]) + 1
    comm.enable_timing(False)
    comm.all_reduce(x)
    assert "device_time" not in comm.stats()
    comm.close()


def test_close_then_reattach(cuda0):
    from nexar_b200.client import NexarClient
    (client,) = NexarClient.bootstrap_local(1)
    try:
        dev = client.attach_device(device=0)
        x = torch.randn(4099, device=cuda0)
        ref = x.clone()
        dev.all_reduce(x, scale=2.0)
        torch.cuda.synchronize()
        torch.testing.assert_close(x, 2.0 * ref, rtol=1e-6, atol=1e-6)
        new = client.reattach_device(dev)
        assert dev.closed and not new.closed
        y = torch.randn(1000, device=cuda0, dtype=torch.bfloat16)
        yr = y.float()
        new.all_reduce(y, scale=0.25)
        torch.cuda.synchronize()
        torch.testing.assert_close(y.float(), 0.25 * yr, rtol=1e-2, atol=1e-2)
        new.check()
        new.close()
        assert new.closed
    finally:
        client.close()
