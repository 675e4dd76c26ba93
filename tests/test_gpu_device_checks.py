"""Device argument checks of the collective kernels (NEXAR_DEVICE_CHECKS=1 or
``DeviceCommunicator.device_checks``), on one GPU with a one-rank communicator.

The failures are made on the host and are harmless even unchecked: a call
counter set back (the next barrier epoch does not increase) and a broadcast
root out of range, launched through a test hook that refuses to run unless
the checks are on, so the kernel's entry check always stands between the bad
root and any memory access. Each failure must show in the status word and
in check(), with the output untouched, and the communicator must work again
after clear_status()."""
import pytest
import torch

from nexar_b200.core import CollectiveFailed

pytestmark = pytest.mark.gpu


def _comm():
    from nexar_b200.device import DeviceCommunicator
    return DeviceCommunicator(0, 1, 0, exchange=lambda h: [h], slot_bytes=4 << 20)


def test_checked_collectives_run_clean(cuda0):
    comm = _comm()
    comm.device_checks = True
    x = torch.arange(1000, device=cuda0, dtype=torch.float32)
    out = torch.empty_like(x)
    comm.broadcast(x, root=0, out=out)
    g = comm.all_gather(x)
    comm.barrier()
    torch.cuda.synchronize()
    comm.check()
    assert comm.status()["code"] == 0
    torch.testing.assert_close(out, x)
    torch.testing.assert_close(g, x)


def test_stale_epoch_is_refused(cuda0):
    comm = _comm()
    comm.device_checks = True
    for _ in range(3):
        comm.barrier()
    torch.cuda.synchronize()
    comm.check()
    comm.native.debug_set_call_counter(0)  # the next barrier's epoch is below the stored ones
    comm.barrier()
    torch.cuda.synchronize()
    st = comm.status()
    assert st["code"] == 3 and st["block"] == 4  # kStatusCheckFailed, kCheckEpoch
    with pytest.raises(CollectiveFailed, match="epoch"):
        comm.check()
    comm.clear_status()
    comm.native.debug_set_call_counter(100)  # above every stored epoch again
    comm.barrier()
    torch.cuda.synchronize()
    comm.check()


def test_root_out_of_range_is_refused_before_any_access(cuda0):
    comm = _comm()
    x = torch.arange(4096, device=cuda0, dtype=torch.float32)
    out = torch.zeros_like(x)
    with pytest.raises(RuntimeError, match="checks"):
        comm.native.debug_broadcast_raw_root(x, out, 1)  # refused on the host: checks are off
    comm.device_checks = True
    comm.native.debug_broadcast_raw_root(x, out, 1)  # root 1 of a one-rank communicator
    torch.cuda.synchronize()
    st = comm.status()
    assert st["code"] == 3 and st["block"] == 2 and st["rank"] == 1 and st["epoch"] == 1
    assert int(out.abs().sum().item()) == 0  # the kernel returned before touching the output
    with pytest.raises(CollectiveFailed, match="root"):
        comm.check()
    comm.clear_status()
    comm.broadcast(x, root=0, out=out)
    torch.cuda.synchronize()
    comm.check()
    torch.testing.assert_close(out, x)
