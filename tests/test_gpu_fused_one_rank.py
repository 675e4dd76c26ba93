"""Fused GEMM + collective kernels on one GPU with a one-rank communicator,
against fp32 references: the GEMM -> reduce-scatter epilogue (TMA stores
into the staging slot, per-tile flags, in-kernel reduction with the bias)
and all-gather -> GEMM, on consecutive calls (both staging slots) and shapes
whose width is not a multiple of the 256-column tile."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rand(shape, seed, dev, scale=1.0):
    g = torch.Generator(device=dev).manual_seed(seed)
    return (scale * torch.randn(*shape, device=dev, generator=g)).to(torch.bfloat16)


def _comm():
    from nexar_b200.device import DeviceCommunicator
    return DeviceCommunicator(0, 1, 0, exchange=lambda h: [h], slot_bytes=64 << 20, timeout_us=5_000_000)


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (256, 768, 512), (384, 640, 1024), (1024, 4096, 1792)])
def test_gemm_reduce_scatter_one_rank(cuda0, M, N, K):
    comm = _comm()
    for rep in range(3):
        A = _rand((M, K), 10 + rep, cuda0)
        B = _rand((N, K), 20 + rep, cuda0, 0.1)
        bias = _rand((N,), 30 + rep, cuda0)
        out = comm.gemm_reduce_scatter(A, B, bias=bias)
        torch.cuda.synchronize()
        comm.check()
        ref = A.float() @ B.float().t() + bias.float()
        torch.testing.assert_close(out.float(), ref, atol=0.05, rtol=2e-2)


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (256, 640, 512)])
def test_all_gather_gemm_one_rank(cuda0, M, N, K):
    comm = _comm()
    for rep in range(2):
        x = _rand((M, K), 40 + rep, cuda0)
        B = _rand((N, K), 50 + rep, cuda0, 0.1)
        out = comm.all_gather_gemm(x, B)
        torch.cuda.synchronize()
        comm.check()
        torch.testing.assert_close(out.float(), x.float() @ B.float().t(), atol=0.05, rtol=2e-2)
