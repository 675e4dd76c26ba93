"""tcgen05 GEMM against a torch fp32 reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 128), (1000, 768, 768), (333, 2304, 768),
                                   (4096, 3072, 768), (96, 200, 136), (8192, 1792, 4096)])
def test_gemm_matches_fp32(cuda0, M, N, K):
    from nexar_b200 import _native
    C = _native.cuda()
    g = torch.Generator(device=cuda0).manual_seed(M + N + K)
    A = torch.randn(M, K, device=cuda0, generator=g).to(torch.bfloat16)
    B = torch.randn(N, K, device=cuda0, generator=g).to(torch.bfloat16)
    out = torch.empty(M, N, device=cuda0, dtype=torch.bfloat16)
    C.gemm(A, B, out)
    torch.cuda.synchronize()
    assert C.gemm_error_flag() == 0
    ref = A.float() @ B.float().t()
    torch.testing.assert_close(out.float(), ref, atol=0.05 * (K ** 0.5) / 8, rtol=2e-2)


def test_gemm_epilogue_bias_gelu_residual(cuda0):
    from nexar_b200 import _native
    C = _native.cuda()
    M, N, K = 512, 768, 256
    A = torch.randn(M, K, device=cuda0).to(torch.bfloat16)
    B = (0.05 * torch.randn(N, K, device=cuda0)).to(torch.bfloat16)
    bias = torch.randn(N, device=cuda0).to(torch.bfloat16)
    res = torch.randn(M, N, device=cuda0).to(torch.bfloat16)
    out = torch.empty(M, N, device=cuda0, dtype=torch.bfloat16)
    pre = torch.empty_like(out)
    C.gemm(A, B, out, bias=bias, pre=pre, act=1)
    ref_pre = A.float() @ B.float().t() + bias.float()
    torch.testing.assert_close(pre.float(), ref_pre, atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(out.float(), torch.nn.functional.gelu(ref_pre, approximate="tanh"), atol=3e-2, rtol=2e-2)
    C.gemm(A, B, out, residual=res, alpha=0.5)
    torch.testing.assert_close(out.float(), 0.5 * (A.float() @ B.float().t()) + res.float(), atol=3e-2, rtol=2e-2)


def test_gemm_strided_operands(cuda0):
    from nexar_b200 import _native
    C = _native.cuda()
    big = torch.randn(300, 1024, device=cuda0).to(torch.bfloat16)
    A = big[:, 128:640]          # leading dim 1024, K = 512
    B = torch.randn(384, 512, device=cuda0).to(torch.bfloat16)
    out_big = torch.zeros(300, 1024, device=cuda0, dtype=torch.bfloat16)
    out = out_big[:, :384]
    C.gemm(A, B, out)
    torch.testing.assert_close(out.float(), A.float() @ B.float().t(), atol=0.1, rtol=2e-2)
    assert torch.all(out_big[:, 384:] == 0)
