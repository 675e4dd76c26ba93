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


@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K,splits", [(256, 512, 128, 1), (328, 200, 520, 1), (768, 768, 8192, 0),
                                          (136, 264, 1000, 3), (2304, 768, 4096, 2)])
def test_gemm_operand_majors_and_split_k(cuda0, a_t, b_t, M, N, K, splits):
    """opA / opB given transposed (MN-major smem operands) and split-K, vs fp32.

    A transposed operand's row length (M or N) must be a multiple of 8 (16-byte
    TMA rows); tile-ragged sizes are covered."""
    from nexar_b200 import _native, ops
    C = _native.cuda()
    g = torch.Generator(device=cuda0).manual_seed(M * 7 + N * 3 + K + 2 * a_t + b_t)
    A = torch.randn(M, K, device=cuda0, generator=g).to(torch.bfloat16)
    B = torch.randn(N, K, device=cuda0, generator=g).to(torch.bfloat16)
    bias = torch.randn(N, device=cuda0, generator=g).to(torch.bfloat16)
    a_arg = A.t().contiguous() if a_t else A
    b_arg = B.t().contiguous() if b_t else B
    out = ops.matmul_nt(a_arg, b_arg, bias=bias, a_t=a_t, b_t=b_t, splits=splits)
    torch.cuda.synchronize()
    assert C.gemm_error_flag() == 0
    ref = A.float() @ B.float().t() + bias.float()
    torch.testing.assert_close(out.float(), ref, atol=0.05 * (K ** 0.5) / 8, rtol=2e-2)


def test_gemm_accumulate_and_split_gelu(cuda0):
    from nexar_b200 import ops
    M, N, K = 384, 512, 2048
    A = torch.randn(M, K, device=cuda0).to(torch.bfloat16)
    B = (0.03 * torch.randn(N, K, device=cuda0)).to(torch.bfloat16)
    base = torch.randn(M, N, device=cuda0).to(torch.bfloat16)
    for sp in (1, 4):
        out = base.clone()
        ops.matmul_nt(A, B, out=out, accumulate=True, splits=sp)
        torch.testing.assert_close(out.float(), base.float() + A.float() @ B.float().t(), atol=0.1, rtol=2e-2)
        pre = torch.empty_like(out)
        ops.matmul_nt(A, B, out=out, act=1, pre=pre, splits=sp)
        ref_pre = A.float() @ B.float().t()
        torch.testing.assert_close(pre.float(), ref_pre, atol=0.05, rtol=2e-2)
        torch.testing.assert_close(out.float(), torch.nn.functional.gelu(ref_pre, approximate="tanh"),
                                   atol=0.05, rtol=2e-2)


def test_linear_op_grads_match_fp32(cuda0):
    """ops.linear backward (MN-major GEMMs, split-K wgrad, colsum bias grad) vs torch autograd."""
    from nexar_b200 import ops
    g = torch.Generator(device=cuda0).manual_seed(11)
    M, Kin, Nout = 1024, 768, 2304
    x = torch.randn(M, Kin, device=cuda0, generator=g).to(torch.bfloat16).requires_grad_(True)
    w = (0.02 * torch.randn(Nout, Kin, device=cuda0, generator=g)).to(torch.bfloat16).requires_grad_(True)
    b = (0.1 * torch.randn(Nout, device=cuda0, generator=g)).to(torch.bfloat16).requires_grad_(True)
    dy = torch.randn(M, Nout, device=cuda0, generator=g).to(torch.bfloat16)
    for act in (None, "gelu"):
        for t in (x, w, b):
            t.grad = None
        y = ops.linear(x, w, b, act=act)
        y.backward(dy)
        xf, wf, bf = (t.detach().float().requires_grad_(True) for t in (x, w, b))
        yf = xf @ wf.t() + bf
        if act:
            yf = torch.nn.functional.gelu(yf, approximate="tanh")
        yf.backward(dy.float())
        torch.testing.assert_close(y.float(), yf.detach(), atol=3e-2, rtol=2e-2)
        for ours, ref in ((x.grad, xf.grad), (w.grad, wf.grad), (b.grad, bf.grad)):
            err = (ours.float() - ref).norm() / ref.norm()
            assert err < 1e-2, (act, err.item())


def test_gemm_rejects_unaligned_transposed_operand(cuda0):
    from nexar_b200 import ops
    A = torch.randn(520, 333, device=cuda0).to(torch.bfloat16)  # [K, M] with M*2 bytes not a multiple of 16
    B = torch.randn(200, 520, device=cuda0).to(torch.bfloat16)
    with pytest.raises(RuntimeError, match="invalid argument"):
        ops.matmul_nt(A, B, a_t=True, splits=1)


@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, True)])
@pytest.mark.parametrize("M,N,K,splits", [(256, 256, 64, 1), (8192, 768, 768, 1), (520, 392, 1000, 1),
                                          (768, 768, 8192, 6), (2304, 768, 4096, 2), (8192, 3072, 256, 1),
                                          (4096, 2304, 768, 1)])
def test_gemm_2sm_pair_kernel_matches_fp32(cuda0, a_t, b_t, M, N, K, splits):
    """The CTA-pair (cta_group::2, 256x256 tile) kernel: operand majors, ragged tiles, split-K."""
    from nexar_b200 import _native, ops
    C = _native.cuda()
    g = torch.Generator(device=cuda0).manual_seed(M + 3 * N + 7 * K + a_t + 2 * b_t)
    A = torch.randn(M, K, device=cuda0, generator=g).to(torch.bfloat16)
    B = torch.randn(N, K, device=cuda0, generator=g).to(torch.bfloat16)
    bias = torch.randn(N, device=cuda0, generator=g).to(torch.bfloat16)
    a_arg = A.t().contiguous() if a_t else A
    b_arg = B.t().contiguous() if b_t else B
    prev = C.gemm_get_2sm()
    C.gemm_set_2sm(1)
    try:
        out = ops.matmul_nt(a_arg, b_arg, bias=bias, a_t=a_t, b_t=b_t, splits=splits)
        C.gemm_set_2sm(0)
        out1 = ops.matmul_nt(a_arg, b_arg, bias=bias, a_t=a_t, b_t=b_t, splits=splits)
        torch.cuda.synchronize()
    finally:
        C.gemm_set_2sm(prev)
    torch.testing.assert_close(out.float(), out1.float(), atol=0.05 * (K ** 0.5) / 8, rtol=2e-2)
    assert C.gemm_error_flag() == 0
    ref = A.float() @ B.float().t() + bias.float()
    torch.testing.assert_close(out.float(), ref, atol=0.05 * (K ** 0.5) / 8, rtol=2e-2)
