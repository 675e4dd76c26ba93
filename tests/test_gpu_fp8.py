"""Block-scaled fp8 (e4m3, 1x128 activation / 128x128 weight scales) GEMM and quantisers
against plain torch fp32 references."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _dequant_1x128(q, s):
    R, K = q.shape
    f = q.float()
    kb = (K + 127) // 128
    pad = kb * 128 - K
    f = torch.nn.functional.pad(f, (0, pad)).view(R, kb, 128) * s.view(R, kb, 1)
    return f.view(R, kb * 128)[:, :K]


def _dequant_128x128(q, s):
    N, K = q.shape
    nb, kb = s.shape
    f = torch.nn.functional.pad(q.float(), (0, kb * 128 - K, 0, nb * 128 - N))
    f = f.view(nb, 128, kb, 128) * s.view(nb, 1, kb, 1)
    return f.reshape(nb * 128, kb * 128)[:N, :K]


def test_quantisers_match_torch(cuda0):
    from nexar_b200 import ops
    x = torch.randn(300, 520, device=cuda0).to(torch.bfloat16) * 3
    q, s = ops.quant_fp8_1x128(x)
    xf = x.float()
    for kb in range(s.shape[1]):
        blk = xf[:, kb * 128:(kb + 1) * 128]
        torch.testing.assert_close(s[:, kb], blk.abs().amax(1) / 448.0, rtol=1e-6, atol=0)
    ref_q = (xf / torch.repeat_interleave(s, 128, dim=1)[:, :520]).to(torch.float8_e4m3fn)
    assert torch.equal(q.view(torch.uint8), ref_q.view(torch.uint8))
    w = torch.randn(260, 384, device=cuda0).to(torch.bfloat16)
    qw, sw = ops.quant_fp8_128x128(w)
    assert sw.shape == (3, 3)
    torch.testing.assert_close(_dequant_128x128(qw, sw), w.float(), rtol=0.07, atol=1e-3)


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (256, 384, 512), (300, 200, 528), (2048, 1792, 4096)])
def test_gemm_fp8_blockscaled_matches_fp32(cuda0, M, N, K):
    """K must be a multiple of 16 (16-byte TMA rows); ragged M, N and K blocks are covered."""
    from nexar_b200 import _native, ops
    g = torch.Generator(device=cuda0).manual_seed(M + N + K)
    x = torch.randn(M, K, device=cuda0, generator=g).to(torch.bfloat16)
    w = (0.05 * torch.randn(N, K, device=cuda0, generator=g)).to(torch.bfloat16)
    xq, xs = ops.quant_fp8_1x128(x)
    wq, ws = ops.quant_fp8_128x128(w)
    out = ops.matmul_fp8(xq, xs, wq, ws)
    torch.cuda.synchronize()
    assert _native.cuda().gemm_error_flag() == 0
    ref = _dequant_1x128(xq, xs) @ _dequant_128x128(wq, ws).t()
    torch.testing.assert_close(out.float(), ref, atol=2e-2 * (K / 128) ** 0.5, rtol=1e-2)
    # and close to the bf16 product it approximates
    full = x.float() @ w.float().t()
    rel = ((out.float() - full).norm() / full.norm()).item()
    assert rel < 0.05, rel


def test_gemm_fp8_bias_gelu_epilogue(cuda0):
    from nexar_b200 import ops
    M, N, K = 256, 512, 384
    x = torch.randn(M, K, device=cuda0).to(torch.bfloat16)
    w = (0.05 * torch.randn(N, K, device=cuda0)).to(torch.bfloat16)
    b = torch.randn(N, device=cuda0).to(torch.bfloat16)
    xq, xs = ops.quant_fp8_1x128(x)
    wq, ws = ops.quant_fp8_128x128(w)
    ref_pre = _dequant_1x128(xq, xs) @ _dequant_128x128(wq, ws).t() + b.float()
    out = ops.matmul_fp8(xq, xs, wq, ws, bias=b)
    torch.testing.assert_close(out.float(), ref_pre, atol=3e-2, rtol=2e-2)
    out = ops.matmul_fp8(xq, xs, wq, ws, bias=b, act=1)
    torch.testing.assert_close(out.float(), torch.nn.functional.gelu(ref_pre, approximate="tanh"), atol=3e-2, rtol=2e-2)
