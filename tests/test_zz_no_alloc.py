"""The allocation-free LayerNorm backward, called through its exported C symbol.

`nexar_ln_bwd_noalloc` serves callers that may not allocate device memory
where they run (inside a memory pool owned by another runtime, or on a path
where cudaMalloc's implicit device synchronisation is unacceptable); its
scratch is a fixed static device array. This test calls it with ctypes, the
way such a caller would, and checks it against the regular entry point
(`_cuda.ln_bwd`, which takes a caller-allocated scratch buffer) and against a
plain PyTorch fp32 LayerNorm backward, on two calls in a row, so the second
call also shows that the contents the shared array keeps from the first call
do not leak into its result. This file is collected last on purpose.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from nexar_b200 import _native
    lib = ctypes.CDLL(_native.cuda().__file__)
    fn = lib.nexar_ln_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 9 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return fn


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


@pytest.mark.parametrize("R,C,with_dres", [(4096, 768, True), (333, 1024, False)])
def test_noalloc_matches_regular_entry_point(cuda0, R, C, with_dres):
    from nexar_b200 import _native
    Cx = _native.cuda()
    fn = _lib()
    g = torch.Generator(device=cuda0).manual_seed(7)
    bf = torch.bfloat16
    x = torch.randn(R, C, device=cuda0, generator=g).to(bf)
    w = (1 + 0.1 * torch.randn(C, device=cuda0, generator=g)).to(bf)
    b = (0.1 * torch.randn(C, device=cuda0, generator=g)).to(bf)
    y = torch.empty_like(x)
    mean = torch.empty(R, device=cuda0)
    rstd = torch.empty(R, device=cuda0)
    Cx.ln_fwd(x, None, None, w, b, y, mean, rstd, 1e-5)
    dy = torch.randn(R, C, device=cuda0, generator=g).to(bf)
    dres = torch.randn(R, C, device=cuda0, generator=g).to(bf) if with_dres else None

    # regular entry point: caller-provided scratch
    dx_ref, dw_ref, db_ref = torch.empty_like(x), torch.empty_like(w), torch.empty_like(w)
    scratch = torch.empty(Cx.ln_bwd_scratch_floats(R, C), device=cuda0)
    counter = torch.zeros(1, dtype=torch.int32, device=cuda0)
    Cx.ln_bwd(dy, x, mean, rstd, w, dres, dx_ref, dw_ref, db_ref, scratch, counter)

    # plain PyTorch fp32 reference of the same op
    xf = x.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    bf32 = b.float().requires_grad_(True)
    torch.nn.functional.layer_norm(xf, (C,), wf, bf32, 1e-5).backward(dy.float())
    dx32 = xf.grad + (dres.float() if dres is not None else 0)
    dw32, db32 = wf.grad, bf32.grad

    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        dx, dw, db = torch.full_like(x, 7.0), torch.full_like(w, 7.0), torch.full_like(w, 7.0)
        rc = fn(_ptr(dy), _ptr(x), _ptr(mean), _ptr(rstd), _ptr(w), _ptr(dres), _ptr(dx), _ptr(dw), _ptr(db),
                R, C, ctypes.c_void_p(stream))
        assert rc == 0
        torch.cuda.synchronize()
        torch.testing.assert_close(dx.float(), dx_ref.float(), atol=1e-2, rtol=1e-2)
        torch.testing.assert_close(dw.float(), dw_ref.float(), atol=0.25, rtol=3e-2)
        torch.testing.assert_close(db.float(), db_ref.float(), atol=0.25, rtol=3e-2)
        torch.testing.assert_close(dx.float(), dx32, atol=3e-2, rtol=2e-2)
        torch.testing.assert_close(dw.float(), dw32, atol=2e-2 * dw32.abs().max().item(), rtol=2e-2)
        torch.testing.assert_close(db.float(), db32, atol=2e-2 * db32.abs().max().item(), rtol=2e-2)


def test_noalloc_rejects_oversized_rows(cuda0):
    fn = _lib()
    t = torch.empty(8, 4096, dtype=torch.bfloat16, device=cuda0)
    s = torch.empty(8, device=cuda0)
    w = torch.empty(4096, dtype=torch.bfloat16, device=cuda0)
    rc = fn(_ptr(t), _ptr(t), _ptr(s), _ptr(s), _ptr(w), ctypes.c_void_p(0), _ptr(t), _ptr(w), _ptr(w),
            8, 4096, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 1  # NEXAR_LN_NOALLOC_TOO_LARGE: nothing launched
