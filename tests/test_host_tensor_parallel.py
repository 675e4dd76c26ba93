"""The tensor-parallel MLP training step (nexar_b200/parallel/tensor.py) on CPU
ranks: each rank's output shard and the gradients of its input shard and
weight slices equal those of the unsharded SwiGLU MLP (fp64 autograd)."""
import pytest
import torch

from helpers_host import bootstrap, run_collective
from nexar_b200.parallel.tensor import HostTP, tp_mlp


@pytest.mark.parametrize("W", [2, 4])
def test_tp_mlp_matches_unsharded_block(W):
    T, d, F = 16, 12, 8 * W
    Fl = F // W
    g = torch.Generator().manual_seed(W)
    x = torch.randn(T, d, generator=g, dtype=torch.float64)
    w_gu = torch.randn(2 * F, d, generator=g, dtype=torch.float64) * 0.3  # [gate; up]
    w_down = torch.randn(d, F, generator=g, dtype=torch.float64) * 0.3
    dy = torch.randn(T, d, generator=g, dtype=torch.float64)

    xr, wgr, wdr = (t.clone().requires_grad_(True) for t in (x, w_gu, w_down))
    gu = xr @ wgr.t()
    y = (torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]) @ wdr.t()
    y.backward(dy)

    def slices(r):
        rows = list(range(r * Fl, (r + 1) * Fl)) + list(range(F + r * Fl, F + (r + 1) * Fl))
        return rows, slice(r * Fl, (r + 1) * Fl), slice(r * T // W, (r + 1) * T // W)

    clients = bootstrap(W)
    try:
        def rank_fn(c):
            rows, cols, toks = slices(c.rank)
            xs = x[toks].clone().requires_grad_(True)
            wg = w_gu[rows].clone().requires_grad_(True)
            wd = w_down[:, cols].clone().requires_grad_(True)
            ys = tp_mlp(xs, wg, wd, HostTP(c))
            ys.backward(dy[toks])
            return ys.detach(), xs.grad, wg.grad, wd.grad

        out = run_collective(clients, rank_fn)
    finally:
        for c in clients:
            c.close()
    for r, (ys, gx, gwg, gwd) in enumerate(out):
        rows, cols, toks = slices(r)
        torch.testing.assert_close(ys, y.detach()[toks], rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(gx, xr.grad[toks], rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(gwg, wgr.grad[rows], rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(gwd, wdr.grad[:, cols], rtol=1e-10, atol=1e-10)
