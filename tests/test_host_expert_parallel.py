"""Expert-parallel MoE training step (nexar_b200/parallel/expert.py) on CPU
ranks: outputs and the gradients of the tokens, router logits and each rank's
expert equal those of a dense top-2 MoE evaluated with fp64 autograd."""
import pytest
import torch

from helpers_host import bootstrap, run_collective
from nexar_b200.parallel.expert import HostEP, moe_train_step


def _dense(x, logits, w_up, w_down):
    """out[t] = sum_k g_k(t) * expert_{e_k(t)}(x[t]); gates = softmax of the top-2 logits."""
    top = torch.topk(logits.detach(), 2, dim=1).indices
    g = torch.softmax(torch.gather(logits, 1, top), dim=1)
    out = torch.zeros_like(x)
    F = w_down.shape[2]
    for e in range(w_up.shape[0]):
        gu = x @ w_up[e].t()
        y = (torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]) @ w_down[e].t()
        weight = (g * (top == e)).sum(1, keepdim=True)
        out = out + weight * y
    return out


@pytest.mark.parametrize("W", [2, 3])
def test_moe_train_step_matches_dense_moe(W):
    T, d, F = 6, 8, 5
    gen = torch.Generator().manual_seed(W)
    xs = torch.randn(W, T, d, generator=gen, dtype=torch.float64)
    ls = torch.randn(W, T, W, generator=gen, dtype=torch.float64)
    dys = torch.randn(W, T, d, generator=gen, dtype=torch.float64)
    w_up = torch.randn(W, 2 * F, d, generator=gen, dtype=torch.float64) * 0.4
    w_down = torch.randn(W, d, F, generator=gen, dtype=torch.float64) * 0.4

    xr, lr_, wur, wdr = (t.clone().requires_grad_(True) for t in (xs, ls, w_up, w_down))
    outs = [_dense(xr[q], lr_[q], wur, wdr) for q in range(W)]
    torch.autograd.backward(outs, [dys[q] for q in range(W)])

    clients = bootstrap(W)
    try:
        def rank_fn(c):
            r = c.rank
            ep = HostEP(c, capacity=2 * T * W, d=d)
            return moe_train_step(xs[r], ls[r], dys[r], w_up[r], w_down[r], ep)

        res = run_collective(clients, rank_fn)
    finally:
        for c in clients:
            c.close()
    for r in range(W):
        torch.testing.assert_close(res[r]["out"], outs[r].detach(), rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(res[r]["dx"], xr.grad[r], rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(res[r]["dlogits"].double(), lr_.grad[r], rtol=1e-6, atol=1e-8)
        torch.testing.assert_close(res[r]["dw_up"], wur.grad[r], rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(res[r]["dw_down"], wdr.grad[r], rtol=1e-10, atol=1e-10)
