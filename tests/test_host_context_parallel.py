"""Ring attention (context parallelism) on CPU ranks: every rank's output and
the gradients of its q, k, v shards equal plain attention over the whole
sequence (fp64)."""
import pytest
import torch

from helpers_host import bootstrap, run_collective
from nexar_b200.parallel.context import RingHost, ring_attention


@pytest.mark.parametrize("W,causal", [(2, True), (4, True), (3, False)])
def test_ring_attention_matches_full(W, causal):
    N, S, D = 3, 4, 8
    T = W * S
    g = torch.Generator().manual_seed(W)
    q, k, v, dy = (torch.randn(N, T, D, generator=g, dtype=torch.float64) for _ in range(4))
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    s = torch.einsum("nqd,nkd->nqk", qr, kr) / D ** 0.5
    if causal:
        s = s.masked_fill(torch.ones(T, T, dtype=torch.bool).triu(1), float("-inf"))
    ref = torch.einsum("nqk,nkd->nqd", torch.softmax(s, -1), vr)
    ref.backward(dy)

    clients = bootstrap(W)
    try:
        def rank_fn(c):
            sl = slice(c.rank * S, (c.rank + 1) * S)
            qs, ks, vs = (t[:, sl].clone().requires_grad_(True) for t in (q, k, v))
            y = ring_attention(qs, ks, vs, RingHost(c), causal=causal)
            y.backward(dy[:, sl])
            return y.detach(), qs.grad, ks.grad, vs.grad

        res = run_collective(clients, rank_fn)
    finally:
        for c in clients:
            c.close()
    for r, (y, gq, gk, gv) in enumerate(res):
        sl = slice(r * S, (r + 1) * S)
        torch.testing.assert_close(y, ref.detach()[:, sl], rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(gq, qr.grad[:, sl], rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(gk, kr.grad[:, sl], rtol=1e-10, atol=1e-10)
        torch.testing.assert_close(gv, vr.grad[:, sl], rtol=1e-10, atol=1e-10)
