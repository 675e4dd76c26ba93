"""Data x tensor parallelism on a 2 x 2 grid of CPU ranks: split() builds the
TP groups (same data shard) and the DP groups (same weight slice); each TP
group runs the tensor-parallel MLP step on its data shard, and the weight
gradients are averaged over the DP group. Every rank's weight-slice gradient
equals the gradient of the unsharded MLP over the whole batch."""
import torch

from helpers_host import bootstrap, run_collective
from nexar_b200.parallel.tensor import HostTP, tp_mlp


def test_dp_x_tp_grid_matches_unsharded_mlp():
    DP, TP = 2, 2
    T, d, F = 8, 6, 4 * TP          # T tokens per data shard
    Fl = F // TP
    g = torch.Generator().manual_seed(0)
    x = torch.randn(DP * T, d, generator=g, dtype=torch.float64)
    dy = torch.randn(DP * T, d, generator=g, dtype=torch.float64)
    w_gu = torch.randn(2 * F, d, generator=g, dtype=torch.float64) * 0.3
    w_down = torch.randn(d, F, generator=g, dtype=torch.float64) * 0.3

    wgr, wdr = w_gu.clone().requires_grad_(True), w_down.clone().requires_grad_(True)
    gu = x @ wgr.t()
    y = (torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]) @ wdr.t()
    (y * dy).sum().div(DP).backward()   # DP averages the per-shard gradients

    clients = bootstrap(DP * TP)
    try:
        def rank_fn(c):
            dp_idx, tp_idx = divmod(c.rank, TP)
            tp_comm = c.split(dp_idx, tp_idx)       # ranks sharing a data shard
            dp_comm = c.split(TP + tp_idx, dp_idx)  # ranks sharing a weight slice
            rows = list(range(tp_idx * Fl, (tp_idx + 1) * Fl)) + list(range(F + tp_idx * Fl, F + (tp_idx + 1) * Fl))
            wg = w_gu[rows].clone().requires_grad_(True)
            wd = w_down[:, tp_idx * Fl:(tp_idx + 1) * Fl].clone().requires_grad_(True)
            tl = T // TP                              # sequence-parallel tokens of this TP rank
            t0 = dp_idx * T + tp_idx * tl
            xs = x[t0:t0 + tl]
            out = tp_mlp(xs, wg, wd, HostTP(tp_comm))
            out.backward(dy[t0:t0 + tl])
            for grad in (wg.grad, wd.grad):
                buf = grad.contiguous().view(-1).numpy()
                dp_comm.all_reduce_host(buf)
                grad.copy_(torch.from_numpy(buf).view_as(grad) / DP)
            return wg.grad, wd.grad, rows

        res = run_collective(clients, rank_fn)
    finally:
        for c in clients:
            c.close()
    for r, (gwg, gwd, rows) in enumerate(res):
        tp_idx = r % TP
        torch.testing.assert_close(gwg, wgr.grad[rows], rtol=1e-10, atol=1e-12)
        torch.testing.assert_close(gwd, wdr.grad[:, tp_idx * Fl:(tp_idx + 1) * Fl], rtol=1e-10, atol=1e-12)
