"""The block schedule of the tcgen05 attention kernels (csrc/cuda/attention.cu),
replayed in PyTorch on the CPU: 128-row blocks, exp2-domain online softmax with
the output folded one block behind (O = alpha_{j-1} O + P_{j-1} V_{j-1}), P
rounded to bf16 before the P V product, the log-sum-exp that the forward saves,
and the backward per key block (S^T, dP^T, P^T = exp(S^T scale - lse),
dS^T = P^T (dP^T - Delta), dV += P^T dO, dK += dS^T Q, dQ += dS K). The
replay is checked against autograd of plain softmax attention in fp64, so
the bookkeeping the kernels implement is right independently of the GPU."""
import math

import pytest
import torch

BLK = 128
LOG2E = 1.0 / math.log(2.0)


def bf16(x):
    return x.to(torch.bfloat16).to(x.dtype)


def forward_schedule(q, k, v, causal):
    """q, k, v: [T, 64] of one (batch, head). Returns y [T, 64], lse [T]."""
    T = q.shape[0]
    scale_log2 = LOG2E / 8.0
    y = torch.empty_like(q)
    lse = torch.empty(T, dtype=q.dtype)
    for qb in range(T // BLK):
        rows = slice(qb * BLK, (qb + 1) * BLK)
        nkv = qb + 1 if causal else T // BLK
        m = torch.full((BLK,), -math.inf, dtype=q.dtype)
        l = torch.zeros(BLK, dtype=q.dtype)
        o = torch.zeros(BLK, 64, dtype=q.dtype)
        alpha_pend, pv_pend = None, None
        for j in range(nkv):
            cols = slice(j * BLK, (j + 1) * BLK)
            x = (q[rows] @ k[cols].T) * scale_log2
            if causal and j == qb:
                x = x.masked_fill(torch.ones(BLK, BLK, dtype=torch.bool).triu(1), -math.inf)
            m_new = torch.maximum(m, x.max(dim=1).values)
            alpha = torch.exp2(m - m_new)
            p = torch.exp2(x - m_new[:, None])
            l = l * alpha + p.sum(dim=1)
            m = m_new
            pv = bf16(p) @ v[cols]  # the tensor cores take P in bf16
            if pv_pend is not None:  # fold one block behind
                o = o * alpha_pend[:, None] + pv_pend
            alpha_pend, pv_pend = alpha, pv
        o = o * alpha_pend[:, None] + pv_pend
        y[rows] = o / l[:, None]
        lse[rows] = (m + torch.log2(l)) * math.log(2.0)
    return y, lse


def backward_schedule(q, k, v, y, dy, lse, causal):
    T = q.shape[0]
    scale = 1.0 / 8.0
    delta = (dy * y).sum(dim=1)
    dq = torch.zeros_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    for kb in range(T // BLK):
        krows = slice(kb * BLK, (kb + 1) * BLK)
        acc_dv = torch.zeros(BLK, 64, dtype=q.dtype)
        acc_dk = torch.zeros(BLK, 64, dtype=q.dtype)
        for i in range(kb if causal else 0, T // BLK):
            qcols = slice(i * BLK, (i + 1) * BLK)
            st = k[krows] @ q[qcols].T                    # [key, query]
            dpt = v[krows] @ dy[qcols].T
            pt = torch.exp2(st * scale * LOG2E - lse[qcols][None, :] * LOG2E)
            if causal and i == kb:
                pt = pt.masked_fill(torch.ones(BLK, BLK, dtype=torch.bool).tril(-1), 0.0)  # key r > query c
            dst = pt * (dpt - delta[qcols][None, :])
            acc_dv += bf16(pt) @ dy[qcols]
            acc_dk += bf16(dst) @ q[qcols]
            dq[qcols] += bf16(dst).T @ k[krows]
        dk[krows] = acc_dk * scale
        dv[krows] = acc_dv
    return dq * scale, dk, dv


@pytest.mark.parametrize("causal", [True, False])
def test_schedule_matches_softmax_attention(causal):
    torch.manual_seed(0)
    T = 384
    q, k, v = (torch.randn(T, 64, dtype=torch.float64) for _ in range(3))
    dy = torch.randn(T, 64, dtype=torch.float64)
    qr, kr, vr = (t.clone().requires_grad_(True) for t in (q, k, v))
    s = (qr @ kr.T) / 8.0
    if causal:
        s = s.masked_fill(torch.ones(T, T, dtype=torch.bool).triu(1), -math.inf)
    ref = torch.softmax(s, dim=1) @ vr
    ref.backward(dy)
    ref_lse = torch.logsumexp(s.detach(), dim=1)

    y, lse = forward_schedule(q, k, v, causal)
    torch.testing.assert_close(lse, ref_lse, rtol=1e-12, atol=1e-10)
    torch.testing.assert_close(y, ref.detach(), rtol=2e-2, atol=1e-2)  # bf16 P
    dq, dk, dv = backward_schedule(q, k, v, ref.detach(), dy, lse, causal)
    for got, want in ((dq, qr.grad), (dk, kr.grad), (dv, vr.grad)):
        torch.testing.assert_close(got, want, rtol=3e-2, atol=3e-2 * want.abs().max().item())
