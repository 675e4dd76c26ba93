"""Autograd wrappers around the sm_100a model kernels.

Each function calls exactly one (or two) native kernels per direction; the
shapes are flattened to [rows, features] internally.
"""
from __future__ import annotations

import torch

from .. import _native

_SCRATCH = {}


def _scratch(device, nfloats: int) -> torch.Tensor:
    """Per-device reusable fp32 scratch plus a zeroed uint32 ticket counter."""
    key = (device, "f")
    buf = _SCRATCH.get(key)
    if buf is None or buf.numel() < nfloats:
        buf = torch.empty(max(nfloats, 1 << 16), dtype=torch.float32, device=device)
        _SCRATCH[key] = buf
    return buf


def _counter(device, slot: int = 0) -> torch.Tensor:
    key = (device, "c")
    c = _SCRATCH.get(key)
    if c is None:
        c = torch.zeros(64, dtype=torch.int32, device=device)
        _SCRATCH[key] = c
    return c[slot:slot + 1]


class _LayerNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, eps):
        C = x.shape[-1]
        x2 = x.reshape(-1, C)
        R = x2.shape[0]
        y = torch.empty_like(x2)
        mean = torch.empty(R, dtype=torch.float32, device=x.device)
        rstd = torch.empty(R, dtype=torch.float32, device=x.device)
        _native.cuda().ln_fwd(x2, None, None, w, b, y, mean, rstd, eps)
        ctx.save_for_backward(x2, w, mean, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, mean, rstd = ctx.saved_tensors
        C = x2.shape[-1]
        dy2 = dy.contiguous().view(-1, C)
        dx = torch.empty_like(x2)
        dw = torch.empty_like(w)
        db = torch.empty_like(w)
        C_ = _native.cuda()
        scratch = _scratch(x2.device, C_.ln_bwd_scratch_floats(x2.shape[0], C))
        C_.ln_bwd(dy2, x2, mean, rstd, w, None, dx, dw, db, scratch, _counter(x2.device))
        return dx.view(ctx.shape), dw, db, None


def layer_norm(x, w, b, eps: float = 1e-5):
    return _LayerNorm.apply(x, w, b, eps)


class _ResidualLayerNorm(torch.autograd.Function):
    """s = x + r ; y = LayerNorm(s). Returns (s, y)."""

    @staticmethod
    def forward(ctx, x, r, w, b, eps):
        C = x.shape[-1]
        x2 = x.reshape(-1, C)
        r2 = r.reshape(-1, C)
        R = x2.shape[0]
        s = torch.empty_like(x2)
        y = torch.empty_like(x2)
        mean = torch.empty(R, dtype=torch.float32, device=x.device)
        rstd = torch.empty(R, dtype=torch.float32, device=x.device)
        _native.cuda().ln_fwd(x2, r2, s, w, b, y, mean, rstd, eps)
        ctx.save_for_backward(s, w, mean, rstd)
        ctx.shape = x.shape
        return s.view(x.shape), y.view(x.shape)

    @staticmethod
    def backward(ctx, ds, dy):
        s, w, mean, rstd = ctx.saved_tensors
        C = s.shape[-1]
        dx = torch.empty_like(s)
        dw = torch.empty_like(w)
        db = torch.empty_like(w)
        C_ = _native.cuda()
        scratch = _scratch(s.device, C_.ln_bwd_scratch_floats(s.shape[0], C))
        dres = None if ds is None else ds.contiguous().view(-1, C)
        if dy is None:
            dy = torch.zeros_like(s)
        C_.ln_bwd(dy.contiguous().view(-1, C), s, mean, rstd, w, dres, dx, dw, db, scratch, _counter(s.device))
        dx = dx.view(ctx.shape)
        return dx, dx, dw, db, None


def residual_layer_norm(x, r, w, b, eps: float = 1e-5):
    return _ResidualLayerNorm.apply(x, r, w, b, eps)


class _Gelu(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        x = x.contiguous()
        y = torch.empty_like(x)
        _native.cuda().gelu_fwd(x, y)
        ctx.save_for_backward(x)
        return y

    @staticmethod
    def backward(ctx, dy):
        (x,) = ctx.saved_tensors
        dx = torch.empty_like(x)
        _native.cuda().gelu_bwd(x, dy.contiguous(), dx)
        return dx


def gelu(x):
    return _Gelu.apply(x)


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        gu = gu.contiguous()
        F = gu.shape[-1] // 2
        y = torch.empty(*gu.shape[:-1], F, dtype=gu.dtype, device=gu.device)
        _native.cuda().swiglu_fwd(gu, y)
        ctx.save_for_backward(gu)
        return y

    @staticmethod
    def backward(ctx, dy):
        (gu,) = ctx.saved_tensors
        dgu = torch.empty_like(gu)
        _native.cuda().swiglu_bwd(gu, dy.contiguous(), dgu)
        return dgu


def swiglu(gu):
    """silu(gate) * up for gu = [..., 2F] laid out as [gate | up]."""
    return _SwiGLU.apply(gu)


class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tok, wte, wpe):
        B, T = tok.shape
        C = wte.shape[1]
        out = torch.empty(B, T, C, dtype=wte.dtype, device=wte.device)
        _native.cuda().embed_fwd(tok, wte, wpe, out, T)
        ctx.save_for_backward(tok)
        ctx.shapes = (wte.shape, wpe.shape)
        return out

    @staticmethod
    def backward(ctx, dout):
        (tok,) = ctx.saved_tensors
        B, T = tok.shape
        wte_shape, wpe_shape = ctx.shapes
        dwte = torch.zeros(wte_shape, dtype=dout.dtype, device=dout.device)
        dwpe = torch.zeros(wpe_shape, dtype=dout.dtype, device=dout.device)
        _native.cuda().embed_bwd(tok, dout.contiguous(), dwte, dwpe, B, T)
        return None, dwte, dwpe


def embedding(tok, wte, wpe):
    return _Embedding.apply(tok, wte, wpe)


class _CrossEntropy(torch.autograd.Function):
    """Mean token cross-entropy over padded-vocab logits.

    The gradient is computed in the forward pass, written over the logits
    buffer (the logits are not needed afterwards), and scaled by the incoming
    grad in backward.
    """

    @staticmethod
    def forward(ctx, logits, targets, V, unit_grad):
        ctx.unit_grad = unit_grad
        Vp = logits.shape[-1]
        l2 = logits.view(-1, Vp)
        R = l2.shape[0]
        losses = torch.empty(R, dtype=torch.float32, device=logits.device)
        _native.cuda().xent(l2, targets.reshape(-1), losses, l2, V, 1.0 / R)
        ctx.save_for_backward(l2)
        ctx.shape = logits.shape
        return losses.mean()

    @staticmethod
    def backward(ctx, g):
        (dl,) = ctx.saved_tensors
        if ctx.unit_grad:
            # The caller guarantees d(loss) == 1 (loss.backward() on this
            # loss), which saves a full pass over the logits.
            return dl.view(ctx.shape), None, None, None
        return (dl * g.to(dl.dtype)).view(ctx.shape), None, None, None


def cross_entropy(logits, targets, vocab_size: int, unit_grad: bool = False):
    """Mean cross-entropy; ``unit_grad=True`` skips scaling by d(loss) (must be 1)."""
    return _CrossEntropy.apply(logits, targets, vocab_size, unit_grad)


def cross_entropy_loss_only(logits, targets, vocab_size: int):
    Vp = logits.shape[-1]
    l2 = logits.reshape(-1, Vp).contiguous()
    losses = torch.empty(l2.shape[0], dtype=torch.float32, device=logits.device)
    _native.cuda().xent(l2, targets.reshape(-1).contiguous(), losses, None, vocab_size, 1.0)
    return losses
