"""Autograd wrappers around the sm_100a model kernels.

Each function calls exactly one (or two) native kernels per direction; the
shapes are flattened to [rows, features] internally.

Gradient sinks: a parameter that carries ``main_grad`` (a view into a flat
gradient buffer, see ``nexar_b200.utils.flat``) gets its gradient written
there directly by the backward kernels — the weight-gradient GEMM stores
into it, LayerNorm / bias reductions write their column sums into it — and
autograd sees ``None`` for that input, so there is no zero-fill of the
gradient buffer and no accumulate kernel per parameter. After the write the
parameter's ``_nexar_on_ready`` callback (if any) runs; the data-parallel
trainer uses it to launch bucket all-reduces during backward. Parameters
without ``main_grad`` get ordinary autograd gradients.
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


def _gemm_ws(device, nfloats: int) -> torch.Tensor:
    """Per-device fp32 split-K workspace (grown on demand, never shrunk)."""
    key = (device, "gemm_ws")
    buf = _SCRATCH.get(key)
    if buf is None or buf.numel() < nfloats:
        buf = torch.empty(max(nfloats, 1 << 20), dtype=torch.float32, device=device)
        _SCRATCH[key] = buf
    return buf


def _sink(p):
    return getattr(p, "main_grad", None)


def _ready(p):
    cb = getattr(p, "_nexar_on_ready", None)
    if cb is not None:
        cb()


def _grad_out(p, fill):
    """Write a parameter gradient: into its sink (returns None) or a new tensor."""
    g = _sink(p)
    if g is not None:
        fill(g)
        _ready(p)
        return None
    g = torch.empty_like(p)
    fill(g)
    return g


def matmul_nt(a, b, out=None, bias=None, act: int = 0, pre=None, a_t: bool = False, b_t: bool = False,
              accumulate: bool = False, splits: int = 0):
    """out = act(opA . opB^T + bias) on the tcgen05 GEMM.

    opA = a ([M, K]) or a^T when ``a_t`` (a stored as [K, M]); opB = b ([N, K])
    or b^T when ``b_t`` (b stored as [K, N]). ``splits=0`` picks split-K by
    the kernel's cost model (fp32 partials, deterministic reduction).
    """
    C = _native.cuda()
    M = a.shape[1] if a_t else a.shape[0]
    N = b.shape[1] if b_t else b.shape[0]
    K = a.shape[0] if a_t else a.shape[1]
    if out is None:
        out = torch.empty(M, N, dtype=a.dtype, device=a.device)
    sp = C.gemm_choose_splits(M, N, K) if splits == 0 else splits
    ws = _gemm_ws(a.device, C.gemm_split_workspace_bytes(M, N, sp) // 4) if sp > 1 else None
    C.gemm_ex(a, b, out, a_t, b_t, bias, None, pre, act, 1.0, accumulate, sp, ws)
    return out


def colsum(x, out, accumulate: bool = False):
    """out[c] (+)= sum over rows of x[:, c] (bf16 in/out, fp32 accumulation)."""
    C = _native.cuda()
    x2 = x.reshape(-1, x.shape[-1])
    scratch = _scratch(x.device, C.colsum_scratch_floats(x2.shape[0], x2.shape[1]))
    C.colsum(x2, out, scratch, accumulate)
    return out


class _Linear(torch.autograd.Function):
    """y = act(x . w^T + b) with the tcgen05 GEMM in all three products.

    backward: dx = dz . w (w read MN-major), dw = dz^T . x (both operands
    MN-major, split-K when the output has few tiles), db = column sums of dz,
    where dz = dy or gelu'(pre) * dy.
    """

    @staticmethod
    def forward(ctx, x, w, b, act, ready):
        K = x.shape[-1]
        x2 = x.reshape(-1, K)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        M, N = x2.shape[0], w.shape[0]
        y = torch.empty(M, N, dtype=x.dtype, device=x.device)
        pre = torch.empty_like(y) if act else None
        matmul_nt(x2, w, out=y, bias=b, act=act, pre=pre, splits=1)
        ctx.save_for_backward(x2, w, pre)
        ctx.has_b = b is not None
        ctx.bias_param = b
        ctx.act, ctx.ready = act, ready
        ctx.in_shape = x.shape
        return y.view(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, dy):
        x2, w, pre = ctx.saved_tensors
        N = w.shape[0]
        dz = dy.reshape(-1, N)
        if not dz.is_contiguous():
            dz = dz.contiguous()
        if ctx.act:
            d = torch.empty_like(pre)
            _native.cuda().gelu_bwd(pre, dz, d)
            dz = d
        dx = matmul_nt(dz, w, b_t=True) if ctx.needs_input_grad[0] else None

        def fill_w(g):
            matmul_nt(dz, x2, out=g.view(N, -1), a_t=True, b_t=True)

        if ctx.ready:
            gw = _grad_out(w, fill_w)
        else:
            # shared (tied) weight: another op adds to the sink afterwards and signals
            g = _sink(w)
            if g is not None:
                fill_w(g)
                gw = None
            else:
                gw = torch.empty_like(w)
                fill_w(gw)
        gb = None
        if ctx.has_b:
            gb = _grad_out(ctx.bias_param, lambda g: colsum(dz, g))
        return (dx.view(ctx.in_shape) if dx is not None else None), gw, gb, None, None


def linear(x, w, b=None, act: str = None, ready: bool = True):
    """x . w^T (+ b), optionally followed by GELU (tanh) fused into the GEMM epilogue.

    ``ready=False`` marks a weight whose gradient sink receives a further
    contribution later in backward (tied embeddings): it is overwritten here
    and the later op signals readiness.
    """
    return _Linear.apply(x, w, b, 1 if act == "gelu" else 0, ready)


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
        ctx.b = b
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, mean, rstd = ctx.saved_tensors
        C = x2.shape[-1]
        dy2 = dy.contiguous().view(-1, C)
        dx = torch.empty_like(x2)
        dw, db = _sink(w), _sink(ctx.b)
        ret_w = ret_b = None
        if dw is None:
            dw = ret_w = torch.empty_like(w)
        if db is None:
            db = ret_b = torch.empty_like(w)
        C_ = _native.cuda()
        scratch = _scratch(x2.device, C_.ln_bwd_scratch_floats(x2.shape[0], C))
        C_.ln_bwd(dy2, x2, mean, rstd, w, None, dx, dw, db, scratch, _counter(x2.device))
        if ret_w is None:
            _ready(w)
        if ret_b is None:
            _ready(ctx.b)
        return dx.view(ctx.shape), ret_w, ret_b, None


def layer_norm(x, w, b, eps: float = 1e-5):
    return _LayerNorm.apply(x, w, b, eps)


class _ResidualLayerNorm(torch.autograd.Function):
    """s = x + r (+ rb) ; y = LayerNorm(s). Returns (s, y).

    ``rb`` is the bias of the layer that produced r, folded into the add so
    that layer's GEMM needs no bias epilogue; its gradient (column sums of
    ds) comes out of the LayerNorm backward kernel.
    """

    @staticmethod
    def forward(ctx, x, r, w, b, rb, eps):
        C = x.shape[-1]
        x2 = x.reshape(-1, C)
        r2 = r.reshape(-1, C)
        R = x2.shape[0]
        s = torch.empty_like(x2)
        y = torch.empty_like(x2)
        mean = torch.empty(R, dtype=torch.float32, device=x.device)
        rstd = torch.empty(R, dtype=torch.float32, device=x.device)
        _native.cuda().ln_fwd(x2, r2, s, w, b, y, mean, rstd, eps, rb)
        ctx.save_for_backward(s, w, mean, rstd)
        ctx.b, ctx.rb = b, rb
        ctx.shape = x.shape
        return s.view(x.shape), y.view(x.shape)

    @staticmethod
    def backward(ctx, ds, dy):
        s, w, mean, rstd = ctx.saved_tensors
        C = s.shape[-1]
        dx = torch.empty_like(s)
        outs = []
        for p in (w, ctx.b, ctx.rb):
            if p is None:
                outs.append((None, None))
                continue
            g = _sink(p)
            outs.append((g, None) if g is not None else (None, torch.empty_like(p)))
        dw = outs[0][0] if outs[0][0] is not None else outs[0][1]
        db = outs[1][0] if outs[1][0] is not None else outs[1][1]
        drb = None
        if ctx.rb is not None:
            drb = outs[2][0] if outs[2][0] is not None else outs[2][1]
        C_ = _native.cuda()
        scratch = _scratch(s.device, C_.ln_bwd_scratch_floats(s.shape[0], C, drb is not None))
        dres = None if ds is None else ds.contiguous().view(-1, C)
        if dy is None:
            dy = torch.zeros_like(s)
        C_.ln_bwd(dy.contiguous().view(-1, C), s, mean, rstd, w, dres, dx, dw, db, scratch, _counter(s.device), drb)
        for p, (sink, _) in zip((w, ctx.b, ctx.rb), outs):
            if p is not None and sink is not None:
                _ready(p)
        dx = dx.view(ctx.shape)
        return dx, dx, outs[0][1], outs[1][1], (outs[2][1] if ctx.rb is not None else None), None


def residual_layer_norm(x, r, w, b, eps: float = 1e-5, rbias=None):
    return _ResidualLayerNorm.apply(x, r, w, b, rbias, eps)


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


class _Attention(torch.autograd.Function):
    """Multi-head self-attention on the tcgen05 kernels (head dimension 64).

    qkv: [B*T, 3C] bf16 ([B, T, 3, H, 64] flattened, the QKV projection's
    output); returns y [B*T, C] bf16 ([B, T, H, 64]). The forward saves the
    per-row log-sum-exp; the backward recomputes the probabilities from it and
    writes the gradient of qkv in one buffer."""

    @staticmethod
    def forward(ctx, qkv, B: int, T: int, H: int, causal: bool):
        qkv = qkv.contiguous()
        C = H * 64
        y = torch.empty(B * T, C, dtype=qkv.dtype, device=qkv.device)
        lse = torch.empty(B * H * T, dtype=torch.float32, device=qkv.device)
        _native.cuda().attn_fwd(qkv, y, lse, B, T, H, causal)
        ctx.save_for_backward(qkv, y, lse)
        ctx.shape = (B, T, H, causal)
        return y

    @staticmethod
    def backward(ctx, dy):
        qkv, y, lse = ctx.saved_tensors
        B, T, H, causal = ctx.shape
        C = _native.cuda()
        dqkv = torch.empty_like(qkv)
        ws = _SCRATCH.get((qkv.device, "attn_ws"))
        need = C.attn_bwd_workspace_floats(B, T, H)
        if ws is None or ws.numel() < need:
            ws = torch.empty(need, dtype=torch.float32, device=qkv.device)
            _SCRATCH[(qkv.device, "attn_ws")] = ws
        C.attn_bwd(qkv, y, dy.contiguous(), lse, dqkv, ws, B, T, H, causal)
        return dqkv, None, None, None, None


def attention_supported(B: int, T: int, H: int, head_dim: int) -> bool:
    """Shapes the tcgen05 attention kernels take: head dimension 64, T a multiple of 128."""
    return bool(_native.cuda().attn_supported(B, T, H, head_dim))


def attention(qkv, B: int, T: int, H: int, causal: bool = True):
    """softmax(Q K^T / 8 [+ causal mask]) V for every head of qkv [B*T, 3C]; returns [B*T, C]."""
    return _Attention.apply(qkv, B, T, H, causal)


class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tok, wte, wpe):
        B, T = tok.shape
        C = wte.shape[1]
        out = torch.empty(B, T, C, dtype=wte.dtype, device=wte.device)
        _native.cuda().embed_fwd(tok, wte, wpe, out, T)
        ctx.save_for_backward(tok)
        ctx.shapes = (wte.shape, wpe.shape)
        ctx.params = (wte, wpe)
        return out

    @staticmethod
    def backward(ctx, dout):
        (tok,) = ctx.saved_tensors
        B, T = tok.shape
        wte_shape, wpe_shape = ctx.shapes
        wte, wpe = ctx.params
        # wte's sink already holds the tied head's gradient (written earlier
        # in backward): the token scatter adds onto it. wpe is overwritten.
        swte, swpe = _sink(wte), _sink(wpe)
        dwte = swte if swte is not None else torch.zeros(wte_shape, dtype=dout.dtype, device=dout.device)
        dwpe = swpe if swpe is not None else torch.zeros(wpe_shape, dtype=dout.dtype, device=dout.device)
        _native.cuda().embed_bwd(tok, dout.contiguous(), dwte, dwpe, B, T)
        if T < wpe_shape[0]:
            dwpe[T:].zero_()  # positions past T get no gradient this step
        if swte is not None:
            _ready(wte)
        if swpe is not None:
            _ready(wpe)
        return None, (None if swte is not None else dwte), (None if swpe is not None else dwpe)


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


def quant_fp8_1x128(x):
    """bf16 [R, K] -> (e4m3 [R, K], fp32 scales [R, ceil(K/128)]), scale = amax/448 per 1x128 block."""
    x2 = x.reshape(-1, x.shape[-1])
    R, K = x2.shape
    q = torch.empty(R, K, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(R, (K + 127) // 128, dtype=torch.float32, device=x.device)
    _native.cuda().quant_fp8_1x128(x2, q, s)
    return q, s


def quant_fp8_128x128(w):
    """bf16 [N, K] -> (e4m3 [N, K], fp32 scales [ceil(N/128), ceil(K/128)]) per 128x128 block."""
    N, K = w.shape
    q = torch.empty(N, K, dtype=torch.float8_e4m3fn, device=w.device)
    s = torch.empty((N + 127) // 128, (K + 127) // 128, dtype=torch.float32, device=w.device)
    _native.cuda().quant_fp8_128x128(w, q, s)
    return q, s


def matmul_fp8(a_q, a_s, b_q, b_s, out=None, bias=None, act: int = 0, pre=None, alpha: float = 1.0):
    """out[M, N] = act(alpha * (a_q * a_s) . (b_q * b_s)^T + bias) on the block-scaled fp8 tcgen05 GEMM."""
    M, N = a_q.shape[0], b_q.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.bfloat16, device=a_q.device)
    _native.cuda().gemm_fp8(a_q, a_s, b_q, b_s, out, bias, pre, act, alpha)
    return out


def swiglu_quant_fp8(gu):
    """gu [R, 2F] bf16 (gate | up) -> (e4m3 [R, F], fp32 scales [R, ceil(F/128)]) of silu(gate) * up."""
    R, F2 = gu.shape
    F = F2 // 2
    q = torch.empty(R, F, dtype=torch.float8_e4m3fn, device=gu.device)
    s = torch.empty(R, (F + 127) // 128, dtype=torch.float32, device=gu.device)
    _native.cuda().swiglu_quant_fp8(gu.contiguous(), q, s)
    return q, s
