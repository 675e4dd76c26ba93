"""The data-parallel trainer counts every parameter once per step before it
launches a gradient bucket (CPU; no GPU needed).

PyTorch runs a parameter's post-accumulate hook after its AccumulateGrad
node even when every backward op returned None for it. The trainer's
kernels write gradients straight into the flat buffer and report readiness
themselves, so the autograd hook must not count those parameters a second
time: with the double count, a bucket was reduced while half of its
gradients were still being written.
"""
import torch

from nexar_b200.parallel.dp import DataParallelTrainer


class _Sink(torch.autograd.Function):
    """Writes nothing through autograd (returns None for w) and reports w ready itself."""

    @staticmethod
    def forward(ctx, x, w):
        ctx.w = w
        return x * 2

    @staticmethod
    def backward(ctx, g):
        ctx.w._nexar_on_ready()
        return g * 2, None


def _trainer_shell(buckets):
    """A DataParallelTrainer with only the bookkeeping the ready hooks use."""
    tr = DataParallelTrainer.__new__(DataParallelTrainer)
    tr.buckets = buckets
    tr._bucket_of = {n: bi for bi, (_, _, names) in enumerate(buckets) for n in names}
    tr._bucket_need = [len(names) for _, _, names in buckets]
    tr._bucket_left = list(tr._bucket_need)
    tr._seen = set()
    tr._zero_grads = False
    tr.launched = []
    tr._launch_bucket = lambda bi: tr.launched.append((bi, sorted(tr._seen)))
    return tr


def test_post_accumulate_hook_fires_on_none_gradients():
    # The PyTorch behaviour the trainer has to allow for.
    w = torch.nn.Parameter(torch.ones(3))
    w.grad = torch.zeros(3)
    calls = []
    w._nexar_on_ready = lambda: calls.append("kernel")
    w.register_post_accumulate_grad_hook(lambda p: calls.append("autograd"))
    _Sink.apply(torch.ones(3, requires_grad=True), w).sum().backward()
    assert calls == ["kernel", "autograd"]


def test_bucket_launches_once_all_its_parameters_are_ready():
    tr = _trainer_shell([(0, 6, ["a", "b"]), (6, 9, ["c"])])
    params = {}
    for n in ("a", "b", "c"):
        p = torch.nn.Parameter(torch.ones(3))
        p.grad = torch.zeros(3)
        p._nexar_on_ready = tr._make_hook(n)
        p.register_post_accumulate_grad_hook(tr._make_acc_hook(n))
        params[n] = p
    x = torch.ones(3, requires_grad=True)
    # backward order: c, then b, then a (each op reports its parameter, autograd then runs its hook)
    y = _Sink.apply(_Sink.apply(_Sink.apply(x, params["a"]), params["b"]), params["c"])
    y.sum().backward()
    assert tr.launched == [(1, ["c"]), (0, ["a", "b", "c"])]
    assert tr._zero_grads is False  # no gradient went through autograd accumulation


def test_autograd_accumulated_gradient_counts_once():
    tr = _trainer_shell([(0, 3, ["w"])])
    w = torch.nn.Parameter(torch.ones(3))
    w._nexar_on_ready = tr._make_hook("w")
    w.register_post_accumulate_grad_hook(tr._make_acc_hook("w"))
    (torch.ones(3, requires_grad=True) * w).sum().backward()  # plain autograd: no kernel report
    assert tr.launched == [(0, ["w"])]
    assert tr._zero_grads is True  # accumulation needs a zeroed buffer next step
