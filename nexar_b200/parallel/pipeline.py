"""Pipeline parallelism: one model stage per rank, a 1F1B micro-batch schedule.

Rank s of W runs stage s. Activations travel forward (stage s -> s + 1) and
their gradients backward (s + 1 -> s) as point-to-point messages: on the box
over NCCL p2p (:class:`NcclP2P`, an ``NcclGroup`` carrying device send /
recv), on CPU tensors over a host ``NexarClient`` (:class:`HostP2P`, tagged
send / recv). The reference has no pipeline schedule; it offers the tagged
send / recv this builds on (nexar/src/client/async_client.rs:312-379).

Schedule (one-forward-one-backward, as in PipeDream-Flush / Megatron): stage
s runs min(W - 1 - s, M) warm-up forwards, then alternates one forward and
one backward until all M forwards ran, then drains the remaining backwards.
At most W - s micro-batches are in flight on stage s, so activation memory is
bounded by the pipeline depth rather than by M. Gradients of the stage's
parameters accumulate over the micro-batches (the caller zeroes them and
steps the optimizer).
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence

import torch


class HostP2P:
    """Activation / gradient transfer between CPU ranks over a host client.
    Messages are tagged by (micro-batch, direction); host sends never wait
    for the receiver, so a combined send + receive is a send then a receive."""

    def __init__(self, client):
        self.client = client
        self.rank = client.rank
        self.world_size = client.world_size

    @staticmethod
    def _tag(mb: int, backward: bool) -> int:
        return (mb << 1) | int(backward)

    def send(self, t: torch.Tensor, dst: int, mb: int, backward: bool):
        t = t.detach().contiguous()
        self.client.send(t.data_ptr(), t.numel() * t.element_size(), dst, self._tag(mb, backward))

    def recv(self, shape, dtype, src: int, mb: int, backward: bool) -> torch.Tensor:
        t = torch.empty(shape, dtype=dtype)
        self.client.recv(t.data_ptr(), t.numel() * t.element_size(), src, self._tag(mb, backward))
        return t

    def send_recv(self, t, dst, send_mb, send_bwd, shape, dtype, src, recv_mb, recv_bwd):
        self.send(t, dst, send_mb, send_bwd)
        return self.recv(shape, dtype, src, recv_mb, recv_bwd)


class NcclP2P:
    """Activation / gradient transfer between GPUs over an NcclGroup. A
    combined send + receive is one NCCL group (send_recv), so two neighbours
    that each send to the other first cannot wait on each other."""

    def __init__(self, group, device: Optional[torch.device] = None):
        self.group = group
        self.rank = group.local_rank
        self.world_size = group.local_world
        self.device = device or torch.device("cuda", group.device)

    def send(self, t: torch.Tensor, dst: int, mb: int, backward: bool):
        self.group.send(t.detach().contiguous(), dst)

    def recv(self, shape, dtype, src: int, mb: int, backward: bool) -> torch.Tensor:
        t = torch.empty(shape, dtype=dtype, device=self.device)
        self.group.recv(t, src)
        return t

    def send_recv(self, t, dst, send_mb, send_bwd, shape, dtype, src, recv_mb, recv_bwd):
        out = torch.empty(shape, dtype=dtype, device=self.device)
        self.group.send_recv(t.detach().contiguous(), dst, out, src)
        return out


def schedule_1f1b(stage: int, stages: int, micro_batches: int) -> List[tuple]:
    """The (kind, micro-batch) sequence stage `stage` runs: kind "F" or "B"."""
    warm = min(stages - 1 - stage, micro_batches)
    out = [("F", i) for i in range(warm)]
    f, b = warm, 0
    while f < micro_batches:
        out.append(("F", f))
        f += 1
        out.append(("B", b))
        b += 1
    while b < micro_batches:
        out.append(("B", b))
        b += 1
    return out


def run_1f1b(module: torch.nn.Module, p2p, micro_batches: Sequence[torch.Tensor],
             act_shape: Sequence[int], act_dtype=torch.float32,
             loss_fn: Optional[Callable[[torch.Tensor, int], torch.Tensor]] = None) -> List[float]:
    """Run forward + backward of all micro-batches through this rank's stage.

    micro_batches: the inputs of the first stage (other stages only use their
    count; they receive activations of shape ``act_shape``, and every stage's
    output has that shape). loss_fn(output, i) gives the scalar loss of
    micro-batch i on the last stage. Returns the last stage's losses (empty
    elsewhere).

    Transfers follow the usual 1F1B pairing: in the steady phase a stage sends
    its forward output together with receiving the gradient it needs next,
    and sends an input gradient together with receiving the next input."""
    s, W = p2p.rank, p2p.world_size
    M = len(micro_batches)
    first, last = s == 0, s == W - 1
    if last and loss_fn is None:
        raise ValueError("the last stage needs a loss_fn")
    shape = tuple(act_shape)
    losses: List[float] = []
    inputs: dict = {}
    outputs: dict = {}

    def recv_forward(i):
        if first:
            return micro_batches[i]
        return p2p.recv(shape, act_dtype, s - 1, i, False).requires_grad_(True)

    def forward(i, x):
        y = module(x)
        inputs[i] = x
        if last:
            loss = loss_fn(y, i)
            losses.append(float(loss.detach()))
            outputs[i] = loss
        else:
            outputs[i] = y
        return y

    def backward(i, dy):
        y, x = outputs.pop(i), inputs.pop(i)
        if last:
            y.backward()
        else:
            y.backward(dy)
        return None if first else x.grad

    warm = min(W - 1 - s, M)
    steady = M - warm
    for i in range(warm):
        y = forward(i, recv_forward(i))
        if not last:
            p2p.send(y, s + 1, i, False)
    x = recv_forward(warm) if steady > 0 else None
    for k in range(steady):
        i, j = warm + k, k          # forward of micro-batch i, then backward of micro-batch j
        y = forward(i, x)
        if last:
            dy = None
        else:
            dy = p2p.send_recv(y, s + 1, i, False, shape, act_dtype, s + 1, j, True)
        dx = backward(j, dy)
        if k == steady - 1:
            if not first:
                p2p.send(dx, s - 1, j, True)
        elif first:
            x = recv_forward(i + 1)
        else:
            x = p2p.send_recv(dx, s - 1, j, True, shape, act_dtype, s - 1, i + 1, False).requires_grad_(True)
    for j in range(steady, M):
        dy = None if last else p2p.recv(shape, act_dtype, s + 1, j, True)
        dx = backward(j, dy)
        if not first:
            p2p.send(dx, s - 1, j, True)
    return losses
