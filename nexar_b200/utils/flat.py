"""Flat parameter / gradient storage.

All trainable tensors of a model live as views of a few flat buffers:
  * ``param_bf16``   compute copy used by forward/backward,
  * ``master``       fp32 master weights, ``exp_avg``/``exp_avg_sq`` (AdamW),
  * ``grad``         bf16 gradients (may live in the symmetric heap so the
                     data-parallel all-reduce runs in place without copies).

Layout: parameters that take weight decay (matrices) come first, in the
reverse of their forward-use order, then the ones that do not (biases,
norms). Gradient buckets are contiguous ranges of this layout, so the first
bucket to complete in backward is the first one in memory.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch


@dataclass
class FlatEntry:
    name: str
    shape: Tuple[int, ...]
    offset: int
    numel: int
    decay: bool


class FlatParams:
    def __init__(self, specs: Sequence[Tuple[str, Tuple[int, ...], bool]], device,
                 grad_alloc: Optional[Callable[[int], torch.Tensor]] = None, align: int = 64):
        """specs: (name, shape, decay) in forward-use order."""
        decay = [s for s in specs if s[2]]
        nodecay = [s for s in specs if not s[2]]
        ordered = list(reversed(decay)) + list(reversed(nodecay))
        self.entries: List[FlatEntry] = []
        off = 0
        for name, shape, dec in ordered:
            n = 1
            for d in shape:
                n *= d
            self.entries.append(FlatEntry(name, tuple(shape), off, n, dec))
            off += (n + align - 1) // align * align
        self.numel = off
        self.decay_end = sum((e.numel + align - 1) // align * align for e in self.entries if e.decay)
        self.device = device
        self.param_bf16 = torch.zeros(self.numel, dtype=torch.bfloat16, device=device)
        self.master = torch.zeros(self.numel, dtype=torch.float32, device=device)
        self.exp_avg = torch.zeros(self.numel, dtype=torch.float32, device=device)
        self.exp_avg_sq = torch.zeros(self.numel, dtype=torch.float32, device=device)
        if grad_alloc is not None:
            self.grad = grad_alloc(self.numel)
        else:
            self.grad = torch.zeros(self.numel, dtype=torch.bfloat16, device=device)
        self.by_name: Dict[str, FlatEntry] = {e.name: e for e in self.entries}

    def view(self, buf: torch.Tensor, name: str) -> torch.Tensor:
        e = self.by_name[name]
        return buf[e.offset:e.offset + e.numel].view(e.shape)

    def params(self) -> Dict[str, torch.nn.Parameter]:
        out = {}
        for e in self.entries:
            p = torch.nn.Parameter(self.view(self.param_bf16, e.name), requires_grad=True)
            p.grad = self.view(self.grad, e.name)
            p.main_grad = p.grad  # gradient sink written directly by the backward kernels
            out[e.name] = p
        return out

    def sync_master_from_bf16(self):
        self.master.copy_(self.param_bf16.float())

    def buckets(self, bucket_bytes: int) -> List[Tuple[int, int, List[str]]]:
        """Contiguous (start, end, names) ranges of about bucket_bytes of bf16 grads."""
        cap = max(1, bucket_bytes // 2)
        out: List[Tuple[int, int, List[str]]] = []
        cur_start, cur_names = None, []
        for i, e in enumerate(self.entries):
            if cur_start is None:
                cur_start = e.offset
            cur_names.append(e.name)
            end = self.entries[i + 1].offset if i + 1 < len(self.entries) else self.numel
            last_of_section = (i + 1 == len(self.entries)) or (self.entries[i + 1].decay != e.decay)
            if end - cur_start >= cap or last_of_section:
                out.append((cur_start, end, cur_names))
                cur_start, cur_names = None, []
        return out
