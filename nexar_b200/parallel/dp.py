"""Data-parallel training entry point (the GPT-2-small benchmark configuration).

One process per GPU. Gradients live in one flat bf16 buffer inside the
symmetric heap, split into ~25 MB buckets (contiguous ranges). A
parameter's ready callback (called by the backward kernel that wrote its
gradient, or autograd's post-accumulate hook when autograd did) counts
finished parameters per bucket, each once per step; when a bucket is
complete its all-reduce (two-shot over NVLink, averaging scale 1/world fused
into the kernel, in place, no staging copies) is launched on the
communicator's side stream, overlapping the rest of backward. Buckets that
overlap backward run on a small grid (``overlap_blocks`` CTAs,
``NEXAR_DP_AR_BLOCKS``, default 64: 2-GPU step 10.35 ms against 10.52 ms
with 32) so the persistent GEMM kernels keep most of their SMs; the
last buckets, which run after backward has finished, take the whole GPU.
With ``timeline=True`` (``NEXAR_DP_TIMELINE=1``) CUDA events mark, per
bucket, when it became ready on the compute stream and when its all-reduce
started and ended, plus the end of backward (:meth:`timeline`). The optimizer
step (global-norm clip + fused AdamW over flat fp32 master weights) runs
after the last bucket joins. The whole step can be captured in one CUDA graph.

The reference offers only the primitives for this (all_reduce_nb +
CollectiveGroup, nexar/src/client/collectives_nb.rs:33-47; host-only bucketed
all-reduce, nexar/src/collective/bucketed_allreduce.rs:23-75).
"""
from __future__ import annotations

import dataclasses
import os
import time
from typing import List, Optional

import torch

from .. import _native
from ..models.gpt2 import GPT2, GPT2Config


class DataParallelTrainer:
    def __init__(self, cfg: GPT2Config, micro_batch: int, seq_len: int, comm=None, device=None,
                 lr: float = 6e-4, betas=(0.9, 0.95), eps: float = 1e-8, weight_decay: float = 0.1,
                 grad_clip: float = 1.0, bucket_bytes: int = 25 << 20, seed: int = 0,
                 use_cuda_graph: bool = True, overlap_blocks: Optional[int] = None,
                 timeline: Optional[bool] = None):
        self.cfg = cfg
        self.B, self.T = micro_batch, seq_len
        self.comm = comm
        self.world = comm.world_size if comm is not None else 1
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        grad_alloc = None
        if self.world > 1:
            # NVLS region when NVLS is the better all-reduce at this size of job,
            # else the peer-mapped heap (zero-copy two-shot)
            grad_alloc = lambda n: comm.symmetric_empty(  # noqa: E731
                [n], torch.bfloat16, nvls=getattr(comm, "nvls_preferred", False))
        self.model = GPT2(cfg, self.device, grad_alloc=grad_alloc, seed=seed)
        flat = self.model.flat
        flat.grad.zero_()  # padding between parameters is never written
        if self.world > 1:
            # identical start on every rank (ranks share the seed; this makes it exact)
            comm.broadcast(flat.master, root=0)
            flat.param_bf16.copy_(flat.master)
        self.lr, self.betas, self.eps, self.wd, self.clip = lr, betas, eps, weight_decay, grad_clip
        self.step_dev = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.lr_dev = torch.full((1,), lr, dtype=torch.float32, device=self.device)
        C = _native.cuda()
        self._C = C
        self.norm_scratch = torch.empty(C.grad_norm_blocks(flat.numel), dtype=torch.float32, device=self.device)
        self.norm_counter = torch.zeros(4, dtype=torch.int32, device=self.device)
        self.grad_norm = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.clip_coef = torch.ones(1, dtype=torch.float32, device=self.device)
        # buckets + hooks
        self.buckets = flat.buckets(bucket_bytes) if self.world > 1 else []
        self._bucket_of = {}
        self._bucket_need: List[int] = []
        for bi, (_, _, names) in enumerate(self.buckets):
            for n in names:
                self._bucket_of[n] = bi
            self._bucket_need.append(len(names))
        self._bucket_left: List[int] = list(self._bucket_need)
        self._launched: List[bool] = [False] * len(self.buckets)
        self.overlap_blocks = int(overlap_blocks if overlap_blocks is not None
                                  else os.environ.get("NEXAR_DP_AR_BLOCKS", "64"))
        self.tail_buckets = 2  # launched once backward has (nearly) finished: full grid
        if timeline is None:
            timeline = os.environ.get("NEXAR_DP_TIMELINE", "0") == "1"
        self._tl = None
        if timeline and self.world > 1:
            # external: recorded as event nodes when the step is captured in a
            # CUDA graph, so the replayed step still timestamps them.
            ev = lambda: torch.cuda.Event(enable_timing=True, external=True)  # noqa: E731
            self._tl = {"step0": ev(), "bwd_end": ev(), "step_end": ev(),
                        "ready": [ev() for _ in self.buckets], "start": [ev() for _ in self.buckets],
                        "end": [ev() for _ in self.buckets], "order": []}
        # Backward kernels write each gradient straight into the flat buffer
        # and then call the parameter's ready callback (no zero-fill, no
        # accumulation). A parameter that is ever missed falls back to
        # zero-fill + autograd accumulation for every later step.
        self._zero_grads = False
        self._seen = set()
        for name, par in self.model.p.items():
            par._nexar_on_ready = self._make_hook(name)
            par.register_post_accumulate_grad_hook(self._make_acc_hook(name))
        self.static_idx = torch.zeros(self.B, self.T, dtype=torch.int64, device=self.device)
        self.static_tgt = torch.zeros(self.B, self.T, dtype=torch.int64, device=self.device)
        self.static_loss = torch.zeros((), dtype=torch.float32, device=self.device)
        self.use_cuda_graph = use_cuda_graph
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.graph_launches = 0
        self._host_loss = torch.zeros((), dtype=torch.float32).pin_memory()

    # ---------------------------------------------------------------- hooks
    def _make_hook(self, name):
        bi = self._bucket_of.get(name)

        def hook():
            self._seen.add(name)
            if bi is None:
                return
            self._bucket_left[bi] -= 1
            if self._bucket_left[bi] == 0:
                self._launch_bucket(bi)
        return hook

    def _make_acc_hook(self, name):
        def hook(_param):
            # PyTorch runs this after the parameter's AccumulateGrad node even
            # when every backward op returned None for it (the kernels wrote
            # the sink and reported ready themselves): count it only when
            # autograd really accumulated a gradient, or the bucket would be
            # reduced before its other parameters' gradients exist.
            if name in self._seen:
                return
            # autograd accumulated into the flat view: only valid over a zeroed buffer
            self._zero_grads = True
            self._make_hook(name)()
        return hook

    def _launch_bucket(self, bi):
        start, end, _ = self.buckets[bi]
        side = self.comm.side_stream()
        cur = torch.cuda.current_stream(self.device)
        tl = self._tl
        if tl is not None:
            tl["ready"][bi].record(cur)
            tl["order"].append(bi)
        side.wait_stream(cur)
        n_before = sum(self._launched)
        tail = n_before >= len(self.buckets) - self.tail_buckets
        with torch.cuda.stream(side):
            if tl is not None:
                tl["start"][bi].record(side)
            if tail:
                self.comm.all_reduce(self.model.flat.grad[start:end], scale=1.0 / self.world)
            else:
                with self.comm.block_limit(self.overlap_blocks):
                    self.comm.all_reduce(self.model.flat.grad[start:end], scale=1.0 / self.world)
            if tl is not None:
                tl["end"][bi].record(side)
        self._launched[bi] = True

    # ---------------------------------------------------------------- step
    def _step_body(self):
        flat = self.model.flat
        self._bucket_left = list(self._bucket_need)
        self._launched = [False] * len(self.buckets)
        self._seen = set()
        if self._zero_grads:
            flat.grad.zero_()
        tl = self._tl
        if tl is not None:
            tl["order"] = []
            tl["step0"].record()
        loss = self.model(self.static_idx, self.static_tgt, unit_grad=True)
        loss.backward()
        if tl is not None:
            tl["bwd_end"].record()
        if len(self._seen) != len(self.model.p):
            self._zero_grads = True  # some gradient was not written this step: zero-fill from now on
        if self.world > 1:
            for bi, done in enumerate(self._launched):
                if not done:  # parameters without gradient (none in GPT-2) still need averaging
                    self._launch_bucket(bi)
            torch.cuda.current_stream(self.device).wait_stream(self.comm.side_stream())
        C = self._C
        C.grad_norm_clip(flat.grad, self.clip, self.norm_scratch, self.norm_counter, self.grad_norm,
                         self.clip_coef)
        self.step_dev.add_(1)
        C.adamw(flat.master, flat.exp_avg, flat.exp_avg_sq, flat.grad, flat.param_bf16, flat.decay_end,
                self.lr, self.betas[0], self.betas[1], self.eps, self.wd, 1, self.clip_coef,
                self.step_dev, self.lr_dev)
        self.static_loss.copy_(loss.detach())
        if tl is not None:
            tl["step_end"].record()

    def timeline(self) -> Optional[dict]:
        """Milliseconds from the start of the last step (``timeline=True``):
        end of backward, end of the step, and per bucket (in launch order)
        its size and when it became ready / its all-reduce started / ended."""
        tl = self._tl
        if tl is None:
            return None
        torch.cuda.synchronize(self.device)
        t0 = tl["step0"]
        out = {"bwd_end_ms": t0.elapsed_time(tl["bwd_end"]), "step_end_ms": t0.elapsed_time(tl["step_end"]),
               "overlap_blocks": self.overlap_blocks, "buckets": []}
        for bi in tl["order"]:
            start, end, names = self.buckets[bi]
            out["buckets"].append({"bucket": bi, "mb": round((end - start) * 2 / 2**20, 2),
                                   "first": names[0], "last": names[-1],
                                   "ready_ms": round(t0.elapsed_time(tl["ready"][bi]), 3),
                                   "start_ms": round(t0.elapsed_time(tl["start"][bi]), 3),
                                   "end_ms": round(t0.elapsed_time(tl["end"][bi]), 3)})
        return out

    def capture(self, warmup: int = 3):
        """Warm up eagerly on a side stream, then capture one whole step."""
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._step_body()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        if not self.use_cuda_graph:
            return
        g = torch.cuda.CUDAGraph()
        before = _native.launch_count()
        with torch.cuda.graph(g):
            self._step_body()
        self.graph_launches = _native.launch_count() - before
        self.graph = g
        torch.cuda.synchronize(self.device)

    def run_step(self):
        """One training step on the static device inputs (device-side only)."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self._step_body()

    def set_batch(self, idx: torch.Tensor, tgt: torch.Tensor, non_blocking: bool = True):
        self.static_idx.copy_(idx, non_blocking=non_blocking)
        self.static_tgt.copy_(tgt, non_blocking=non_blocking)

    def step(self, idx_host: torch.Tensor, tgt_host: torch.Tensor) -> float:
        """Public end-to-end step: H2D of the batch, fwd/bwd/all-reduce/AdamW, D2H of the loss."""
        self.set_batch(idx_host, tgt_host)
        self.run_step()
        self._host_loss.copy_(self.static_loss, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        return float(self._host_loss.item())

    def tokens_per_step(self) -> int:
        return self.B * self.T * self.world

    def release(self):
        """Drop the captured graph (call before tearing down the process group)."""
        self.graph = None

    # ---------------------------------------------------------------- checkpoint / resume
    CHECKPOINT_FORMAT = "nexar_b200.dp_trainer/1"

    def state_dict(self) -> dict:
        """Everything a resumed run needs, as CPU tensors and plain values:
        fp32 master weights, both AdamW moments, the step counter, the learning
        rate, the optimizer settings, the model shape and the flat layout.
        Data-parallel ranks hold identical state, so one rank saves it."""
        torch.cuda.synchronize(self.device)
        flat = self.model.flat
        return {
            "format": self.CHECKPOINT_FORMAT,
            "config": dataclasses.asdict(self.cfg),
            "layout": [[e.name, list(e.shape), e.offset, e.numel] for e in flat.entries],
            "master": flat.master.detach().cpu(),
            "exp_avg": flat.exp_avg.detach().cpu(),
            "exp_avg_sq": flat.exp_avg_sq.detach().cpu(),
            "step": int(self.step_dev.item()),
            "lr": float(self.lr_dev.item()),
            "optim": {"betas": list(self.betas), "eps": self.eps, "weight_decay": self.wd, "grad_clip": self.clip},
        }

    def load_state_dict(self, sd: dict) -> None:
        """Restore a :meth:`state_dict` into this trainer's buffers, in place
        (a captured CUDA graph keeps working, unless the checkpoint's optimizer
        settings differ from the ones captured: then the graph is dropped and
        steps run eagerly until :meth:`capture` is called again). The model
        shape and flat layout must match; the bf16 working weights are
        re-derived from the fp32 master weights."""
        if sd.get("format") != self.CHECKPOINT_FORMAT:
            raise ValueError(f"not a {self.CHECKPOINT_FORMAT} checkpoint: {sd.get('format')!r}")
        if sd["config"] != dataclasses.asdict(self.cfg):
            raise ValueError(f"checkpoint is for model {sd['config']}, this trainer runs {dataclasses.asdict(self.cfg)}")
        flat = self.model.flat
        layout = [[e.name, list(e.shape), e.offset, e.numel] for e in flat.entries]
        if [list(x) for x in sd["layout"]] != layout:
            raise ValueError("checkpoint flat-parameter layout differs from this trainer's")
        torch.cuda.synchronize(self.device)
        flat.master.copy_(sd["master"])
        flat.exp_avg.copy_(sd["exp_avg"])
        flat.exp_avg_sq.copy_(sd["exp_avg_sq"])
        flat.param_bf16.copy_(flat.master)
        self.step_dev.fill_(int(sd["step"]))
        self.lr_dev.fill_(float(sd["lr"]))
        o = sd.get("optim", {})
        new = (tuple(o.get("betas", self.betas)), o.get("eps", self.eps), o.get("weight_decay", self.wd),
               o.get("grad_clip", self.clip))
        if new != (tuple(self.betas), self.eps, self.wd, self.clip) and self.graph is not None:
            # these settings are kernel arguments baked into the captured graph:
            # run eagerly until capture() is called again
            self.graph = None
        self.betas, self.eps, self.wd, self.clip = new
        torch.cuda.synchronize(self.device)

    def save(self, path: str) -> None:
        """Write :meth:`state_dict` to ``path`` (call on one rank)."""
        torch.save(self.state_dict(), path)

    def load(self, path: str) -> None:
        """Read a checkpoint written by :meth:`save` (every rank loads the same file)."""
        self.load_state_dict(torch.load(path, map_location="cpu", weights_only=True))
