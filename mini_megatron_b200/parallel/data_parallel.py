"""Data-parallel gradient synchronisation.

``allreduce_grads`` keeps the reference API (parallel/data_parallel.py:5-15):
a blocking per-parameter all-reduce followed by a divide.

``GradSync`` is the framework path: gradients live in a flat buffer split
into buckets (see ParamBuffer); a bucket is reduced as soon as backward has
produced all of its gradients, so the collective overlaps the backward of
the earlier layers.  Buckets are issued strictly in buffer order, which is
the same on every rank, so all ranks run the same collectives in the same
order.  The 1/dp average is NOT applied here: it is folded into the
optimizer kernel (``grad_scale``), saving a pass over the gradients.

Modes:
  ``allreduce``      every rank gets the full summed gradient (plain DP)
  ``reduce_scatter`` each rank gets only its shard of every bucket (ZeRO-1)
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .param_buffer import ParamBuffer


def allreduce_grads(model_or_params, dp_group):
    if dp_group is None or dist.get_world_size(dp_group) <= 1:
        return
    params = model_or_params if isinstance(model_or_params, list) else list(model_or_params.parameters())
    world = dist.get_world_size(dp_group)
    for p in params:
        if p.grad is not None:
            dist.all_reduce(p.grad, group=dp_group)
            p.grad.div_(world)


class GradSync:
    def __init__(self, buf: ParamBuffer, dp_group, mode: str = "allreduce", overlap: bool = True):
        if mode not in ("allreduce", "reduce_scatter"):
            raise ValueError(mode)
        self.buf, self.group, self.mode, self.overlap = buf, dp_group, mode, overlap
        self.world = 1 if dp_group is None else dist.get_world_size(dp_group)
        self.rank = 0 if dp_group is None else dist.get_rank(dp_group)
        self._bucket_of = {}
        for b, (_, _, params) in enumerate(buf.buckets):
            for p in params:
                self._bucket_of[id(p)] = b
        self.reset()

    @property
    def active(self) -> bool:
        return self.world > 1

    def reset(self):
        self._pending = [len(params) for (_, _, params) in self.buf.buckets]
        self._next = 0
        self._works = []

    def attach(self, modules):
        """Mark a module's parameters ready when its native backward finishes."""
        self.attached_params = getattr(self, "attached_params", set())
        for m in modules:
            params = [p for p in m.parameters() if id(p) in self._bucket_of]
            self.attached_params.update(id(p) for p in params)
            hooks = list(getattr(m, "_mmb_grad_ready_hooks", ()))
            hooks.append(lambda ps=params: self.mark_ready(ps))
            m._mmb_grad_ready_hooks = hooks

    def mark_ready(self, params):
        if not (self.active and self.overlap):
            return
        for p in params:
            b = self._bucket_of.get(id(p))
            if b is not None:
                self._pending[b] -= 1
        while self._next < len(self._pending) and self._pending[self._next] <= 0:
            self._launch(self._next)
            self._next += 1

    def _launch(self, b):
        s, e, _ = self.buf.buckets[b]
        g = self.buf.grad[s:e]
        if self.mode == "allreduce":
            self._works.append(dist.all_reduce(g, group=self.group, async_op=True))
        else:
            lo, hi = self.buf.shard_range(b, self.rank)
            self._works.append(dist.reduce_scatter_tensor(self.buf.grad[lo:hi], g, group=self.group, async_op=True))

    def finish(self):
        """Issue the buckets not yet launched (in order) and wait for all of them."""
        if not self.active:
            return
        while self._next < len(self.buf.buckets):
            self._launch(self._next)
            self._next += 1
        for w in self._works:
            w.wait()
        self.reset()


def allreduce_sequence_parallel_grads(params, tp_group):
    """Sum gradients of replicated parameters that saw only a sequence shard (SP LayerNorms)."""
    if tp_group is None or dist.get_world_size(tp_group) == 1:
        return
    grads = [p.main_grad if getattr(p, "main_grad", None) is not None else p.grad for p in params
             if getattr(p, "sequence_parallel_grad", False)]
    grads = [g for g in grads if g is not None]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat, group=tp_group)
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[off:off + n].view_as(g))
        off += n
