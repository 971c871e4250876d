"""ZeRO-1 distributed optimizer over flat, bucketed parameter buffers.

The reference (parallel/distributed_optimizer.py:7-48) assigns whole
parameters round-robin to DP ranks, expects the caller to all-reduce full
gradients first, and broadcasts every parameter from its owner afterwards.
Here ownership is a contiguous, equal shard of every DP bucket of the flat
buffer, so:

1. gradients are reduce-scattered bucket by bucket (overlapped with backward
   by :class:`GradSync` in ``reduce_scatter`` mode): each rank receives only
   the summed gradient of the shard it owns;
2. AdamW runs on the owned shards only (fp32 master + moments exist only for
   the shard: 1/dp of the optimizer memory);
3. the updated fp32 shards are all-gathered back into every rank's flat
   buffer, and the bf16 GEMM shadow is re-derived.

API kept from the reference: ``step()``, ``zero_grad()``, ``sync_params()``,
``param_groups``; plus ``state_dict()/load_state_dict()`` of the shard state.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from .data_parallel import GradSync
from .param_buffer import ParamBuffer


class DistributedOptimizer(torch.optim.Optimizer):
    def __init__(self, buf: ParamBuffer, dp_group, lr=6e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                 overlap=True):
        self.buf, self.dp_group = buf, dp_group
        self.dp_size = 1 if dp_group is None else dist.get_world_size(dp_group)
        self.dp_rank = 0 if dp_group is None else dist.get_rank(dp_group)
        if buf.align % self.dp_size:
            raise ValueError("ParamBuffer must be built with align = dp size")
        super().__init__(list(buf.params), dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self.grad_sync = GradSync(buf, dp_group, mode="reduce_scatter", overlap=overlap)
        self.shards = [buf.shard_range(b, self.dp_rank) for b in range(len(buf.buckets))]
        n = sum(hi - lo for lo, hi in self.shards)
        self.exp_avg = torch.zeros(n, dtype=torch.float32, device=buf.data.device)
        self.exp_avg_sq = torch.zeros_like(self.exp_avg)
        self._step = 0

    @property
    def state_is_sharded(self):
        """Each DP rank holds only its own slice of the moments (checkpoints write one file per DP rank)."""
        return self.dp_size > 1

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        self.grad_sync.finish()  # reduce-scatter whatever backward has not yet issued
        self._step += 1
        g = self.param_groups[0]
        lr, (b1, b2), eps, wd = g["lr"], g["betas"], g["eps"], g["weight_decay"]
        scale = 1.0 / self.dp_size
        off = 0
        use_native = self.buf.data.is_cuda
        if use_native:
            from ..ops import native
            C = native()
        bc1 = 1 - b1 ** self._step
        bc2_sqrt = math.sqrt(1 - b2 ** self._step)
        for lo, hi in self.shards:
            n = hi - lo
            p, gr = self.buf.data[lo:hi], self.buf.grad[lo:hi]
            m, v = self.exp_avg[off:off + n], self.exp_avg_sq[off:off + n]
            if use_native:
                pb = self.buf.bf16[lo:hi] if self.buf.bf16 is not None else None
                C.adamw_flat(p, gr, m, v, pb, lr, b1, b2, eps, wd, self._step, scale)
            else:
                gg = gr * scale
                p.mul_(1 - lr * wd)
                m.lerp_(gg, 1 - b1)
                v.mul_(b2).addcmul_(gg, gg, value=1 - b2)
                p.addcdiv_(m, (v.sqrt() / bc2_sqrt).add_(eps), value=-lr / bc1)
            off += n
        self.sync_params()
        return loss

    @torch.no_grad()
    def sync_params(self):
        """All-gather every bucket's updated shards (fp32), then refresh the bf16 shadow."""
        if self.dp_size > 1:
            works = []
            for b, (s, e, _) in enumerate(self.buf.buckets):
                lo, hi = self.shards[b]
                works.append(dist.all_gather_into_tensor(self.buf.data[s:e], self.buf.data[lo:hi].clone(),
                                                         group=self.dp_group, async_op=True))
            for w in works:
                w.wait()
        self.buf.refresh_bf16()

    def zero_grad(self, set_to_none: bool = False):
        self.buf.zero_grad()

    def state_dict(self):
        return {
            "step": self._step,
            "dp_rank": self.dp_rank,
            "dp_size": self.dp_size,
            "shards": list(self.shards),
            "exp_avg": self.exp_avg.clone(),
            "exp_avg_sq": self.exp_avg_sq.clone(),
            "param_groups": [{k: v for k, v in g.items() if k != "params"} for g in self.param_groups],
        }

    def load_state_dict(self, sd):
        if sd["dp_size"] != self.dp_size or list(map(tuple, sd["shards"])) != list(map(tuple, self.shards)):
            raise ValueError("ZeRO-1 state was saved with a different DP layout")
        self._step = int(sd["step"])
        self.exp_avg.copy_(sd["exp_avg"])
        self.exp_avg_sq.copy_(sd["exp_avg_sq"])
        for g, s in zip(self.param_groups, sd["param_groups"]):
            g.update(s)

