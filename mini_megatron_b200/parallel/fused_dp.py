"""ZeRO-1 AdamW fused with the DP gradient reduce-scatter and parameter all-gather.

One kernel per gradient bucket (csrc/fused_dp.cu) runs on a side stream as
soon as backward has finished every parameter of that bucket:

    peer loads of the owned 1/dp slice of every rank's gradient (NVLink)
    -> sum, scale by 1/dp -> fp32 AdamW with this rank's sharded moments
    -> peer stores into every rank of the copy the forward kernels read:
       the bf16 shadow of a GEMM weight, the fp32 value of a LayerNorm or
       embedding parameter

so the data-parallel communication and the whole optimizer step overlap the
rest of backward, and no rank holds more than 1/dp of the optimizer state.
The fp32 master of a GEMM weight is current only on the rank that owns its
shard (ZeRO-1): :meth:`FusedDPOptimizer.gather_master` copies the other
shards in with peer loads, and runs automatically before the model's
``state_dict()``.  Code that reads GEMM-weight parameters directly between
steps (rather than through ``state_dict``) calls it first.
The parameter, gradient and bf16 buffers of the model chunk live in one
symmetric (peer-mapped) allocation together with a signal pad used for the
cross-rank ready/done flags.  All ranks of the DP group must share a node.

Replaces, for CUDA runs with dp > 1, the reference's per-parameter NCCL
all-reduce + full AdamW on every rank (parallel/data_parallel.py:5-15,
main.py:177) and its round-robin ZeRO-1 (parallel/distributed_optimizer.py).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..comm.symmetric import SymmetricBuffer
from ..ops import native
from .param_buffer import ParamBuffer


def replication_runs(offsets, kinds, numel, shards, max_segs):
    """Replication runs of each owned shard, in float4 units relative to the shard start.

    ``offsets[i]`` / ``kinds[i]``: flat start and kind of parameter i (in buffer order);
    kind 0 = GEMM weight (the kernels read its bf16 shadow: only that is all-gathered), kind 1 =
    LayerNorm / embedding / 1-D parameter (its kernels read fp32).  The padding after a
    parameter belongs to that parameter's run; adjacent runs of one kind merge.  Returns, per
    ``(lo, hi)`` in ``shards``, a list of ``[begin4, end4, kind, 0]`` covering ``[lo, hi)``, or
    None when it would need more than ``max_segs`` runs (the kernel then all-gathers every
    element in both precisions).
    """
    out = []
    for lo, hi in shards:
        runs = []
        for i, (off, kind) in enumerate(zip(offsets, kinds)):
            end = offsets[i + 1] if i + 1 < len(offsets) else numel
            a, z = max(off, lo), min(end, hi)
            if a >= z:
                continue
            if runs and runs[-1][2] == kind and runs[-1][1] == (a - lo) // 4:
                runs[-1][1] = (z - lo) // 4
            else:
                runs.append([(a - lo) // 4, (z - lo) // 4, kind, 0])
        out.append(runs if runs and len(runs) <= max_segs else None)
    return out


class FusedDPOptimizer(torch.optim.Optimizer):
    def __init__(self, module: torch.nn.Module, dp_group, lr=6e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                 bucket_elems=16 << 20, overlap=True, max_ctas=64, defer_done=False, tail_ctas=None):
        C = native()
        self.group = dp_group
        self.world = 1 if dp_group is None else dist.get_world_size(dp_group)
        self.rank = 0 if dp_group is None else dist.get_rank(dp_group)
        if self.world > 8:
            raise ValueError("the fused DP kernel supports up to 8 ranks (one NVSwitch node)")
        self.sig_bytes = (C.dp_signal_pad_bytes() + 4095) // 4096 * 4096
        self.symm = None

        def allocate(numel):
            total = self.sig_bytes + numel * (4 + 4 + 2)
            self.symm = SymmetricBuffer(total, dp_group)
            self._numel = numel
            data = self.symm.tensor(self.sig_bytes, numel, torch.float32)
            grad = self.symm.tensor(self.sig_bytes + 4 * numel, numel, torch.float32)
            pb = self.symm.tensor(self.sig_bytes + 8 * numel, numel, torch.bfloat16)
            return data, grad, pb

        self.buf = ParamBuffer(module.parameters(), align=self.world, bucket_elems=bucket_elems, allocator=allocate)
        if len(self.buf.buckets) > 256:
            raise ValueError("too many DP buckets for the signal pad; raise bucket size")
        super().__init__(list(self.buf.params), dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        n = self._numel
        self.ptr_param = [self.symm.peer_ptr(r, self.sig_bytes) for r in range(self.world)]
        self.ptr_grad = [self.symm.peer_ptr(r, self.sig_bytes + 4 * n) for r in range(self.world)]
        self.ptr_bf16 = [self.symm.peer_ptr(r, self.sig_bytes + 8 * n) for r in range(self.world)]
        self.ptr_sig = [self.symm.peer_ptr(r, 0) for r in range(self.world)]
        self.shards = [self.buf.shard_range(b, self.rank) for b in range(len(self.buf.buckets))]
        self.mom_off = []
        off = 0
        for lo, hi in self.shards:
            self.mom_off.append(off)
            off += hi - lo
        dev = self.buf.data.device
        self.exp_avg = torch.zeros(off, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(off, dtype=torch.float32, device=dev)
        self.counters = torch.zeros(len(self.buf.buckets), dtype=torch.int32, device=dev)
        self.segs = self._replication_runs(module)
        self._master_stale = False
        # state_dict() must see the current fp32 master of every shard
        self._sd_hook = module.register_state_dict_pre_hook(lambda *args, **kw: self.gather_master())
        self.stream = torch.cuda.Stream(device=dev)
        self.overlap = overlap
        self._default_overlap = overlap
        self.max_ctas = max_ctas
        # defer_done: bucket kernels publish "done" without waiting for the peers; one bounded wait for
        # every bucket runs at the end of the step (no cross-rank barrier between consecutive buckets).
        # Buckets launched after backward (nothing left to overlap with) get tail_ctas CTAs.
        self.defer_done = bool(defer_done)
        self.tail_ctas = tail_ctas if tail_ctas is not None else (
            4 * torch.cuda.get_device_properties(self.buf.data.device).multi_processor_count)
        self._step = 0
        self._epoch = 0
        self._bucket_of = {}
        for b, (_, _, params) in enumerate(self.buf.buckets):
            for p in params:
                self._bucket_of[id(p)] = b
        self._pending = []
        self._next = 0
        self._launched_step = False
        self._dev_epoch = self._dev_step = self._dev_hyper = self._lr_table = None
        # every rank's buffers hold the same initial values (same seed) -- make the bf16 shadow current
        self.buf.refresh_bf16()
        if self.world > 1:
            dist.barrier(group=dp_group)

    def _replication_runs(self, module):
        """Per bucket: int32 [nseg, 4] runs {begin4, end4, kind, 0} of this rank's owned range (or None)."""
        from .tensor_parallel import VocabParallelEmbedding
        fp32_ids = set()
        for m in module.modules():
            if isinstance(m, (torch.nn.LayerNorm, torch.nn.Embedding, VocabParallelEmbedding)):
                fp32_ids.update(id(p) for p in m.parameters(recurse=False))
        kinds = [1 if (id(p) in fp32_ids or p.dim() != 2) else 0 for p in self.buf.params]
        runs = replication_runs(self.buf.offsets, kinds, self.buf.numel, self.shards, native().dp_max_segments())
        return [None if r is None else torch.tensor(r, dtype=torch.int32).to(self.buf.data.device) for r in runs]

    @torch.no_grad()
    def gather_master(self):
        """Make this rank's fp32 master current everywhere (peer loads of the owners' shards).

        Stream-ordered after the last step on this rank; the owners cannot
        update their shards again before this rank starts its next step.
        """
        if self.world == 1 or not self._master_stale:
            return
        torch.cuda.current_stream().wait_stream(self.stream)
        C = native()
        for (lo, hi, _) in self.buf.buckets:
            C.dp_gather_master(self.ptr_param, self.rank, lo, hi)
        self._master_stale = False

    @property
    def state_is_sharded(self):
        """Each DP rank holds only its own slice of the moments (checkpoints write one file per DP rank)."""
        return self.world > 1

    # ----------------------------------------------------------- GradSync interface
    @property
    def active(self):
        return True

    def reset(self):
        """Start a new optimizer step: new epoch for the cross-rank flags."""
        self._pending = [len(params) for (_, _, params) in self.buf.buckets]
        self._next = 0
        self._launched_step = False

    def attach(self, modules):
        self.attached_params = getattr(self, "attached_params", set())
        for m in modules:
            params = [p for p in m.parameters() if id(p) in self._bucket_of]
            self.attached_params.update(id(p) for p in params)
            hooks = list(getattr(m, "_mmb_grad_ready_hooks", ()))
            hooks.append(lambda ps=params: self.mark_ready(ps))
            m._mmb_grad_ready_hooks = hooks

    def mark_ready(self, params):
        if not self.overlap:
            return
        for p in params:
            b = self._bucket_of.get(id(p))
            if b is not None:
                self._pending[b] -= 1
        while self._next < len(self._pending) and self._pending[self._next] <= 0:
            self._launch(self._next)
            self._next += 1

    def _begin(self):
        if not self._launched_step:
            self._launched_step = True
            self._step += 1
            self._epoch += 1

    def enable_device_schedule(self, lr_table: torch.Tensor):
        """Keep the flag epoch, the step count and lr on the device, so a captured step replays correctly.

        At the first bucket of each step a one-thread kernel advances the epoch
        and another derives lr and the bias corrections from the step counter
        (``lr_table[step - 1]``); the bucket kernels read them from memory.
        """
        dev = self.buf.data.device
        self._dev_epoch = torch.tensor([self._epoch], dtype=torch.int32, device=dev)
        self._dev_step = torch.tensor([self._step], dtype=torch.int32, device=dev)
        self._dev_hyper = torch.zeros(4, dtype=torch.float32, device=dev)
        self._lr_table = lr_table.to(device=dev, dtype=torch.float32).contiguous()

    def advance_host_counters(self):
        """Host-side bookkeeping of one replayed step (the replay itself advances the device counters)."""
        self._step += 1
        self._epoch += 1
        self._master_stale = True

    def _launch(self, b, tail=False):
        first = not self._launched_step
        self._begin()
        C = native()
        g = self.param_groups[0]
        lo, hi = self.shards[b]
        n = hi - lo
        off = self.mom_off[b]
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream())
        self.stream.wait_event(ev)
        with torch.cuda.stream(self.stream):
            if first and self._dev_epoch is not None:
                C.dp_epoch_step(self._dev_epoch)
                C.adamw_hyper_step(self._dev_step, self._lr_table, g["betas"][0], g["betas"][1], self._dev_hyper)
            C.dp_rs_adamw_ag(self.ptr_param, self.ptr_grad, self.ptr_bf16, self.ptr_sig, self.rank, b, self._epoch,
                             lo, hi, self.exp_avg[off:off + n], self.exp_avg_sq[off:off + n], self.counters[b:b + 1],
                             g["lr"], g["betas"][0], g["betas"][1], g["eps"], g["weight_decay"], self._step,
                             1.0 / self.world, self.tail_ctas if tail else self.max_ctas, int(self.defer_done),
                             self._dev_epoch, self._dev_hyper, self.segs[b])
        self._master_stale = True

    def finish(self):
        """Launch the buckets not yet issued (in order), then (deferred mode) the wait for every rank's "done"."""
        while self._next < len(self.buf.buckets):
            self._launch(self._next, tail=True)
            self._next += 1
        if self.defer_done and self._launched_step:
            with torch.cuda.stream(self.stream):
                native().dp_wait_done(self.ptr_sig[self.rank], len(self.buf.buckets), self.world, self._epoch,
                                      self._dev_epoch)

    # ----------------------------------------------------------- optimizer interface
    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        self.finish()
        torch.cuda.current_stream().wait_stream(self.stream)
        self.overlap = self._default_overlap
        return loss

    def zero_grad(self, set_to_none: bool = False):
        self.buf.zero_grad()

    def state_dict(self):
        return {"step": self._step, "epoch": self._epoch, "dp_rank": self.rank, "dp_size": self.world,
                "shards": list(self.shards), "exp_avg": self.exp_avg.clone(), "exp_avg_sq": self.exp_avg_sq.clone(),
                "param_groups": [{k: v for k, v in g.items() if k != "params"} for g in self.param_groups]}

    def load_state_dict(self, sd):
        if sd["dp_size"] != self.world or list(map(tuple, sd["shards"])) != list(map(tuple, self.shards)):
            raise ValueError("fused-DP state was saved with a different DP layout")
        self._step = int(sd["step"])
        self._epoch = int(sd.get("epoch", self._epoch))
        if self._dev_step is not None:
            self._dev_step.fill_(self._step)
            self._dev_epoch.fill_(self._epoch)
        self.exp_avg.copy_(sd["exp_avg"])
        self.exp_avg_sq.copy_(sd["exp_avg_sq"])
        # a model state loaded with it holds the full fp32 master on every rank
        self._master_stale = False
        for g, s in zip(self.param_groups, sd["param_groups"]):
            g.update(s)
        self.buf.refresh_bf16()

    def close(self):
        if getattr(self, "_sd_hook", None) is not None:
            self._sd_hook.remove()
            self._sd_hook = None
        if self.symm is not None:
            torch.cuda.synchronize()
            if self.world > 1:
                dist.barrier(group=self.group)
            self.symm.close()
            self.symm = None
