"""Masked mean cross-entropy, vocabulary-parallel when the logits are sharded.

Reference: model/loss.py:4-16 computes ``sum(CE * mask) / sum(mask)`` on the
full-vocabulary logits (which its TP path all-gathers first).  Here the
logits may be this rank's vocabulary shard: the softmax statistics are
combined with three all-reduces of per-token scalars (max, sum-exp, target
logit) instead of gathering ``[tokens, V]``.  Columns at or beyond the real
vocabulary size (padding) are excluded.  Labels equal to -100 contribute
zero loss (the ``F.cross_entropy`` default) but stay in the denominator, as
in the reference.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from ..parallel import process_groups as pg


class _VocabParallelCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, labels, vocab_start, n_valid, group):
        x = logits.float()
        V_local = x.size(-1)
        if n_valid < V_local:
            x = x.clone()
            x[:, n_valid:] = float("-inf")
        mx = x.max(dim=-1).values
        world = 1 if group is None else dist.get_world_size(group)
        if world > 1:
            dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=group)
        ex = torch.exp(x - mx.unsqueeze(-1))
        se = ex.sum(dim=-1)
        local = labels - vocab_start
        inside = (local >= 0) & (local < n_valid)
        idx = local.clamp(0, V_local - 1)
        tgt = torch.where(inside, x.gather(-1, idx.unsqueeze(-1)).squeeze(-1), torch.zeros_like(mx))
        if world > 1:
            dist.all_reduce(se, group=group)
            dist.all_reduce(tgt, group=group)
        lse = mx + torch.log(se)
        valid = labels != -100
        loss = torch.where(valid, lse - tgt, torch.zeros_like(lse))
        ctx.save_for_backward(ex, se, idx, inside, valid)
        ctx.dtype = logits.dtype
        return loss

    @staticmethod
    def backward(ctx, dloss):
        ex, se, idx, inside, valid = ctx.saved_tensors
        grad = ex / se.unsqueeze(-1)
        grad.scatter_add_(-1, idx.unsqueeze(-1), -inside.to(grad.dtype).unsqueeze(-1))
        grad = grad * (dloss * valid).unsqueeze(-1)
        return grad.to(ctx.dtype), None, None, None, None


def vocab_parallel_cross_entropy(logits, labels, vocab_start=0, n_valid=None, group=None):
    """Per-token CE over a (possibly sharded, possibly padded) vocabulary."""
    n_valid = logits.size(-1) if n_valid is None else n_valid
    return _VocabParallelCE.apply(logits, labels, vocab_start, n_valid, group)


class CrossEntropyLoss(nn.Module):
    """``sum(CE * mask) / sum(mask)``; ``vocab_size`` marks padded columns."""

    def __init__(self, vocab_size=None, vocab_parallel=None):
        super().__init__()
        self.vocab_size = vocab_size
        self.vocab_parallel = vocab_parallel

    def forward(self, logits, labels, loss_mask):
        V_local = logits.size(-1)
        logits = logits.reshape(-1, V_local)
        labels = labels.reshape(-1)
        loss_mask = loss_mask.reshape(-1).to(torch.float32)
        group = pg.tp_group()
        world = 1 if group is None else dist.get_world_size(group)
        sharded = self.vocab_parallel
        if sharded is None:
            sharded = world > 1 and (self.vocab_size is None or V_local < self.vocab_size)
        if not sharded:
            group, world = None, 1
        full_vocab = self.vocab_size if self.vocab_size is not None else V_local * world
        if world == 1 and full_vocab >= V_local:
            loss = F.cross_entropy(logits.float(), labels, reduction="none")
        else:
            start = pg.tp_rank() * V_local if world > 1 else 0
            n_valid = max(0, min(V_local, full_vocab - start))
            loss = vocab_parallel_cross_entropy(logits, labels, start, n_valid, group)
        return torch.sum(loss * loss_mask) / loss_mask.sum()
