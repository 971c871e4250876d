"""Megatron-style sequence parallelism collectives (wired, unlike the reference).

Activations outside the tensor-parallel GEMMs (LayerNorm, residual, dropout
sites) are sharded along the sequence dimension inside the TP group.  The
model keeps ``[B, S, H]`` layout, so the sequence dimension is ``-2``.

* ``GatherFromSequenceParallelRegion``    forward all-gather(seq), backward reduce-scatter(seq)
  (before a ColumnParallel GEMM)
* ``ReduceScatterToSequenceParallelRegion`` forward reduce-scatter(seq), backward all-gather(seq)
  (after a RowParallel GEMM, replacing its all-reduce)

Reference: comm/sequence_parallel.py:8-61.  Differences: the group argument is
honoured (the reference's ``sp_all_reduce`` re-reads the global group), and
non-leading-dim chunks are made contiguous before the collective (the
reference passes strided chunks to ``reduce_scatter`` when B > 1).
"""
from __future__ import annotations

import torch

from .mappings import _world, all_gather_dim, reduce_scatter_dim
from ..parallel import process_groups as pg

SEQ_DIM = -2


def _default_group(group):
    return pg.tp_group() if group is None else group


def sp_all_gather(tensor, dim=SEQ_DIM, group=None):
    """All-gather TP shards along the sequence dimension (no autograd)."""
    return all_gather_dim(tensor, _default_group(group), dim)


def sp_reduce_scatter(tensor, dim=SEQ_DIM, group=None):
    """Reduce-scatter along the sequence dimension (no autograd)."""
    return reduce_scatter_dim(tensor, _default_group(group), dim)


class GatherFromSequenceParallelRegion(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tensor, group, seq_dim):
        ctx.group, ctx.seq_dim = group, seq_dim
        return all_gather_dim(tensor, group, seq_dim)

    @staticmethod
    def backward(ctx, grad_output):
        return reduce_scatter_dim(grad_output, ctx.group, ctx.seq_dim), None, None


class ReduceScatterToSequenceParallelRegion(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tensor, group, seq_dim):
        ctx.group, ctx.seq_dim = group, seq_dim
        return reduce_scatter_dim(tensor, group, seq_dim)

    @staticmethod
    def backward(ctx, grad_output):
        return all_gather_dim(grad_output, ctx.group, ctx.seq_dim), None, None


def gather_from_sequence_parallel_region(tensor, group=None, seq_dim=SEQ_DIM):
    group = _default_group(group)
    if _world(group) == 1:
        return tensor
    return GatherFromSequenceParallelRegion.apply(tensor, group, seq_dim)


def reduce_scatter_to_sequence_parallel_region(tensor, group=None, seq_dim=SEQ_DIM):
    group = _default_group(group)
    if _world(group) == 1:
        return tensor
    return ReduceScatterToSequenceParallelRegion.apply(tensor, group, seq_dim)


def sp_all_reduce(tensor, group=None, seq_dim=SEQ_DIM):
    """SP replacement of the Row-parallel all-reduce: RS forward, AG backward."""
    return reduce_scatter_to_sequence_parallel_region(tensor, group, seq_dim)


def sp_all_gather_qkv(qkv, dim=SEQ_DIM, group=None):
    """Keep local Q, all-gather K and V along the sequence (comm/sequence_parallel.py:56-61)."""
    q, k, v = qkv
    return q, sp_all_gather(k, dim, group), sp_all_gather(v, dim, group)


def scatter_to_sequence_parallel_region(tensor, group=None, seq_dim=SEQ_DIM):
    """Take this rank's sequence shard of a replicated tensor (used after the embedding)."""
    from .mappings import scatter_to_model_parallel_region
    group = _default_group(group)
    if _world(group) == 1:
        return tensor
    return scatter_to_model_parallel_region(tensor, group, seq_dim)
