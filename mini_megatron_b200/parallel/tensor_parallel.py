"""Tensor-parallel layers: ColumnParallelLinear, RowParallelLinear, VocabParallelEmbedding.

Shapes and initialisation follow the reference (parallel/tensor_parallel.py:13-105):
weights are N(0, 0.02), Column shards the output dimension (``[out/tp, in]``),
Row shards the input dimension (``[out, in/tp]``), the vocabulary embedding
shards rows (``[V/tp, H]``).  Additions:

* sequence parallelism (``sequence_parallel=True``): Column all-gathers its
  sequence-sharded input and reduce-scatters its input gradient; Row
  reduce-scatters its output instead of all-reducing it;
* vocabulary padding (``padded_vocab_size``) so an odd vocabulary (50257)
  shards over any TP size and keeps 16-byte-aligned rows for TMA;
* a native path on CUDA tensors: bf16 GEMMs on the tcgen05 kernel, fp32
  weight gradients accumulated straight into ``param.main_grad``.

On CPU the modules run plain PyTorch (the oracle for tests).
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..comm import mappings as mp
from ..comm import sequence_parallel as spc
from . import process_groups as pg
from .param_buffer import bf16_weight, grad_target


def _normal_init(tensor, std=0.02):
    nn.init.normal_(tensor, std=std)


def strided_partition_rows(tensor, world_size, rank, stride=1):
    """One TP row shard using the stride convention of the reference.

    ``stride=1`` is a contiguous split of the rows.  For the fused QKV weight
    (logical rows ``[all Q | all K | all V]``) ``stride=3`` hands every rank an
    equal set of Q, K and V heads: the rows are cut into ``world_size*stride``
    chunks and rank ``r`` takes chunks ``r, r+world, r+2*world``
    (parallel/tensor_parallel.py:13-31).
    """
    n_chunks = world_size * stride
    ok = (tensor.dim() >= 1 and world_size >= 1 and 0 <= rank < world_size and stride >= 1
          and tensor.size(0) % n_chunks == 0)
    if not ok:
        raise ValueError(f"cannot take TP shard {rank} of {world_size} (stride {stride}) from a tensor of shape "
                         f"{tuple(tensor.shape)}: need a leading dimension that splits into world_size * stride "
                         "equal chunks and 0 <= rank < world_size")
    chunk = tensor.size(0) // n_chunks
    pieces = [tensor.narrow(0, (s * world_size + rank) * chunk, chunk) for s in range(stride)]
    return torch.cat(pieces, dim=0)


def strided_gather_rows(shards, stride=1):
    """Inverse of :func:`strided_partition_rows` given every rank's shard (rank order)."""
    world = len(shards)
    chunk = shards[0].size(0) // stride
    pieces = []
    for s in range(stride):
        for r in range(world):
            pieces.append(shards[r].narrow(0, s * chunk, chunk))
    return torch.cat(pieces, dim=0)


def pad_vocab_size(vocab_size: int, tp_size: int = 1, multiple: int = 128) -> int:
    """Smallest size >= vocab_size divisible by ``multiple * tp_size``."""
    m = multiple * max(1, tp_size)
    return (vocab_size + m - 1) // m * m


# ---------------------------------------------------------------------------
# native autograd functions (CUDA only)
# ---------------------------------------------------------------------------
class _ColumnLinearFn(torch.autograd.Function):
    """y = x W^T on this rank's output shard; dgrad all-reduced (or RS under SP)."""

    @staticmethod
    def forward(ctx, x, weight, group, sp, gather_output):
        from ..ops.linear import linear_fwd
        xb = x.to(torch.bfloat16)
        if sp:
            xb = spc.sp_all_gather(xb.contiguous(), group=group)
        full_shape = xb.shape
        x2 = xb.reshape(-1, full_shape[-1]).contiguous()
        y = linear_fwd(x2, bf16_weight(weight)).view(full_shape[:-1] + (weight.shape[0],))
        ctx.save_for_backward(x2)
        ctx.weight, ctx.group, ctx.sp, ctx.gather_output = weight, group, sp, gather_output
        ctx.in_shape, ctx.full_shape, ctx.in_dtype = x.shape, full_shape, x.dtype
        if gather_output:
            y = mp.all_gather_dim(y, group, -1)
        return y

    @staticmethod
    def backward(ctx, dy):
        from ..ops.linear import linear_dgrad, linear_wgrad
        (x2,) = ctx.saved_tensors
        w = ctx.weight
        if ctx.gather_output and pg_world(ctx.group) > 1:
            r = torch.distributed.get_rank(group=ctx.group)
            n = w.shape[0]
            dy = dy.narrow(-1, r * n, n)
        dy2 = dy.reshape(-1, dy.shape[-1]).to(torch.bfloat16).contiguous()
        if w.requires_grad:
            linear_wgrad(dy2, x2, grad_target(w))
        dx = linear_dgrad(dy2, bf16_weight(w))
        if ctx.sp:
            dx = spc.sp_reduce_scatter(dx.view(ctx.full_shape), group=ctx.group)
        elif pg_world(ctx.group) > 1:
            torch.distributed.all_reduce(dx, group=ctx.group)
        return dx.reshape(ctx.in_shape).to(ctx.in_dtype), None, None, None, None


class _RowLinearFn(torch.autograd.Function):
    """y = sum_ranks x_r W_r^T (all-reduce, or reduce-scatter under SP)."""

    @staticmethod
    def forward(ctx, x, weight, group, sp):
        from ..ops.linear import linear_fwd
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        y = linear_fwd(x2, bf16_weight(weight))
        y = y.view(shape[:-1] + (y.shape[-1],))
        if sp:
            y = spc.sp_reduce_scatter(y, group=group)
        elif pg_world(group) > 1:
            torch.distributed.all_reduce(y, group=group)
        ctx.save_for_backward(x2)
        ctx.weight, ctx.group, ctx.sp, ctx.in_shape, ctx.in_dtype = weight, group, sp, shape, x.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        from ..ops.linear import linear_dgrad, linear_wgrad
        (x2,) = ctx.saved_tensors
        w = ctx.weight
        if ctx.sp:
            dy = spc.sp_all_gather(dy.contiguous(), group=ctx.group)
        dy2 = dy.reshape(-1, dy.shape[-1]).to(torch.bfloat16).contiguous()
        if w.requires_grad:
            linear_wgrad(dy2, x2, grad_target(w))
        dx = linear_dgrad(dy2, bf16_weight(w))
        return dx.reshape(ctx.in_shape).to(ctx.in_dtype), None, None, None


def pg_world(group) -> int:
    return 1 if group is None else torch.distributed.get_world_size(group=group)


# ---------------------------------------------------------------------------
# modules
# ---------------------------------------------------------------------------
class ColumnParallelLinear(nn.Module):
    """Linear layer with the output dimension split across TP ranks."""

    def __init__(self, in_features, out_features, bias=False, stride=1, gather_output=False,
                 sequence_parallel=None):
        super().__init__()
        tp = pg.tp_size()
        if out_features % (tp * stride):
            raise ValueError("out_features must divide evenly by TP size * stride")
        self.in_features = in_features
        self.out_features = out_features
        self.out_features_per_partition = out_features // tp
        self.stride = stride
        self.gather_output = gather_output
        self.sequence_parallel = pg.sequence_parallel_enabled() if sequence_parallel is None else sequence_parallel
        self.weight = nn.Parameter(torch.empty(self.out_features_per_partition, in_features))
        _normal_init(self.weight)
        if bias:
            self.bias = nn.Parameter(torch.zeros(self.out_features_per_partition))
        else:
            self.bias = None

    def forward(self, x):
        group = pg.tp_group()
        sp = self.sequence_parallel and pg_world(group) > 1
        if x.is_cuda and self.bias is None:
            return _ColumnLinearFn.apply(x, self.weight, group, sp, self.gather_output)
        if sp:
            x = spc.gather_from_sequence_parallel_region(x, group)
        else:
            x = mp.copy_to_model_parallel_region(x, group)
        out = F.linear(x, self.weight, self.bias)
        return mp.gather_from_model_parallel_region(out, group) if self.gather_output else out


class RowParallelLinear(nn.Module):
    """Linear layer with the input dimension split across TP ranks."""

    def __init__(self, in_features, out_features, bias=False, input_is_parallel=True, sequence_parallel=None):
        super().__init__()
        tp = pg.tp_size()
        if in_features % tp:
            raise ValueError("in_features must divide evenly by TP size")
        self.in_features = in_features
        self.out_features = out_features
        self.in_features_per_partition = in_features // tp
        self.input_is_parallel = input_is_parallel
        self.sequence_parallel = pg.sequence_parallel_enabled() if sequence_parallel is None else sequence_parallel
        self.weight = nn.Parameter(torch.empty(out_features, self.in_features_per_partition))
        _normal_init(self.weight)
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features))
        else:
            self.bias = None

    def forward(self, x):
        group = pg.tp_group()
        sp = self.sequence_parallel and pg_world(group) > 1
        if not self.input_is_parallel:
            x = mp.scatter_to_model_parallel_region(x, group, -1)
        if x.is_cuda and self.bias is None:
            return _RowLinearFn.apply(x, self.weight, group, sp)
        out = F.linear(x, self.weight)
        out = spc.sp_all_reduce(out, group) if sp else mp.reduce_from_model_parallel_region(out, group)
        if self.bias is not None:
            out = out + self.bias
        return out


class _VocabEmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, weight, vstart, vend, group):
        from ..ops import native
        ids_c = ids.contiguous()
        out = torch.empty(ids.shape + (weight.shape[1],), device=ids.device, dtype=torch.float32)
        native().embedding_fwd(ids_c.view(-1), weight.detach(), None, out.view(-1, weight.shape[1]), 1, vstart, vend)
        if pg_world(group) > 1:
            torch.distributed.all_reduce(out, group=group)
        ctx.save_for_backward(ids_c)
        ctx.weight, ctx.vstart, ctx.vend = weight, vstart, vend
        return out

    @staticmethod
    def backward(ctx, dout):
        from ..ops import native
        (ids,) = ctx.saved_tensors
        w = ctx.weight
        if w.requires_grad:
            native().embedding_bwd(ids.view(-1), dout.contiguous().float().view(-1, w.shape[1]), grad_target(w),
                                   None, 1, ids.numel(), ctx.vstart, ctx.vend)
        return None, None, None, None, None


class VocabParallelEmbedding(nn.Module):
    """Vocabulary-row sharded embedding with a replicated (summed) output."""

    def __init__(self, num_embeddings, embedding_dim, padded_num_embeddings=None):
        super().__init__()
        self.tp_size = pg.tp_size()
        self.tp_rank = pg.tp_rank()
        padded = padded_num_embeddings or num_embeddings
        if padded % self.tp_size:
            raise ValueError("vocabulary size must divide evenly by TP size (pad it)")
        self.num_embeddings = num_embeddings
        self.num_embeddings_per_partition = padded // self.tp_size
        self.vocab_start_index = self.tp_rank * self.num_embeddings_per_partition
        self.vocab_end_index = self.vocab_start_index + self.num_embeddings_per_partition
        self.weight = nn.Parameter(torch.empty(self.num_embeddings_per_partition, embedding_dim))
        _normal_init(self.weight)
        if padded > num_embeddings:
            # rows past the real vocabulary are never looked up; keep them zero
            with torch.no_grad():
                lo = max(0, num_embeddings - self.vocab_start_index)
                self.weight[lo:].zero_()

    def forward(self, input_ids):
        group = pg.tp_group()
        if input_ids.is_cuda:
            return _VocabEmbeddingFn.apply(input_ids, self.weight, self.vocab_start_index, self.vocab_end_index,
                                           group)
        outside = (input_ids < self.vocab_start_index) | (input_ids >= self.vocab_end_index)
        local_ids = (input_ids - self.vocab_start_index).masked_fill(outside, 0)
        output = F.embedding(local_ids, self.weight).masked_fill(outside.unsqueeze(-1), 0)
        return mp.reduce_from_model_parallel_region(output, group)
