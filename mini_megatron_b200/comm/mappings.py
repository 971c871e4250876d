"""Autograd-aware tensor-parallel collectives (the f / g operators of Megatron).

Semantics follow the reference's comm/all_reduce.py:5-86:

* ``copy_to_model_parallel_region``     forward identity, backward all-reduce
* ``reduce_from_model_parallel_region`` forward all-reduce, backward identity
* ``gather_from_model_parallel_region`` forward all-gather(dim), backward narrow
* ``scatter_to_model_parallel_region``  forward narrow(dim), backward all-gather

A ``None`` group (or a group of one) makes every operator the identity, which
is how single-GPU and CPU unit tests run.  These are the NCCL/gloo path; the
fused NVLink kernels in :mod:`mini_megatron_b200.ops.fused_tp` implement the
same contracts inside GEMM kernels.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def _world(group) -> int:
    return 1 if group is None else dist.get_world_size(group=group)


def all_gather_dim(tensor: torch.Tensor, group, dim: int) -> torch.Tensor:
    world = _world(group)
    if world == 1:
        return tensor
    dim = dim % tensor.dim()
    tensor = tensor.contiguous()
    if dim == 0:
        out = torch.empty((world * tensor.size(0),) + tuple(tensor.shape[1:]), dtype=tensor.dtype,
                          device=tensor.device)
        dist.all_gather_into_tensor(out, tensor, group=group)
        return out
    pieces = [torch.empty_like(tensor) for _ in range(world)]
    dist.all_gather(pieces, tensor, group=group)
    return torch.cat(pieces, dim=dim)


def reduce_scatter_dim(tensor: torch.Tensor, group, dim: int) -> torch.Tensor:
    world = _world(group)
    if world == 1:
        return tensor
    dim = dim % tensor.dim()
    if tensor.size(dim) % world:
        raise ValueError(f"dim {dim} of size {tensor.size(dim)} is not divisible by {world}")
    if dim == 0:
        tensor = tensor.contiguous()
        out = torch.empty((tensor.size(0) // world,) + tuple(tensor.shape[1:]), dtype=tensor.dtype,
                          device=tensor.device)
        dist.reduce_scatter_tensor(out, tensor, group=group)
        return out
    chunks = [c.contiguous() for c in tensor.chunk(world, dim=dim)]
    out = torch.empty_like(chunks[0])
    dist.reduce_scatter(out, chunks, group=group)
    return out


class ReduceFromModelParallelRegion(torch.autograd.Function):
    """Sum the TP partial outputs in forward; gradient passes through."""

    @staticmethod
    def forward(ctx, tensor, group):
        output = tensor.clone()
        if _world(group) > 1:
            dist.all_reduce(output, group=group)
        return output

    @staticmethod
    def backward(ctx, grad_output):
        return grad_output, None


class CopyToModelParallelRegion(torch.autograd.Function):
    """Identity in forward; all-reduce of the input gradient in backward."""

    @staticmethod
    def forward(ctx, tensor, group):
        ctx.group = group
        return tensor

    @staticmethod
    def backward(ctx, grad_output):
        if _world(ctx.group) > 1:
            grad_output = grad_output.contiguous().clone()
            dist.all_reduce(grad_output, group=ctx.group)
        return grad_output, None


class GatherFromModelParallelRegion(torch.autograd.Function):
    """All-gather equal shards along ``dim``; backward keeps the local slice."""

    @staticmethod
    def forward(ctx, tensor, group, dim):
        ctx.group, ctx.dim, ctx.local = group, dim, tensor.size(dim)
        return all_gather_dim(tensor, group, dim)

    @staticmethod
    def backward(ctx, grad_output):
        if _world(ctx.group) == 1:
            return grad_output, None, None
        r = dist.get_rank(group=ctx.group)
        return grad_output.narrow(ctx.dim, r * ctx.local, ctx.local).contiguous(), None, None


class ScatterToModelParallelRegion(torch.autograd.Function):
    """Keep this rank's slice along ``dim``; backward all-gathers."""

    @staticmethod
    def forward(ctx, tensor, group, dim):
        ctx.group, ctx.dim = group, dim
        world = _world(group)
        if world == 1:
            return tensor
        local = tensor.size(dim) // world
        r = dist.get_rank(group=group)
        return tensor.narrow(dim, r * local, local).contiguous()

    @staticmethod
    def backward(ctx, grad_output):
        return all_gather_dim(grad_output, ctx.group, ctx.dim), None, None


def reduce_from_model_parallel_region(tensor, group):
    return ReduceFromModelParallelRegion.apply(tensor, group)


def copy_to_model_parallel_region(tensor, group):
    return CopyToModelParallelRegion.apply(tensor, group)


def gather_from_model_parallel_region(tensor, group, dim=-1):
    return GatherFromModelParallelRegion.apply(tensor, group, dim)


def scatter_to_model_parallel_region(tensor, group, dim=-1):
    return ScatterToModelParallelRegion.apply(tensor, group, dim)


# Reference-compatible aliases (comm/all_reduce.py:82-86).
AllReduce = ReduceFromModelParallelRegion


def all_reduce(tensor, group):
    return reduce_from_model_parallel_region(tensor, group)
