"""(dp, pp, tp) process-group topology.

Rank layout (same as the reference, parallel/process_groups.py:3-47)::

    rank = dp_rank * (tp * pp) + pp_rank * tp + tp_rank

so a tensor-parallel group is a contiguous block of ``tp`` ranks (one NVSwitch
hop apart on a node, which is where the fused TP kernels want them), a
pipeline group strides by ``tp`` and a data-parallel group strides by
``tp * pp``.  Every rank calls ``dist.new_group`` for every group, in the
same order, as torch.distributed requires.  Groups of size 1 are ``None``.

The returned dict keeps the reference's keys (``tp_rank``, ``pp_rank``,
``dp_rank``, ``tp_size``, ``pp_size``, ``dp_size``, ``tp_group``,
``pp_group``, ``dp_group``) and adds the global rank lists of this rank's
groups plus the sequence-parallel switch.
"""
from __future__ import annotations

import torch.distributed as dist

_MPU = None


def rank_coords(rank: int, tp_size: int, pp_size: int):
    """(tp_rank, pp_rank, dp_rank) of a global rank."""
    return rank % tp_size, (rank // tp_size) % pp_size, rank // (tp_size * pp_size)


def init_model_parallel(tp_size: int = 1, pp_size: int = 1, sequence_parallel: bool = False):
    """Build the topology dict for the current process group.

    Mirrors parallel/process_groups.py:3-47 of the reference; additionally
    validates that ``tp * pp`` divides the world and records the ranks of
    each of this rank's groups (``tp_ranks``, ``pp_ranks``, ``dp_ranks``).
    """
    world_size = dist.get_world_size()
    if tp_size < 1 or pp_size < 1 or world_size % (tp_size * pp_size):
        raise ValueError(f"world size {world_size} is not divisible by tp*pp = {tp_size * pp_size}")
    if sequence_parallel and tp_size == 1:
        sequence_parallel = False
    dp_size = world_size // (tp_size * pp_size)
    rank = dist.get_rank()
    tp_rank, pp_rank, dp_rank = rank_coords(rank, tp_size, pp_size)

    tp_group = pp_group = dp_group = None
    tp_ranks = [rank]
    pp_ranks = [rank]
    dp_ranks = [rank]

    if tp_size > 1:
        for i in range(pp_size * dp_size):
            ranks = list(range(i * tp_size, (i + 1) * tp_size))
            group = dist.new_group(ranks=ranks)
            if rank in ranks:
                tp_group, tp_ranks = group, ranks
    if pp_size > 1:
        for i in range(tp_size * dp_size):
            # i enumerates (dp, tp) pairs; the stage ranks stride by tp.
            base = (i // tp_size) * tp_size * pp_size + i % tp_size
            ranks = [base + j * tp_size for j in range(pp_size)]
            group = dist.new_group(ranks=ranks)
            if rank in ranks:
                pp_group, pp_ranks = group, ranks
    if dp_size > 1:
        for i in range(tp_size * pp_size):
            ranks = [i + j * (tp_size * pp_size) for j in range(dp_size)]
            group = dist.new_group(ranks=ranks)
            if rank in ranks:
                dp_group, dp_ranks = group, ranks

    return {
        "rank": rank,
        "world_size": world_size,
        "tp_rank": tp_rank,
        "pp_rank": pp_rank,
        "dp_rank": dp_rank,
        "tp_size": tp_size,
        "pp_size": pp_size,
        "dp_size": dp_size,
        "tp_group": tp_group,
        "pp_group": pp_group,
        "dp_group": dp_group,
        "tp_ranks": tp_ranks,
        "pp_ranks": pp_ranks,
        "dp_ranks": dp_ranks,
        "sequence_parallel": bool(sequence_parallel),
    }


def set_model_parallel(mpu):
    global _MPU
    _MPU = mpu


def get_model_parallel():
    return _MPU


def tp_size() -> int:
    return _MPU["tp_size"] if _MPU else 1


def tp_rank() -> int:
    return _MPU["tp_rank"] if _MPU else 0


def tp_group():
    return _MPU["tp_group"] if _MPU else None


def sequence_parallel_enabled() -> bool:
    return bool(_MPU and _MPU.get("sequence_parallel", False) and _MPU["tp_size"] > 1)


def pp_peers():
    """(prev_rank, next_rank) global ranks of this stage's neighbours (None at the ends)."""
    if not _MPU or _MPU["pp_size"] == 1:
        return None, None
    ranks, r = _MPU["pp_ranks"], _MPU["pp_rank"]
    return (ranks[r - 1] if r > 0 else None), (ranks[r + 1] if r + 1 < len(ranks) else None)
