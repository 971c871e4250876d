"""Blocking point-to-point helpers (reference comm/send_recv.py:5-21)."""
import torch
import torch.distributed as dist


def send(tensor, dst, tag=0, group=None):
    dist.send(tensor.contiguous(), dst=dst, tag=tag, group=group)


def recv(tensor, src, tag=0, group=None):
    dist.recv(tensor, src=src, tag=tag, group=group)


def send_recv(tensor, dst, src, group=None, tag=0):
    """Move ``tensor`` from global rank ``src`` to ``dst``; other ranks get a copy back."""
    if dst == src:
        return tensor
    me = dist.get_rank()
    if me == dst:
        result = torch.empty_like(tensor)
        dist.recv(result, src=src, tag=tag, group=group)
        return result
    if me == src:
        dist.send(tensor.contiguous(), dst=dst, tag=tag, group=group)
    return tensor.clone()
