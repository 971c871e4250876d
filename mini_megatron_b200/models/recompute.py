"""Activation recomputation (reference model/recompute.py:4-6).

On CPU this is torch.utils.checkpoint around the layer body; on CUDA the
native DecoderLayer Function re-runs its own forward inside backward when
``layer.recompute`` is set (only the layer input is kept).
"""
import torch
import torch.utils.checkpoint


def checkpoint(layer, x):
    if x.is_cuda and hasattr(layer, "native_forward"):
        return layer.native_forward(x, recompute=True)
    return torch.utils.checkpoint.checkpoint(layer._forward, x, use_reentrant=False)
