"""Causal self-attention on the fused QKV activation.

``qkv`` is the ``[B*S, 3*Hl]`` bf16 output of the QKV GEMM whose columns are
``[Q heads | K heads | V heads]`` (each ``nh*d`` wide) -- exactly the layout
the reference reshapes to ``[B, S, 3, nh, d]`` (model/transformer.py:27-33).
Outputs are ``ctx [B*S, nh*d]`` bf16 (token-major, ready for the O GEMM) and
``lse [B, nh, S]`` fp32 for the backward.  ``flash_attn_bwd`` returns
``dqkv`` in the same packed layout as ``qkv``.
"""
from __future__ import annotations

import torch

from . import native


def _views(qkv, B, S, nh, d):
    t = qkv.view(B, S, 3, nh, d)
    return t[:, :, 0].transpose(1, 2), t[:, :, 1].transpose(1, 2), t[:, :, 2].transpose(1, 2)


def flash_attn_fwd(qkv, B, S, nh, d):
    C = native()
    if hasattr(C, "flash_attn_fwd"):
        return C.flash_attn_fwd(qkv, B, S, nh, d)
    # Interim path until the tcgen05 attention kernel lands: aten flash kernel.
    q, k, v = _views(qkv, B, S, nh, d)
    out, lse = torch.ops.aten._scaled_dot_product_flash_attention(q, k, v, 0.0, True, False)[:2]
    return out.transpose(1, 2).reshape(B * S, nh * d), lse


def flash_attn_bwd(dctx, qkv, ctx, lse, B, S, nh, d):
    C = native()
    if hasattr(C, "flash_attn_bwd"):
        return C.flash_attn_bwd(dctx, qkv, ctx, lse, B, S, nh, d)
    # Interim path: recompute the forward under autograd and differentiate it.
    with torch.enable_grad():
        q2 = qkv.detach().requires_grad_(True)
        q, k, v = _views(q2, B, S, nh, d)
        out = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
        (dqkv,) = torch.autograd.grad(out, (q2,), dctx.view(B, S, nh, d).transpose(1, 2))
    return dqkv.reshape(B * S, 3 * nh * d)
