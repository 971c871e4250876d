"""Causal self-attention on the fused QKV activation (tcgen05 kernels in csrc/flash_attn.cu).

``qkv`` is the ``[B*S, 3*Hl]`` bf16 output of the QKV GEMM whose columns are
``[Q heads | K heads | V heads]`` (each ``nh*d`` wide) -- exactly the layout
the reference reshapes to ``[B, S, 3, nh, d]`` (model/transformer.py:27-33).
Outputs are ``ctx [B*S, nh*d]`` bf16 (token-major, ready for the O GEMM) and
``lse [B, nh, S]`` fp32 for the backward.  ``flash_attn_bwd`` returns
``dqkv`` in the same packed layout as ``qkv``.  There is no library fallback:
without the built extension :func:`native` raises.
"""
from __future__ import annotations

from . import native


def flash_attn_fwd(qkv, B, S, nh, d):
    return native().flash_attn_fwd(qkv, B, S, nh, d)


def flash_attn_bwd(dctx, qkv, ctx, lse, B, S, nh, d):
    return native().flash_attn_bwd(dctx, qkv, ctx, lse, B, S, nh, d)
