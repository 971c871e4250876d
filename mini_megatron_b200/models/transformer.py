"""GPT decoder: Attention, MLP, DecoderLayer, Decoder, GPT.

Module tree and parameter names match the reference (model/transformer.py:8-109)
so its ``state_dict`` keys are unchanged:
``decoder.layers.{i}.{ln1,attn.qkv,attn.o,ln2,mlp.fc1,mlp.fc2}``,
``embedding.{token,position}_embedding``, ``ln_f``, ``lm_head``.

Two execution paths share these modules:

* CUDA tensors -> :class:`DecoderLayer` runs as ONE native autograd Function
  (``native_layers.DecoderLayerFn``) over the sm_100a kernels; ``GPT`` fuses
  ``ln_f -> lm_head -> vocab-parallel CE`` likewise.
* CPU tensors -> the same math in plain PyTorch ops (pre-LN, fused QKV with
  the stride-3 TP layout, causal SDPA, exact GELU, no biases), which is the
  oracle the native path is tested against.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..parallel import process_groups as pg
from ..parallel.tensor_parallel import ColumnParallelLinear, RowParallelLinear


class Attention(nn.Module):
    """Causal multi-head self-attention with a fused, TP-sharded QKV projection."""

    def __init__(self, hidden_size, num_heads, sequence_parallel=None):
        super().__init__()
        tp = pg.tp_size()
        if num_heads % tp:
            raise ValueError("num_heads must divide evenly by TP size")
        self.num_heads = num_heads // tp
        self.head_dim = hidden_size // num_heads
        self.hidden_size_per_partition = hidden_size // tp
        # stride 3: each TP rank holds an equal subset of Q, K and V heads
        self.qkv = ColumnParallelLinear(hidden_size, 3 * hidden_size, bias=False, stride=3,
                                        sequence_parallel=sequence_parallel)
        self.o = RowParallelLinear(hidden_size, hidden_size, bias=False, sequence_parallel=sequence_parallel)

    def core_attention(self, qkv):
        B, S, _ = qkv.shape
        qkv = qkv.reshape(B, S, 3, self.num_heads, self.head_dim)
        q, k, v = (t.transpose(1, 2) for t in qkv.unbind(2))
        out = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return out.transpose(1, 2).reshape(B, S, self.hidden_size_per_partition)

    def forward(self, x):
        qkv = self.qkv(x)
        if qkv.is_cuda:
            from ..ops.attention import flash_attn_fwd
            B, S, _ = qkv.shape
            ctx = _AttnFn.apply(qkv, self.num_heads, self.head_dim)
            return self.o(ctx)
        return self.o(self.core_attention(qkv))


class _AttnFn(torch.autograd.Function):
    """Native causal attention on a packed [B, S, 3*Hl] qkv tensor (standalone module use)."""

    @staticmethod
    def forward(ctx, qkv, nh, d):
        from ..ops.attention import flash_attn_fwd
        B, S, W = qkv.shape
        q2 = qkv.reshape(B * S, W).to(torch.bfloat16).contiguous()
        out, lse = flash_attn_fwd(q2, B, S, nh, d)
        ctx.save_for_backward(q2, out, lse)
        ctx.shape, ctx.nh, ctx.d, ctx.dtype = (B, S, W), nh, d, qkv.dtype
        return out.view(B, S, nh * d)

    @staticmethod
    def backward(ctx, dout):
        from ..ops.attention import flash_attn_bwd
        q2, out, lse = ctx.saved_tensors
        B, S, W = ctx.shape
        d2 = dout.reshape(B * S, -1).to(torch.bfloat16).contiguous()
        dqkv = flash_attn_bwd(d2, q2, out, lse, B, S, ctx.nh, ctx.d)
        return dqkv.view(B, S, W).to(ctx.dtype), None, None


class MLP(nn.Module):
    def __init__(self, hidden_size, ffn_hidden_size, sequence_parallel=None):
        super().__init__()
        self.fc1 = ColumnParallelLinear(hidden_size, ffn_hidden_size, bias=False, sequence_parallel=sequence_parallel)
        self.fc2 = RowParallelLinear(ffn_hidden_size, hidden_size, bias=False, sequence_parallel=sequence_parallel)

    def forward(self, x):
        return self.fc2(F.gelu(self.fc1(x)))


class DecoderLayer(nn.Module):
    """Pre-LN block: x + attn(ln1(x)), then + mlp(ln2(.))."""

    def __init__(self, hidden_size, num_heads, ffn_hidden_size, sequence_parallel=None, recompute=False):
        super().__init__()
        self.ln1 = nn.LayerNorm(hidden_size)
        self.attn = Attention(hidden_size, num_heads, sequence_parallel)
        self.ln2 = nn.LayerNorm(hidden_size)
        self.mlp = MLP(hidden_size, ffn_hidden_size, sequence_parallel)
        self.sequence_parallel = pg.sequence_parallel_enabled() if sequence_parallel is None else sequence_parallel
        self.recompute = recompute
        # LayerNorm parameters see only the local sequence shard under SP:
        # their gradients need a TP all-reduce before the optimizer step.
        for p in list(self.ln1.parameters()) + list(self.ln2.parameters()):
            p.sequence_parallel_grad = bool(self.sequence_parallel)

    def _forward(self, x):
        x = x + self.attn(self.ln1(x))
        x = x + self.mlp(self.ln2(x))
        return x

    def native_forward(self, x, recompute=None):
        from .native_layers import DecoderLayerFn
        group = pg.tp_group()
        sp = bool(self.sequence_parallel and group is not None)
        rc = self.recompute if recompute is None else recompute
        return DecoderLayerFn.apply(x.float().contiguous(), self, group, sp, rc, *self.parameters())

    def forward(self, x, use_checkpoint=False):
        if x.is_cuda:
            return self.native_forward(x, recompute=use_checkpoint or self.recompute)
        if use_checkpoint or self.recompute:
            return torch.utils.checkpoint.checkpoint(self._forward, x, use_reentrant=False)
        return self._forward(x)


class Decoder(nn.Module):
    """Stack of DecoderLayer blocks (``layer_ids`` is metadata for pipeline stages)."""

    def __init__(self, hidden_size, num_heads, ffn_hidden_size, num_layers, layer_ids=None, sequence_parallel=None,
                 recompute=False):
        super().__init__()
        self.layer_ids = list(range(num_layers)) if layer_ids is None else list(layer_ids)
        self.layers = nn.ModuleList([
            DecoderLayer(hidden_size, num_heads, ffn_hidden_size, sequence_parallel, recompute)
            for _ in self.layer_ids
        ])

    def forward(self, x):
        for layer in self.layers:
            x = layer(x)
        return x


class GPT(nn.Module):
    """embedding -> decoder -> ln_f -> lm_head [-> loss].

    Returns ``logits`` or ``(logits, loss)`` when labels, loss_mask and a loss
    function are given (reference model/transformer.py:90-109).  Logits are
    this rank's vocabulary shard when TP > 1 (use
    ``gather_from_model_parallel_region`` for the full vocabulary).  On CUDA
    with the package's CrossEntropyLoss the head runs fused
    (``native_layers.HeadLossFn``) and the returned logits buffer is
    overwritten by its gradient during backward.
    """

    def __init__(self, embedding, decoder, ln_f, lm_head, loss_fn=None):
        super().__init__()
        self.embedding = embedding
        self.decoder = decoder
        self.ln_f = ln_f
        self.lm_head = lm_head
        self.loss_fn = loss_fn

    def forward(self, input_ids, labels=None, loss_mask=None):
        x = self.embedding(input_ids)
        x = self.decoder(x)
        return head_forward(self.ln_f, self.lm_head, self.loss_fn, x, labels, loss_mask)


def head_forward(ln_f, lm_head, loss_fn, x, labels=None, loss_mask=None):
    """ln_f -> lm_head [-> loss], fused on CUDA when the loss is the package's CE."""
    from .loss import CrossEntropyLoss
    want_loss = labels is not None and loss_mask is not None and loss_fn is not None
    if (want_loss and x.is_cuda and isinstance(loss_fn, CrossEntropyLoss) and lm_head.bias is None
            and not lm_head.gather_output):
        from .native_layers import HeadLossFn
        group = pg.tp_group()
        sp = bool(lm_head.sequence_parallel and group is not None)
        n_vocab = loss_fn.vocab_size if loss_fn.vocab_size is not None else lm_head.out_features
        loss, logits = HeadLossFn.apply(x.float().contiguous(), ln_f, lm_head, labels, loss_mask, n_vocab, group,
                                        sp, ln_f.weight, ln_f.bias, lm_head.weight)
        B = labels.shape[0]
        return logits.view(B, -1, logits.shape[-1]), loss
    h = ln_f(x)
    logits = lm_head(h)
    if want_loss:
        return logits, loss_fn(logits, labels, loss_mask)
    return logits
