"""Builders for a full GPT and for one pipeline stage.

``build_gpt`` mirrors the module construction of the reference's non-PP path
(main.py:168-173); ``GPTStage`` is the pipeline-stage container whose
parameter names (``embedding.*`` on the first stage, ``decoder_layers.{i}.*``,
``ln_f.*`` / ``lm_head.*`` on the last) match the reference's PP layout
(main.py:116-134 and its MiniPipelineStage harness module).

Layers are split as in the reference: ``L // pp`` per stage, the last stage
takes the remainder (main.py:119-121).
"""
from __future__ import annotations

import torch.nn as nn

from ..config import GPTConfig
from ..parallel import process_groups as pg
from ..parallel.tensor_parallel import ColumnParallelLinear, pad_vocab_size
from .embedding import Embedding
from .loss import CrossEntropyLoss
from .transformer import GPT, Decoder, DecoderLayer, head_forward


def padded_vocab(cfg: GPTConfig) -> int:
    return pad_vocab_size(cfg.vocab_size, pg.tp_size(), cfg.vocab_pad_multiple)


def _lm_head(cfg):
    vp = padded_vocab(cfg)
    head = ColumnParallelLinear(cfg.hidden_size, vp, bias=False, gather_output=False)
    if vp > cfg.vocab_size:
        # padded vocabulary rows produce masked logits; keep them zero
        import torch
        with torch.no_grad():
            start = pg.tp_rank() * head.out_features_per_partition
            lo = max(0, cfg.vocab_size - start)
            head.weight[lo:].zero_()
    return head


def build_gpt(cfg: GPTConfig, device=None, sequence_parallel=None, recompute=False) -> GPT:
    vp = padded_vocab(cfg)
    embedding = Embedding(cfg.vocab_size, cfg.hidden_size, cfg.max_seq_len, vp, sequence_parallel)
    decoder = Decoder(cfg.hidden_size, cfg.num_attention_heads, cfg.ffn_hidden_size, cfg.num_layers,
                      sequence_parallel=sequence_parallel, recompute=recompute)
    ln_f = nn.LayerNorm(cfg.hidden_size)
    sp = pg.sequence_parallel_enabled() if sequence_parallel is None else sequence_parallel
    for p in ln_f.parameters():
        p.sequence_parallel_grad = bool(sp)
    model = GPT(embedding, decoder, ln_f, _lm_head(cfg), CrossEntropyLoss(cfg.vocab_size))
    return model.to(device) if device is not None else model


def stage_layer_range(num_layers: int, pp_rank: int, pp_size: int):
    per = num_layers // pp_size
    start = pp_rank * per
    end = start + per if pp_rank < pp_size - 1 else num_layers
    return start, end


class GPTStage(nn.Module):
    """One pipeline stage: [embedding] + decoder_layers + [ln_f, lm_head, loss]."""

    def __init__(self, cfg: GPTConfig, pp_rank: int, pp_size: int, sequence_parallel=None, recompute=False):
        super().__init__()
        self.cfg = cfg
        self.pp_rank, self.pp_size = pp_rank, pp_size
        self.is_first, self.is_last = pp_rank == 0, pp_rank == pp_size - 1
        start, end = stage_layer_range(cfg.num_layers, pp_rank, pp_size)
        self.layer_ids = list(range(start, end))
        vp = padded_vocab(cfg)
        self.embedding = (Embedding(cfg.vocab_size, cfg.hidden_size, cfg.max_seq_len, vp, sequence_parallel)
                          if self.is_first else None)
        self.decoder_layers = nn.ModuleList([
            DecoderLayer(cfg.hidden_size, cfg.num_attention_heads, cfg.ffn_hidden_size, sequence_parallel, recompute)
            for _ in self.layer_ids
        ])
        sp = pg.sequence_parallel_enabled() if sequence_parallel is None else sequence_parallel
        if self.is_last:
            self.ln_f = nn.LayerNorm(cfg.hidden_size)
            for p in self.ln_f.parameters():
                p.sequence_parallel_grad = bool(sp)
            self.lm_head = _lm_head(cfg)
            self.loss_fn = CrossEntropyLoss(cfg.vocab_size)
        else:
            self.ln_f = self.lm_head = self.loss_fn = None

    def forward(self, x_or_ids, labels=None, loss_mask=None):
        x = self.embedding(x_or_ids) if self.is_first else x_or_ids
        for layer in self.decoder_layers:
            x = layer(x)
        if self.is_last:
            return head_forward(self.ln_f, self.lm_head, self.loss_fn, x, labels, loss_mask)
        return x
