"""Model and training configuration.

Module-level constants and ``get_model_config()`` mirror the reference's
config.py:3-30 (so code written against it keeps working); ``GPTConfig`` and
the presets add the BASELINE model sizes, which the reference can only reach
by editing its constants.
"""
from __future__ import annotations

import dataclasses

import torch

NUM_LAYERS = 12
HIDDEN_SIZE = 768
NUM_ATTENTION_HEADS = 12
FFN_HIDDEN_SIZE = 3072
MAX_SEQ_LEN = 512
VOCAB_SIZE = 50304

MICRO_BATCH_SIZE = 4
LEARNING_RATE = 6e-4
MIN_LR = 1e-5
WEIGHT_DECAY = 0.1
WARMUP_STEPS = 10
MAX_TRAIN_STEPS = 100
MAX_GRAD_NORM = 1.0


def get_model_config():
    return {
        "num_layers": NUM_LAYERS,
        "hidden_size": HIDDEN_SIZE,
        "num_attention_heads": NUM_ATTENTION_HEADS,
        "ffn_hidden_size": FFN_HIDDEN_SIZE,
        "max_seq_len": MAX_SEQ_LEN,
        "vocab_size": VOCAB_SIZE,
    }


def enable_tf32():
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.backends.cudnn.allow_tf32 = True


@dataclasses.dataclass
class GPTConfig:
    num_layers: int = NUM_LAYERS
    hidden_size: int = HIDDEN_SIZE
    num_attention_heads: int = NUM_ATTENTION_HEADS
    ffn_hidden_size: int = FFN_HIDDEN_SIZE
    max_seq_len: int = MAX_SEQ_LEN
    vocab_size: int = VOCAB_SIZE
    vocab_pad_multiple: int = 128

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    def as_dict(self):
        return dataclasses.asdict(self)

    def num_params(self, padded_vocab: int | None = None) -> int:
        h, f, L = self.hidden_size, self.ffn_hidden_size, self.num_layers
        v = padded_vocab or self.vocab_size
        per_layer = 3 * h * h + h * h + 2 * h * f + 4 * h
        return L * per_layer + 2 * v * h + self.max_seq_len * h + 2 * h

    def flops_per_token(self, seq_len: int) -> float:
        """Training FLOPs per token (fwd + bwd, causal attention counted at half)."""
        h, f, L, v = self.hidden_size, self.ffn_hidden_size, self.num_layers, self.vocab_size
        dense = 2 * (3 * h * h + h * h + 2 * h * f) * L + 2 * h * v
        attn = 2 * 2 * seq_len * h * L / 2
        return 3.0 * (dense + attn)


PRESETS = {
    "tiny": GPTConfig(num_layers=4, hidden_size=64, num_attention_heads=4, ffn_hidden_size=256, max_seq_len=32,
                      vocab_size=1024),
    "gpt-125m": GPTConfig(num_layers=12, hidden_size=768, num_attention_heads=12, ffn_hidden_size=3072,
                          max_seq_len=1024, vocab_size=50257),
    "gpt-1.3b": GPTConfig(num_layers=24, hidden_size=2048, num_attention_heads=16, ffn_hidden_size=8192,
                          max_seq_len=2048, vocab_size=50257),
    "gpt-6.7b": GPTConfig(num_layers=32, hidden_size=4096, num_attention_heads=32, ffn_hidden_size=16384,
                          max_seq_len=2048, vocab_size=50257),
    "reference-125m": GPTConfig(),
}
