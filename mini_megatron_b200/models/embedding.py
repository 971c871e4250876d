"""Token (vocab-parallel) + learned absolute position embedding.

Reference: model/embedding.py:5-16 (output = tok_emb + pos_emb, [B, S, H]).
Under sequence parallelism the output is this rank's sequence shard
``[B, S/tp, H]``.  On CUDA the whole block is one native Function (gather
kernel + TP reduction; scatter-add backward into the fp32 main grads).
"""
import torch
import torch.nn as nn

from ..comm import sequence_parallel as spc
from ..parallel import process_groups as pg
from ..parallel.tensor_parallel import VocabParallelEmbedding


class Embedding(nn.Module):
    def __init__(self, vocab_size, hidden_size, max_seq_len, padded_vocab_size=None, sequence_parallel=None):
        super().__init__()
        self.token_embedding = VocabParallelEmbedding(vocab_size, hidden_size, padded_vocab_size)
        self.position_embedding = nn.Embedding(max_seq_len, hidden_size)
        self.sequence_parallel = pg.sequence_parallel_enabled() if sequence_parallel is None else sequence_parallel

    def forward(self, input_ids):
        group = pg.tp_group()
        sp = self.sequence_parallel and group is not None
        if input_ids.is_cuda:
            from .native_layers import EmbeddingFn
            return EmbeddingFn.apply(input_ids, self, group, sp, self.token_embedding.weight,
                                     self.position_embedding.weight)
        seq_len = input_ids.size(-1)
        pos_ids = torch.arange(seq_len, dtype=torch.long, device=input_ids.device)
        out = self.token_embedding(input_ids) + self.position_embedding(pos_ids)
        if sp:
            out = spc.scatter_to_sequence_parallel_region(out, group)
        return out
