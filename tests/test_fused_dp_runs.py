"""Replication runs of the fused data-parallel kernel (host-side layout logic, CPU).

The kernel all-gathers only the copy of each parameter that the forward kernels read: the
bf16 shadow of a GEMM weight, the fp32 value of a LayerNorm / embedding parameter.  The runs
handed to it must tile every owned shard exactly, in order, with the right kind.
"""
import torch

from mini_megatron_b200.config import GPTConfig
from mini_megatron_b200.models import build_gpt
from mini_megatron_b200.parallel.fused_dp import replication_runs
from mini_megatron_b200.parallel.param_buffer import ParamBuffer
from mini_megatron_b200.parallel.tensor_parallel import VocabParallelEmbedding


def _layout(world, bucket_elems):
    torch.manual_seed(0)
    model = build_gpt(GPTConfig(num_layers=2, hidden_size=64, num_attention_heads=4, ffn_hidden_size=256,
                                max_seq_len=32, vocab_size=1000))
    buf = ParamBuffer(model.parameters(), align=world, bucket_elems=bucket_elems)
    fp32 = {id(p) for m in model.modules() if isinstance(m, (torch.nn.LayerNorm, torch.nn.Embedding,
                                                               VocabParallelEmbedding))
            for p in m.parameters(recurse=False)}
    kinds = [1 if (id(p) in fp32 or p.dim() != 2) else 0 for p in buf.params]
    return buf, kinds


def _kind_at(buf, kinds, e):
    for i, off in enumerate(buf.offsets):
        end = buf.offsets[i + 1] if i + 1 < len(buf.offsets) else buf.numel
        if off <= e < end:
            return kinds[i]
    raise AssertionError(e)


def test_runs_tile_each_shard_with_the_right_kind():
    for world in (1, 2, 4):
        for bucket_elems in (0, 20000):
            buf, kinds = _layout(world, bucket_elems)
            shards = [buf.shard_range(b, r) for b in range(len(buf.buckets)) for r in range(world)]
            runs = replication_runs(buf.offsets, kinds, buf.numel, shards, max_segs=64)
            for (lo, hi), rs in zip(shards, runs):
                assert rs is not None
                assert rs[0][0] == 0 and rs[-1][1] == (hi - lo) // 4
                for a, b in zip(rs, rs[1:]):
                    assert a[1] == b[0] and a[2] != b[2]       # contiguous, adjacent kinds differ
                for b4, e4, kind, _ in rs:
                    assert b4 < e4 and kind in (0, 1)
                    for e in (lo + 4 * b4, lo + 4 * e4 - 1):    # both ends of the run
                        assert _kind_at(buf, kinds, e) == kind


def test_gemm_weights_are_kind_0_and_the_rest_kind_1():
    buf, kinds = _layout(1, 0)
    names = {id(p): n for n, p in build_gpt(GPTConfig(num_layers=2, hidden_size=64, num_attention_heads=4,
                                                        ffn_hidden_size=256, max_seq_len=32,
                                                        vocab_size=1000)).named_parameters()}
    by_shape = [(tuple(p.shape), k) for p, k in zip(buf.params, kinds)]
    assert (tuple([64 * 3, 64]), 0) in by_shape          # QKV weight
    assert (tuple([64]), 1) in by_shape                  # LayerNorm vectors
    assert sum(1 for p, k in zip(buf.params, kinds) if k == 1 and p.dim() == 2) == 2  # token + position tables
    assert names  # the model built


def test_too_many_runs_fall_back_to_full_replication():
    buf, kinds = _layout(1, 0)
    runs = replication_runs(buf.offsets, kinds, buf.numel, [buf.shard_range(0, 0)], max_segs=2)
    assert runs == [None]
