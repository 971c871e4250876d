"""Activation recomputation (``--recompute``) changes memory, never results.

The reference wraps each decoder layer in ``torch.utils.checkpoint``
(model/recompute.py:4-6, model/transformer.py:49-67).  Here the CPU path does
the same and the native CUDA path re-runs the layer's fused forward inside its
backward.  Every case trains the same model from the same seed with and
without recomputation and requires the same losses and parameters.
"""
import pytest
import torch

from dist_util import run_ranks

CFG = dict(num_layers=2, hidden_size=64, num_attention_heads=4, ffn_hidden_size=256, max_seq_len=32,
           vocab_size=1000)
B, S = 2, 32


def _worker(rank, world, tp, pp, sp, recompute, micro, steps):
    from mini_megatron_b200.config import GPTConfig
    from mini_megatron_b200.training import TrainConfig, Trainer, synthetic_batch
    cfg = TrainConfig(model=GPTConfig(**CFG), micro_batch_size=B, seq_len=S, num_microbatches=micro, tp=tp, pp=pp,
                      sequence_parallel=sp, recompute=recompute, lr=1e-3, warmup_steps=0, num_steps=10)
    t = Trainer(cfg, device="cpu")
    losses = []
    for s in range(steps):
        tok, lab = synthetic_batch(micro, B, S, CFG["vocab_size"], seed=50 + s)
        loss = t.train_step(tok, lab)
        losses.append(None if loss is None else float(loss))
    state = {k: v.detach().clone() for k, v in t.model.state_dict().items()}
    t.destroy()
    return {"losses": losses, "state": state}


def _compare(a, b):
    for ra, rb in zip(a, b):
        assert ra["losses"] == pytest.approx(rb["losses"], rel=1e-6, abs=1e-6), (ra["losses"], rb["losses"])
        for k, v in ra["state"].items():
            torch.testing.assert_close(v, rb["state"][k], rtol=1e-5, atol=1e-6, msg=k)


def test_recompute_single_process_matches():
    _compare(run_ranks(_worker, 1, 1, 1, False, True, 2, 2), run_ranks(_worker, 1, 1, 1, False, False, 2, 2))


@pytest.mark.parametrize("sp", [False, True])
def test_recompute_tp2_matches(sp):
    _compare(run_ranks(_worker, 2, 2, 1, sp, True, 2, 2), run_ranks(_worker, 2, 2, 1, sp, False, 2, 2))


def test_recompute_pp2_1f1b_matches():
    _compare(run_ranks(_worker, 2, 1, 2, False, True, 4, 2), run_ranks(_worker, 2, 1, 2, False, False, 4, 2))
