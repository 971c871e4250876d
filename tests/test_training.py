"""End-to-end CPU training behaviour (reference tests/test_training.py in spirit) and the CLI."""
import os
import subprocess
import sys

import pytest
import torch

from mini_megatron_b200 import config as cfg
from mini_megatron_b200.models import GPT, CrossEntropyLoss, Decoder, Embedding
from mini_megatron_b200.parallel.data_parallel import allreduce_grads

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _tiny_gpt():
    torch.manual_seed(0)
    return GPT(Embedding(64, 64, 16), Decoder(64, 4, 256, 2), torch.nn.LayerNorm(64),
               torch.nn.Linear(64, 64, bias=False), CrossEntropyLoss())


def _batch():
    return torch.tensor([[(i + 1) % 64 for i in range(8)]] * 4)


def test_loss_decreases():
    torch.manual_seed(42)
    model = _tiny_gpt()
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    x = _batch()
    with torch.no_grad():
        start = model(x, x, torch.ones(4, 8))[1].item()
    for _ in range(200):
        opt.zero_grad()
        model(x, x, torch.ones(4, 8))[1].backward()
        opt.step()
    with torch.no_grad():
        end = model(x, x, torch.ones(4, 8))[1].item()
    assert end < start - 1.0 and end < 3.5, (start, end)


def test_gradients_reach_every_parameter_and_step_updates():
    model = _tiny_gpt()
    x = _batch()
    model(x, x, torch.ones(4, 8))[1].backward()
    assert not [n for n, p in model.named_parameters() if p.grad is None]
    before = [p.detach().clone() for p in model.parameters()]
    torch.optim.AdamW(model.parameters(), lr=1e-2).step()
    assert any(not torch.allclose(a, b) for a, b in zip(before, model.parameters()))


def test_allreduce_grads_without_group_is_noop():
    model = _tiny_gpt()
    x = _batch()
    model(x, x, torch.ones(4, 8))[1].backward()
    g = {n: p.grad.clone() for n, p in model.named_parameters()}
    allreduce_grads(model, None)
    for n, p in model.named_parameters():
        assert torch.equal(p.grad, g[n])


def test_config_consistency():
    c = cfg.get_model_config()
    assert c["hidden_size"] == cfg.HIDDEN_SIZE and c["vocab_size"] % 8 == 0
    assert cfg.HIDDEN_SIZE % cfg.NUM_ATTENTION_HEADS == 0
    for name, p in cfg.PRESETS.items():
        assert p.hidden_size % p.num_attention_heads == 0, name


def test_lr_lambda_matches_reference_shape():
    from mini_megatron_b200.training import make_lr_lambda
    f = make_lr_lambda(10, 100)
    assert f(0) == 0.0 and abs(f(5) - 0.5) < 1e-12 and abs(f(10) - 1.0) < 1e-12 and abs(f(100)) < 1e-12


def test_cli_runs_pp2_tp1_dp1_on_gloo(tmp_path):
    env = dict(os.environ, PYTHONPATH=ROOT)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29655", os.path.join(ROOT, "main.py"), "--model", "tiny",
           "--pp", "2", "--num-steps", "4", "--warmup-steps", "1", "--micro-batch-size", "2",
           "--num-microbatches", "2", "--log-interval", "2", "--save", str(tmp_path / "ck")]
    out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=240)
    assert out.returncode == 0, out.stdout[-2000:] + out.stderr[-4000:]
    assert "Throughput:" in out.stdout and "step    2 | loss" in out.stdout
    assert (tmp_path / "ck" / "manifest.json").exists()


@pytest.mark.parametrize("pp", [1])
def test_trainer_attaches_every_parameter_to_a_grad_ready_hook(pp):
    """DP buckets launch strictly in order during backward, so every parameter of the
    chunk must belong to a module whose backward announces its gradients."""
    import torch.distributed as dist
    from mini_megatron_b200.config import PRESETS
    from mini_megatron_b200.parallel import process_groups as pg
    from mini_megatron_b200.training import TrainConfig, Trainer
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29588")
        dist.init_process_group("gloo", rank=0, world_size=1)
    t = Trainer(TrainConfig(model=PRESETS["tiny"], micro_batch_size=2, seq_len=32, pp=pp, dp_early_buckets=True),
                device="cpu")
    assert t.grad_sync.attached_params == {id(p) for p in t.buf.params}
    pg.set_model_parallel(None)
