"""Checkpointing: reference-compatible single file, distributed manifest + checksums, corruption."""
import json
import os

import pytest
import torch

from dist_util import run_ranks


def _tiny():
    from mini_megatron_b200.config import PRESETS
    from mini_megatron_b200.models import build_gpt
    torch.manual_seed(0)
    return build_gpt(PRESETS["tiny"])


def _train_one(model, opt, sched):
    ids = torch.randint(0, 1024, (2, 32))
    opt.zero_grad()
    model(ids, ids, torch.ones(2, 32))[1].backward()
    opt.step()
    sched.step()


def test_reference_layout_round_trip(tmp_path):
    from mini_megatron_b200.utils.checkpoint import load_checkpoint, save_checkpoint
    m = _tiny()
    opt = torch.optim.AdamW(m.parameters(), lr=1e-3)
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda s: 1.0)
    _train_one(m, opt, sched)
    path = str(tmp_path / "ck" / "model.pt")
    save_checkpoint(m, opt, sched, 7, path)
    state = torch.load(path, weights_only=True)
    assert set(state) == {"model_state", "optimizer_state", "scheduler_state", "step"}
    m2 = _tiny()
    opt2 = torch.optim.AdamW(m2.parameters(), lr=1e-3)
    sched2 = torch.optim.lr_scheduler.LambdaLR(opt2, lambda s: 1.0)
    assert load_checkpoint(m2, opt2, sched2, path, "cpu") == 7
    for a, b in zip(m.state_dict().values(), m2.state_dict().values()):
        torch.testing.assert_close(a, b)


def test_fused_adamw_state_dict_has_torch_layout(tmp_path):
    from mini_megatron_b200.optim import FusedAdamW
    m = _tiny()
    opt = FusedAdamW(m.parameters(), lr=1e-3, weight_decay=0.1)
    ref_m = _tiny()
    ref = torch.optim.AdamW(ref_m.parameters(), lr=1e-3, weight_decay=0.1)
    for model, o in ((m, opt), (ref_m, ref)):
        ids = torch.randint(0, 1024, (2, 32), generator=torch.Generator().manual_seed(1))
        model(ids, ids, torch.ones(2, 32))[1].backward()
        o.step()
    sd, rsd = opt.state_dict(), ref.state_dict()
    assert set(sd) == set(rsd) and set(sd["state"]) == set(rsd["state"])
    for k in sd["state"]:
        assert set(sd["state"][k]) >= {"exp_avg", "exp_avg_sq", "step"}
        torch.testing.assert_close(sd["state"][k]["exp_avg"], rsd["state"][k]["exp_avg"])
    for a, b in zip(m.parameters(), ref_m.parameters()):
        torch.testing.assert_close(a, b)


def _dist_ckpt_worker(rank, world, directory, zero1):
    from mini_megatron_b200.config import PRESETS
    from mini_megatron_b200.training import TrainConfig, Trainer, synthetic_batch
    from mini_megatron_b200.utils.checkpoint import load_distributed_checkpoint, save_distributed_checkpoint
    cfg = TrainConfig(model=PRESETS["tiny"], micro_batch_size=2, num_microbatches=1, zero1=zero1, warmup_steps=0,
                      num_steps=10, lr=1e-3)
    t = Trainer(cfg, device="cpu")
    tok, lab = synthetic_batch(1, 2, 32, 1024, seed=rank)
    t.train_step(tok, lab)
    save_distributed_checkpoint(directory, *t.state_for_checkpoint(), 1, mpu=t.mpu, sharded_optimizer=zero1)
    before = t.train_step(tok, lab).item()
    # reload into a fresh trainer and take the same step again
    t2 = Trainer(cfg, device="cpu")
    step = load_distributed_checkpoint(directory, *t2.state_for_checkpoint(), mpu=t2.mpu)
    after = t2.train_step(tok, lab).item()
    return {"step": step, "before": before, "after": after}


@pytest.mark.parametrize("zero1", [False, True])
def test_distributed_checkpoint_resume_is_exact(tmp_path, zero1):
    res = run_ranks(_dist_ckpt_worker, 2, str(tmp_path), zero1)
    for r in res:
        assert r["step"] == 1
        assert abs(r["before"] - r["after"]) < 1e-6
    manifest = json.load(open(tmp_path / "manifest.json"))
    assert manifest["topology"] == {"tp": 1, "pp": 1, "dp": 2}
    assert manifest["sharded_optimizer"] == zero1


def test_corrupt_and_mismatched_checkpoints_fail_cleanly(tmp_path):
    import torch.distributed as dist
    from mini_megatron_b200.utils.checkpoint import (CheckpointError, load_distributed_checkpoint,
                                                     save_distributed_checkpoint)
    m = _tiny()
    opt = torch.optim.AdamW(m.parameters(), lr=1e-3)
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda s: 1.0)
    assert not dist.is_initialized()
    save_distributed_checkpoint(str(tmp_path), m, opt, sched, 3)
    assert load_distributed_checkpoint(str(tmp_path), m, opt, sched) == 3
    # flip bytes in the model file -> checksum mismatch
    f = tmp_path / "model_tp00_pp000.pt"
    data = bytearray(f.read_bytes())
    data[len(data) // 2] ^= 0xFF
    f.write_bytes(bytes(data))
    with pytest.raises(CheckpointError, match="corrupt"):
        load_distributed_checkpoint(str(tmp_path), m, opt, sched)
    # topology mismatch
    man = json.load(open(tmp_path / "manifest.json"))
    man["topology"]["tp"] = 2
    json.dump(man, open(tmp_path / "manifest.json", "w"))
    with pytest.raises(CheckpointError, match="topology"):
        load_distributed_checkpoint(str(tmp_path), m, opt, sched)
    os.remove(tmp_path / "manifest.json")
    with pytest.raises(CheckpointError, match="manifest"):
        load_distributed_checkpoint(str(tmp_path), m, opt, sched)


REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


def _ref_model():
    import sys
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import config as rcfg
    from model.embedding import Embedding
    from model.loss import CrossEntropyLoss
    from model.transformer import GPT, Decoder
    from parallel.process_groups import set_model_parallel
    from parallel.tensor_parallel import ColumnParallelLinear
    from mini_megatron_b200.config import PRESETS
    c = PRESETS["tiny"]
    set_model_parallel(None)
    torch.manual_seed(1)
    return GPT(Embedding(c.vocab_size, c.hidden_size, c.max_seq_len),
               Decoder(c.hidden_size, c.num_attention_heads, c.ffn_hidden_size, c.num_layers),
               torch.nn.LayerNorm(c.hidden_size),
               ColumnParallelLinear(c.hidden_size, c.vocab_size, bias=False, gather_output=True), CrossEntropyLoss())


@pytest.mark.skipif(not os.path.exists(os.path.join(REF, "checkpoint.py")), reason="reference sources not present")
@pytest.mark.parametrize("direction", ["reference_to_ours", "ours_to_reference"])
def test_checkpoints_interchange_with_the_reference(tmp_path, direction):
    """A checkpoint written by the reference's checkpoint.py loads here (model, optimizer, scheduler, step)
    and continues training identically, and vice versa."""
    import importlib.util
    import sys
    if REF not in sys.path:
        sys.path.insert(0, REF)
    spec = importlib.util.spec_from_file_location("ref_checkpoint", os.path.join(REF, "checkpoint.py"))
    ref_ck = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref_ck)
    from mini_megatron_b200.utils import checkpoint as our_ck
    src_model = _ref_model() if direction == "reference_to_ours" else _tiny()
    dst_model = _tiny() if direction == "reference_to_ours" else _ref_model()
    mk = lambda m: torch.optim.AdamW(m.parameters(), lr=1e-3, weight_decay=0.1)  # noqa: E731
    src_opt, dst_opt = mk(src_model), mk(dst_model)
    src_sched = torch.optim.lr_scheduler.LambdaLR(src_opt, lambda s: min(1.0, (s + 1) / 10))
    dst_sched = torch.optim.lr_scheduler.LambdaLR(dst_opt, lambda s: min(1.0, (s + 1) / 10))
    torch.manual_seed(5)
    _train_one(src_model, src_opt, src_sched)
    path = str(tmp_path / "ck.pt")
    save = ref_ck.save_checkpoint if direction == "reference_to_ours" else our_ck.save_checkpoint
    load = our_ck.load_checkpoint if direction == "reference_to_ours" else ref_ck.load_checkpoint
    save(src_model, src_opt, src_sched, 3, path)
    assert load(dst_model, dst_opt, dst_sched, path, "cpu") == 3
    for (na, a), (nb, b) in zip(src_model.state_dict().items(), dst_model.state_dict().items()):
        assert na == nb and torch.equal(a, b)
    # one more identical step on both keeps them identical (optimizer state and LR came across)
    torch.manual_seed(9)
    _train_one(src_model, src_opt, src_sched)
    torch.manual_seed(9)
    _train_one(dst_model, dst_opt, dst_sched)
    for a, b in zip(src_model.state_dict().values(), dst_model.state_dict().values()):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)
