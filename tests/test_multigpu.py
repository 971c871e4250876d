"""Multi-GPU checks (need >= 2 GPUs; skipped otherwise).

* fused DP (NVLink reduce-scatter + AdamW + all-gather kernel) gives the same
  parameters as the NCCL all-reduce path after several steps;
* native TP=2 (fused and NCCL, with and without sequence parallelism) and
  PP=2 reproduce the single-GPU loss, gradients and update of one canonical
  model sharded over the ranks.
"""
import os
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

NEED2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")

CFG = dict(num_layers=2, hidden_size=256, num_attention_heads=4, ffn_hidden_size=1024, max_seq_len=256,
           vocab_size=1000)


def _entry(rank, world, port, fn, args, out, env):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0", **env)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        res = fn(rank, world, *args)
        torch.save(res, os.path.join(out, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def _run(fn, world, *args, port=29711, env=None):
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        ps = [ctx.Process(target=_entry, args=(r, world, port, fn, args, d, env or {})) for r in range(world)]
        for p in ps:
            p.start()
        for p in ps:
            p.join(300)
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in ps), [p.exitcode for p in ps]
        return [torch.load(os.path.join(d, f"r{r}.pt"), weights_only=False) for r in range(world)]


def _assert_states_close(state, ref, tensor_rel=2e-3, model_rel=1e-4):
    """Same training math with a different summation order.

    Split-K weight gradients, the attention dQ and the embedding gradient are summed in no fixed
    order, and Adam divides each update by the running gradient magnitude: on tensors that are still
    near zero (LayerNorm biases start at 0; rarely used embedding rows) that turns rounding-level
    gradient differences into visible parameter differences.  So each tensor gets a loose bound and
    the whole parameter vector a tight one; a real defect (a missed bucket, a stale shard, NaN
    poison read before it was overwritten) moves parameters by O(lr) everywhere.
    """
    num = den = 0.0
    for k, v in state.items():
        want = ref[k]
        assert torch.isfinite(v).all(), k
        d = (v - want).norm().item()
        n = want.norm().item()
        assert d <= tensor_rel * n + 1e-6, (k, d / (n + 1e-12))
        num += d * d
        den += n * n
    assert (num ** 0.5) <= model_rel * (den ** 0.5), (num ** 0.5) / (den ** 0.5)


def _train(rank, world, tp, pp, sp, dp_impl, steps, micro, tp_impl="auto", recompute=False):
    from mini_megatron_b200.config import GPTConfig
    from mini_megatron_b200.training import TrainConfig, Trainer, synthetic_batch
    cfg = TrainConfig(model=GPTConfig(**CFG), micro_batch_size=2, seq_len=256, num_microbatches=micro, tp=tp, pp=pp,
                      sequence_parallel=sp, dp_impl=dp_impl, tp_impl=tp_impl, lr=1e-3, warmup_steps=0,
                      num_steps=100, bucket_mb=1.0, recompute=recompute)
    t = Trainer(cfg)
    dp_rank = t.mpu["dp_rank"]
    losses = []
    for s in range(steps):
        tok, lab = synthetic_batch(micro, 2, 256, CFG["vocab_size"], seed=100 * s + dp_rank)
        loss = t.train_step(tok, lab)
        losses.append(None if loss is None else loss.item())
    torch.cuda.synchronize()
    from mini_megatron_b200.ops import check_errors
    check_errors()
    state = {k: v.detach().float().cpu() for k, v in t.model.state_dict().items()}
    t.destroy()
    return {"losses": losses, "state": state}


@NEED2
@pytest.mark.parametrize("early", [False, True])
def test_fused_dp_matches_nccl_dp(early):
    """early: buckets start during backward (head and embedding hooks) and the bucket kernels defer
    their cross-rank completion wait to one wait at the end of the step."""
    env = {"MMB_DP_EARLY_BUCKETS": "1" if early else "0"}
    fused = _run(_train, 2, 1, 1, False, "fused", 3, 1, port=29711 + 10 * int(early), env=env)
    nccl = _run(_train, 2, 1, 1, False, "nccl", 3, 1, port=29712 + 10 * int(early), env=env)
    for r in range(2):
        for a, b in zip(fused[r]["losses"], nccl[r]["losses"]):
            assert abs(a - b) < 1e-4 * abs(b), (fused[r]["losses"], nccl[r]["losses"])
        _assert_states_close(fused[r]["state"], nccl[r]["state"])
    # replicas agree with each other exactly (both received the same all-gathered parameters)
    for k in fused[0]["state"]:
        assert torch.equal(fused[0]["state"][k], fused[1]["state"][k]), k


def _canonical_step(rank, world, tp, pp, sp, tp_impl, path):
    """Shard ONE canonical full model (saved at ``path``) over this rank's (tp, pp) position, run one
    training step on a fixed batch, and return the loss, the reduced gradients and the parameter
    update, all keyed by the full model's parameter names (TP shards are cut out of the full
    tensors by the caller)."""
    from mini_megatron_b200.config import GPTConfig
    from mini_megatron_b200.training import TrainConfig, Trainer, synthetic_batch
    from mini_megatron_b200.utils.checkpoint import _refresh_shadows
    cfg = TrainConfig(model=GPTConfig(**CFG), micro_batch_size=2, seq_len=256, num_microbatches=4, tp=tp, pp=pp,
                      sequence_parallel=sp, tp_impl=tp_impl, dp_impl="nccl", lr=1e-3, warmup_steps=0,
                      num_steps=100, cuda_graph="off")
    t = Trainer(cfg)
    full = torch.load(path, weights_only=True)
    tp_rank, pp_rank = t.mpu["tp_rank"], t.mpu["pp_rank"]
    names = {}
    for k in t.model.state_dict():
        g = k
        if pp > 1 and k.startswith("decoder_layers."):
            i, rest = k[len("decoder_layers."):].split(".", 1)
            g = f"decoder.layers.{t.model.layer_ids[int(i)]}.{rest}"
        names[k] = g
    sd = {k: _shard(full[g], g, tp_rank, tp) for k, g in names.items()}
    t.model.load_state_dict(sd)
    _refresh_shadows(t.model)
    before = {names[k]: v.detach().float().cpu().clone() for k, v in t.model.state_dict().items()}
    tok, lab = synthetic_batch(4, 2, 256, CFG["vocab_size"], seed=5)
    loss = t.train_step(tok, lab)
    torch.cuda.synchronize()
    grads = {names[k]: p.main_grad.detach().float().cpu().clone() for k, p in t.model.named_parameters()}
    after = {names[k]: v.detach().float().cpu() for k, v in t.model.state_dict().items()}
    t.destroy()
    return {"loss": None if loss is None else loss.item(), "grads": grads,
            "update": {k: after[k] - before[k] for k in after}}


def _shard(f, name, rank, world):
    from mini_megatron_b200.parallel.tensor_parallel import strided_partition_rows
    if world == 1:
        return f
    if name.endswith("attn.qkv.weight"):
        return strided_partition_rows(f, world, rank, stride=3)
    if name.endswith(("mlp.fc1.weight", "lm_head.weight", "token_embedding.weight")):
        return strided_partition_rows(f, world, rank, stride=1)
    if name.endswith(("attn.o.weight", "mlp.fc2.weight")):
        n = f.shape[1] // world
        return f[:, rank * n:(rank + 1) * n]
    return f


def _canonical(tmp_path):
    from mini_megatron_b200.config import GPTConfig
    from mini_megatron_b200.models import build_gpt
    torch.manual_seed(123)
    full = build_gpt(GPTConfig(**CFG)).state_dict()   # vocab 1000 -> 1024 rows, also the TP=2 padding
    path = str(tmp_path / "full.pt")
    torch.save(full, path)
    return path


def _rel(a, b):
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def _check_against_full(res, ref, tp):
    """Gradients (bf16 GEMM operands: ~1e-2 noise) and the Adam update direction match the
    single-GPU run of the same canonical model; sequence-parallel LayerNorm gradients are the
    sum over ranks of the local-shard gradients, as their NCCL reduction makes them."""
    for r_i, r in enumerate(res):
        tp_rank = r_i % tp
        for name, g in r["grads"].items():
            want = _shard(ref["grads"][name], name, tp_rank, tp)
            assert _rel(g, want) < 3e-2, (name, _rel(g, want))
            upd, want_u = r["update"][name], _shard(ref["update"][name], name, tp_rank, tp)
            # first Adam step: ~lr * sign(grad) per element; signs of noise-level gradients may differ
            agree = ((upd - want_u).abs() < 2e-4).float().mean().item()
            assert agree > 0.97, (name, agree)


@NEED2
@pytest.mark.parametrize("tp_impl,sp", [("fused", True), ("nccl", False), ("nccl", True)])
def test_native_tp2_matches_single_gpu_on_canonical_model(tp_impl, sp, tmp_path):
    path = _canonical(tmp_path)
    ref = _run(_canonical_step, 1, 1, 1, False, "auto", path, port=29713)[0]
    res = _run(_canonical_step, 2, 2, 1, sp, tp_impl, path, port=29714 + int(sp) + 2 * (tp_impl == "fused"))
    for r in res:
        assert abs(r["loss"] - ref["loss"]) < 2e-3 * ref["loss"], (r["loss"], ref["loss"])
    _check_against_full(res, ref, 2)


@NEED2
def test_native_pp2_matches_single_gpu_on_canonical_model(tmp_path):
    path = _canonical(tmp_path)
    ref = _run(_canonical_step, 1, 1, 1, False, "auto", path, port=29716)[0]
    res = _run(_canonical_step, 2, 1, 2, False, "auto", path, port=29725)
    assert res[0]["loss"] is None
    assert abs(res[1]["loss"] - ref["loss"]) < 2e-3 * ref["loss"], (res[1]["loss"], ref["loss"])
    # each stage returns its own parameters; together they cover the model
    assert set(res[0]["grads"]) | set(res[1]["grads"]) == set(ref["grads"])
    _check_against_full(res, ref, 1)


@NEED2
def test_fused_tp_matches_nccl_tp():
    """Collectives fused into the LN / GEMM kernels reproduce the NCCL sequence-parallel path."""
    fused = _run(_train, 2, 2, 1, True, "nccl", 3, 2, "fused", port=29717)
    nccl = _run(_train, 2, 2, 1, True, "nccl", 3, 2, "nccl", port=29718)
    for r in range(2):
        for a, b in zip(fused[r]["losses"], nccl[r]["losses"]):
            assert abs(a - b) < 2e-3 * abs(b), (fused[r]["losses"], nccl[r]["losses"])
        _assert_states_close(fused[r]["state"], nccl[r]["state"], tensor_rel=1e-2, model_rel=1e-3)


@NEED2
def test_fused_tp_poisoned_workspace_gives_identical_results():
    """Debug mode: every data region of the TP workspace is NaN-filled before each step.
    A kernel that read a gathered row or reduce-scatter slot before its producer wrote it
    in the same step would turn the loss into NaN; results must match the clean run instead
    (up to the order of floating-point reductions, which split-K and atomics leave open)."""
    clean = _run(_train, 2, 2, 1, True, "nccl", 2, 2, "fused", port=29719)
    poisoned = _run(_train, 2, 2, 1, True, "nccl", 2, 2, "fused", port=29720, env={"MMB_POISON_SYMM": "1"})
    for r in range(2):
        assert poisoned[r]["losses"][0] == clean[r]["losses"][0]           # first forward: no reductions differ
        for a, b in zip(poisoned[r]["losses"], clean[r]["losses"]):
            assert abs(a - b) <= 1e-4 * abs(b), (poisoned[r]["losses"], clean[r]["losses"])
        _assert_states_close(poisoned[r]["state"], clean[r]["state"], tensor_rel=1e-2)


@NEED2
def test_fused_tp_recompute_matches():
    """--recompute with the fused TP kernels: backward re-runs each layer's forward, including its
    all-gather pushes and reduce-scatter, so the workspace epochs and slots must still line up."""
    rc = _run(_train, 2, 2, 1, True, "nccl", 2, 2, "fused", True, port=29721)
    ref = _run(_train, 2, 2, 1, True, "nccl", 2, 2, "fused", False, port=29722)
    for r in range(2):
        assert rc[r]["losses"][0] == ref[r]["losses"][0]
        for a, b in zip(rc[r]["losses"], ref[r]["losses"]):
            assert abs(a - b) <= 1e-3 * abs(b), (rc[r]["losses"], ref[r]["losses"])
        _assert_states_close(rc[r]["state"], ref[r]["state"], tensor_rel=1e-2, model_rel=1e-3)


def _resume(rank, world, ckpt, phase):
    """Fused DP (dp=2): phase 0 trains 2 steps, saves, trains 2 more; phase 1 loads and trains 2."""
    from mini_megatron_b200.config import GPTConfig
    from mini_megatron_b200.training import TrainConfig, Trainer, synthetic_batch
    from mini_megatron_b200.utils.checkpoint import load_distributed_checkpoint, save_distributed_checkpoint
    cfg = TrainConfig(model=GPTConfig(**CFG), micro_batch_size=2, seq_len=256, dp_impl="fused", lr=1e-3,
                      warmup_steps=2, num_steps=20, bucket_mb=1.0)
    t = Trainer(cfg)
    dp_rank = t.mpu["dp_rank"]
    losses = []

    def run(steps):
        for s in steps:
            tok, lab = synthetic_batch(1, 2, 256, CFG["vocab_size"], seed=1000 * s + dp_rank)
            losses.append(t.train_step(tok, lab).item())
    if phase == 0:
        run(range(2))
        save_distributed_checkpoint(ckpt, *t.state_for_checkpoint(), 2, mpu=t.mpu)
        run(range(2, 4))
    else:
        step = load_distributed_checkpoint(ckpt, *t.state_for_checkpoint(), mpu=t.mpu, device="cuda")
        assert step == 2
        run(range(2, 4))
    state = {k: v.detach().float().cpu() for k, v in t.model.state_dict().items()}
    t.destroy()
    return {"losses": losses, "state": state}


@NEED2
def test_fused_dp_checkpoint_resume_continues_identically(tmp_path):
    """Every DP rank writes its own optimizer shard (the fused-DP moments are sharded), and a run
    resumed from the checkpoint continues with the same losses and parameters."""
    ckpt = str(tmp_path / "ckpt")
    full = _run(_resume, 2, ckpt, 0, port=29723)
    import json
    manifest = json.load(open(os.path.join(ckpt, "manifest.json")))
    assert manifest["sharded_optimizer"] and len([f for f in manifest["files"] if f.startswith("optim")]) == 2
    resumed = _run(_resume, 2, ckpt, 1, port=29724)
    # split-K weight gradients and the attention dQ are summed with reduce-adds in no fixed order, so
    # two runs agree to rounding, not bit for bit
    for r in range(2):
        for a, b in zip(resumed[r]["losses"], full[r]["losses"][2:]):
            assert abs(a - b) < 1e-4 * abs(b), (resumed[r]["losses"], full[r]["losses"])
        _assert_states_close(resumed[r]["state"], full[r]["state"])


NEED4 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 4, reason="needs 4 GPUs")


@NEED4
@pytest.mark.parametrize("tp,pp", [(2, 1), (1, 2)])
def test_fused_dp_composes_with_tp_and_pp(tp, pp):
    """dp = 2 beside TP2 (fused TP, sequence parallel: the DP buckets start after the LayerNorm
    gradients' TP reduction) or beside PP2 (1F1B; buckets start during the last microbatch's
    backward): the fused DP kernel gives the NCCL all-reduce path's losses and parameters."""
    micro = 2 if pp == 1 else 4
    fused = _run(_train, 4, tp, pp, tp > 1, "fused", 3, micro, port=29731 + 2 * pp)
    nccl = _run(_train, 4, tp, pp, tp > 1, "nccl", 3, micro, port=29732 + 2 * pp)
    for r in range(4):
        for a, b in zip(fused[r]["losses"], nccl[r]["losses"]):
            if b is not None:
                assert abs(a - b) < 1e-3 * abs(b), (fused[r]["losses"], nccl[r]["losses"])
        _assert_states_close(fused[r]["state"], nccl[r]["state"], tensor_rel=1e-2, model_rel=1e-3)


@NEED4
def test_fused_tp_with_pp_matches_nccl_tp():
    """TP2 x PP2: the first stage holds the embedding (rows written by their vocabulary owner,
    gradient rows read back over NVLink), the last stage the fused head; both must reproduce the
    NCCL sequence-parallel path of the same configuration."""
    fused = _run(_train, 4, 2, 2, True, "nccl", 3, 4, "fused", port=29741)
    nccl = _run(_train, 4, 2, 2, True, "nccl", 3, 4, "nccl", port=29742)
    for r in range(4):
        for a, b in zip(fused[r]["losses"], nccl[r]["losses"]):
            if b is not None:
                assert abs(a - b) < 2e-3 * abs(b), (fused[r]["losses"], nccl[r]["losses"])
        _assert_states_close(fused[r]["state"], nccl[r]["state"], tensor_rel=1e-2, model_rel=1e-3)
