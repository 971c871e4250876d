"""Experiment harness: bundles, paired summaries, kernel classification, contracts,
parity gates, frozen artifacts, fair benchmark, queue, campaign ledger, conclusions.

CPU only.  Mirrors the reference's harness tests (tests/test_experiment_artifacts.py,
tests/test_fair_parallel_campaign.py) and adds end-to-end checks against the
reference's own modules where its sources are present.
"""
import json
import subprocess
import sys
from argparse import Namespace
from pathlib import Path

import pytest
import torch

from mini_megatron_b200.harness import bundle as B
from mini_megatron_b200.harness import campaign, conclusions, contract, kernels, legacy, paired, parity, queue
from mini_megatron_b200.harness.artifacts import freeze, load_chunk, verify

REPO = Path(__file__).resolve().parents[1]
HAVE_REF = (REPO / "baseline" / "_ref" / "model" / "transformer.py").exists()
TINY = dict(num_layers=2, hidden_size=32, num_attention_heads=4, ffn_hidden_size=64, max_seq_len=16, vocab_size=100)


def _bundle(tmp_path, name="run", tags=None, metrics=None, preflight=None, clean=True):
    b = Path(tmp_path) / name
    b.mkdir()
    m = {"schema_version": 1, "run_id": name, "kind": "benchmark", "claim_scope": "test",
         "target_command": ["python", "main.py"], "executed_command": ["python", "main.py"],
         "started_at_utc": "2026-01-01T00:00:00+00:00", "finished_at_utc": "2026-01-01T00:00:01+00:00",
         "elapsed_wall_seconds": 1.0, "return_code": 0, "metrics": metrics or {"throughput_tok_s": 100.0},
         "environment_file": "environment.json", "tags": tags or {}, "source_tree_clean": clean,
         "gpu_preflight": preflight if preflight is not None else {"return_code": 0, "active_processes": []}}
    (b / "manifest.json").write_text(json.dumps(m))
    (b / "metrics.json").write_text(json.dumps(m["metrics"]))
    (b / "environment.json").write_text(json.dumps({"git_commit": "abc"}))
    (b / "stdout.log").write_text("ok")
    (b / "stderr.log").write_text("")
    (b / "command.txt").write_text("python main.py\n")
    B.write_checksums(b)
    return b


# ----------------------------------------------------------------------------- bundles
def test_parse_metrics_reads_report_lines_and_bench_json():
    out = ("Throughput:      60,718 tok/s\nPeak memory:     3.88 GB/GPU\nMFU:             42.49%\n"
           "Final loss:      9.8482\n")
    assert B.parse_metrics(out) == {"throughput_tok_s": 60718.0, "peak_memory_gb": 3.88, "mfu_percent": 42.49,
                                    "final_loss": 9.8482}
    js = json.dumps({"metric": "m", "value": 813537.1, "unit": "tok/s", "ms_per_step": 20.1, "n_gpus": 1,
                     "e2e": {"value": 808582.8}})
    m = B.parse_metrics("noise\n" + js + "\n")
    assert m["throughput_tok_s"] == 813537.1 and m["e2e_value"] == 808582.8 and m["ms_per_step"] == 20.1


def test_parse_compute_processes_ignores_idle_messages():
    assert B.parse_compute_processes("No running processes found\n") == []
    assert B.parse_compute_processes("123, python, GPU-abc\n\n") == ["123, python, GPU-abc"]


def test_valid_bundle_passes_and_tampering_fails(tmp_path):
    b = _bundle(tmp_path)
    assert B.validate(b) == []
    (b / "stdout.log").write_text("tampered")
    assert any("checksum mismatch: stdout.log" in e for e in B.validate(b))


def test_uncovered_file_fails_validation(tmp_path):
    b = _bundle(tmp_path)
    (b / "extra.txt").write_text("x")
    assert any("not covered" in e for e in B.validate(b))


def test_run_bundle_end_to_end(tmp_path):
    cmd = [sys.executable, "-c", "print('Throughput:      1,234 tok/s'); print('Final loss:      2.5')"]
    b, m = B.run_bundle(cmd, "smoke", tmp_path, tags={"variant": "ours"}, allow_dirty=True, allow_active_gpus=True)
    assert m["return_code"] == 0 and m["metrics"] == {"throughput_tok_s": 1234.0, "final_loss": 2.5}
    assert B.validate(b) == []
    with pytest.raises(ValueError):
        B.run_bundle(cmd, "bad name!", tmp_path, allow_dirty=True, allow_active_gpus=True)


# ----------------------------------------------------------------------------- kernels
def test_kernel_analysis_keeps_generic_kernels_unclassified():
    rows = [{"name": "mmb::adamw_kernel(float*)", "total_time_ns": 30, "instances": 2},
            {"name": "void mmb::gemm_bf16_sm100<256, false, true, 0>", "total_time_ns": 50, "instances": 3},
            {"name": "vectorized_elementwise_kernel", "total_time_ns": 20, "instances": 4}]
    r = kernels.analyze(rows)
    assert r["categories"]["fused_adamw"]["percent_kernel_time"] == 30.0
    assert r["categories"]["gemm"]["percent_kernel_time"] == 50.0
    assert r["categories"]["unclassified"]["percent_kernel_time"] == 20.0


def test_kernel_classifier_names_fused_collectives():
    assert kernels.classify("mmb::dp_rs_adamw_ag_kernel(...)") == "fused_dp_optimizer"
    assert kernels.classify("mmb::tp_rs_reduce_kernel(...)") == "fused_tp_collective"
    assert kernels.classify("void mmb::attn::flash_bwd_kernel<64>") == "attention"
    assert kernels.classify("ncclDevKernel_AllReduce_Sum_f32") == "nccl"


def test_ncu_launch_list_summary(tmp_path):
    csv = tmp_path / "launches.csv"
    csv.write_text('==PROF== noise\n"ID","Kernel Name","Metric Name","Metric Unit","Metric Value"\n'
                   '"0","k1","gpu__time_duration.sum","us","1.5"\n"1","k1","gpu__time_duration.sum","us","2.5"\n'
                   '"2","k2","gpu__time_duration.sum","ns","700"\n')
    rows = B.ncu_kernel_summary(csv)
    assert rows[0] == {"name": "k1", "total_time_ns": 4000, "instances": 2}
    assert rows[1] == {"name": "k2", "total_time_ns": 700, "instances": 1}


# ----------------------------------------------------------------------------- contracts
def test_qkv_conversion_round_trips():
    w = torch.arange(3 * 8 * 8, dtype=torch.float32).reshape(24, 8)
    mc = contract.qkv_to_mcore(w, 2)
    assert not torch.equal(w, mc)
    assert torch.equal(contract.qkv_from_mcore(mc, 2), w)
    # head 0's Q rows come first, then head 0's K rows
    assert torch.equal(mc[:4], w[:4]) and torch.equal(mc[4:8], w[8:12])


@pytest.mark.parametrize("name", ["decoder.layers.0.attn.qkv.weight", "decoder.layers.0.mlp.fc1.weight",
                                  "decoder.layers.0.attn.o.weight", "lm_head.weight", "ln_f.weight"])
def test_tp_shard_round_trip(name):
    shape = (24, 8) if "ln_f" not in name else (8,)
    full = torch.randn(shape)
    shards = [contract.tp_shard(full, name, 2, r) for r in range(2)]
    assert torch.equal(contract.tp_unshard(shards, name), full)


def test_qkv_shard_gives_matching_heads():
    # rows [Q0 Q1 | K0 K1 | V0 V1] with 2 heads of dim 2: rank 0 must get Q0, K0, V0
    full = torch.arange(12, dtype=torch.float32).repeat_interleave(1).reshape(12, 1)
    s0 = contract.tp_shard(full, "x.attn.qkv.weight", 2, 0)
    assert s0.flatten().tolist() == [0, 1, 4, 5, 8, 9]


def test_mcore_name_map_and_stage_plan_cover_every_parameter():
    names = contract.full_parameter_names(TINY)
    pairs = contract.mcore_name_pairs(TINY)
    assert [a for a, _ in pairs] and sorted(a for a, _ in pairs) == sorted(names)
    plan = [n for r in range(2) for n, _ in contract.stage_parameter_plan(TINY, r, 2)]
    assert sorted(plan) == sorted(names)
    assert ("decoder.layers.1.ln1.weight", "decoder_layers.0.ln1.weight") in contract.stage_parameter_plan(TINY, 1, 2)


def test_vocab_padding_round_trip():
    st = {"embedding.token_embedding.weight": torch.randn(100, 4), "lm_head.weight": torch.randn(100, 4)}
    padded = contract.from_reference_state(st, 128)
    assert padded["lm_head.weight"].shape == (128, 4) and padded["lm_head.weight"][100:].abs().sum() == 0
    back = contract.to_reference_state(padded, 100)
    assert torch.equal(back["lm_head.weight"], st["lm_head.weight"])


# ----------------------------------------------------------------------------- paired summaries
def test_paired_summary_reports_ratios():
    recs = [{"throughput_tok_s": 120.0, "tags": {"variant": "ours", "pair": "01", "condition": "125m"}},
            {"throughput_tok_s": 100.0, "tags": {"variant": "reference", "pair": "01", "condition": "125m"}},
            {"throughput_tok_s": 110.0, "tags": {"variant": "ours", "pair": "02", "condition": "125m"}},
            {"throughput_tok_s": 100.0, "tags": {"variant": "reference", "pair": "02", "condition": "125m"}}]
    r = paired.summarize(recs, "ours", "reference", min_pairs=2)
    assert r["paired_ratio_left_over_right"]["count"] == 2
    assert r["paired_ratio_left_over_right"]["mean"] == pytest.approx(1.15)
    with pytest.raises(ValueError, match="at least 3"):
        paired.summarize(recs, "ours", "reference", min_pairs=3)


def test_paired_summary_rejects_mismatched_conditions():
    recs = [{"throughput_tok_s": 120.0, "tags": {"variant": "ours", "pair": "01", "condition": "125m"}},
            {"throughput_tok_s": 100.0, "tags": {"variant": "reference", "pair": "01", "condition": "1b"}}]
    with pytest.raises(ValueError, match="same non-empty condition"):
        paired.summarize(recs, "ours", "reference", min_pairs=1)


def test_load_bundles_filters_busy_gpus_and_dirty_trees(tmp_path):
    _bundle(tmp_path, "a", tags={"variant": "ours", "pair": "01", "condition": "c"})
    _bundle(tmp_path, "b", tags={"variant": "ours", "pair": "02", "condition": "c"},
            preflight={"return_code": 0, "active_processes": ["123, python, GPU-abc"]})
    _bundle(tmp_path, "c", tags={"variant": "ours", "pair": "03", "condition": "c"}, clean=False)
    recs = paired.load_bundles(tmp_path)
    assert [r["tags"]["pair"] for r in recs] == ["01"]
    assert len(paired.load_bundles(tmp_path, allow_dirty=True)) == 2


# ----------------------------------------------------------------------------- queue and campaign
def test_abba_schedule_is_fixed_and_balanced():
    s = queue.abba_schedule("ours", "reference", 5)
    assert [e["variant"] for e in s] == ["ours", "reference", "reference", "ours", "ours", "reference", "reference",
                                         "ours", "ours", "reference"]
    assert [e["pair"] for e in s] == ["01", "01", "02", "02", "03", "03", "04", "04", "05", "05"]


def test_queue_stops_at_first_failure(tmp_path):
    calls = []

    def runner(cmd, name, results_dir, tags, allow_dirty=False):
        calls.append(name)
        return Path(tmp_path) / name, {"return_code": 1 if len(calls) == 3 else 0}

    with pytest.raises(RuntimeError, match="failed"):
        queue.run_queue({"ours": ["a"], "reference": ["b"]}, "tp1", "c", 5, tmp_path, runner=runner,
                        preflight=lambda: None)
    assert len(calls) == 3


def test_queue_requires_idle_gpus():
    with pytest.raises(RuntimeError, match="compute processes"):
        queue.require_idle({"return_code": 0, "active_processes": ["1, python, GPU-x"]})


def test_campaign_records_hashes_and_detects_tampering(tmp_path):
    d = tmp_path / "camp"
    campaign.init(d, "camp-test")
    src = tmp_path / "artifact.json"
    src.write_text(json.dumps({"ok": True}))
    campaign.record(d, "artifact", "tp2-pp1-dp1", src)
    res = campaign.validate(d)
    assert res["valid"] and res["topologies"]["tp2-pp1-dp1"]["missing_publishable_evidence"] == [
        "benchmark_summary", "numerical_parity", "profile"]
    for kind in ("numerical_parity", "benchmark_summary", "profile"):
        campaign.record(d, kind, "tp2-pp1-dp1", src)
    assert campaign.validate(d)["topologies"]["tp2-pp1-dp1"]["unconditional_publishable"]
    src.write_text(json.dumps({"ok": False}))
    res = campaign.validate(d)
    assert not res["valid"] and any("checksum mismatch" in e for e in res["errors"])
    with pytest.raises(ValueError):
        campaign.init(d, "again")
    with pytest.raises(ValueError, match="unknown topology"):
        campaign.record(d, "artifact", "tp9", src)


# ----------------------------------------------------------------------------- artifacts, parity, fair bench
def test_artifacts_freeze_verify_and_refuse_overwrite(tmp_path):
    d = tmp_path / "art"
    m = freeze(d, TINY, tp=2, pp=1, num_batches=4, batch_size=2)
    assert verify(d) == [] and m["padded_vocab"] == 256
    st0, _ = load_chunk(d, "ours", 0, 2, 1)
    st1, _ = load_chunk(d, "ours", 1, 2, 1)
    full = torch.load(d / "source_full.pt", weights_only=True)["state_dict"]
    n = "decoder.layers.0.attn.qkv.weight"
    assert torch.equal(contract.tp_unshard([st0[n], st1[n]], n), full[n])
    assert st0["lm_head.weight"].shape[0] == 128          # padded vocabulary, split over tp=2
    ref0, _ = load_chunk(d, "reference", 0, 2, 1)
    assert ref0["lm_head.weight"].shape[0] == 50           # the reference's exact-vocabulary shard
    data = torch.load(d / "next_token_batches.pt", weights_only=True)
    assert torch.equal(data["labels"][..., :-1], data["input_ids"][..., 1:]) and (data["labels"][..., -1] == -100).all()
    with pytest.raises(ValueError):
        freeze(d, TINY)
    (d / "source_full.pt").write_bytes(b"x")
    assert verify(d) and pytest.raises(ValueError, load_chunk, d, "ours", 0, 2, 1)


def test_parity_gate_evaluation():
    rep = {"initial_parameters": {"global_max_abs": 0.0}, "loss_abs": 1e-5, "logits_relative_l2": 1e-4,
           "gradients": {"worst_relative_l2": {"relative_l2": 4e-4}, "global_relative_l2": 1e-4},
           "parameters_after_one_step": {"worst_relative_l2": {"relative_l2": 2e-4}, "global_relative_l2": 5e-5,
                                         "global_max_abs": 1e-4}}
    assert not parity.evaluate(rep, parity.GATES["fp32"])["passed"]          # per-tensor param 2e-4 > 1e-4
    assert parity.evaluate(rep, parity.GATES["pp-calibrated"])["passed"]     # global view passes


@pytest.mark.skipif(not HAVE_REF, reason="reference sources not present")
def test_parity_ours_vs_reference_cpu():
    from mini_megatron_b200.config import PRESETS
    c = PRESETS["tiny"]
    mc = dict(num_layers=c.num_layers, hidden_size=c.hidden_size, num_attention_heads=c.num_attention_heads,
              ffn_hidden_size=c.ffn_hidden_size, max_seq_len=c.max_seq_len, vocab_size=c.vocab_size)
    torch.manual_seed(0)
    dev = torch.device("cpu")
    a, b = parity.build_impl("reference", mc, dev, False), parity.build_impl("ours", mc, dev, False)
    tok, lab, mask = parity.fixed_batch(2, mc["max_seq_len"], mc["vocab_size"], 1)
    rep = parity.run_parity(a, b, mc, tok, lab, mask, dev)
    assert parity.evaluate(rep, parity.GATES["fp32"])["passed"], rep


@pytest.mark.skipif(not HAVE_REF, reason="reference sources not present")
def test_fair_bench_same_losses_as_reference_cpu(tmp_path):
    d = tmp_path / "art"
    freeze(d, TINY, num_batches=8, batch_size=2)
    losses = {}
    for impl in ("ours", "reference"):
        r = subprocess.run([sys.executable, "-m", "mini_megatron_b200.harness.fair_bench", "--implementation", impl,
                            "--artifact-dir", str(d), "--num-updates", "2", "--warmup-updates", "1",
                            "--microbatches-per-update", "2", "--report-losses", "--device", "cpu"],
                           capture_output=True, text=True, timeout=600, cwd=REPO)
        assert r.returncode == 0, r.stderr[-2000:]
        rep = json.loads(next(l for l in r.stdout.splitlines() if l.startswith("{")))
        assert B.parse_metrics(r.stdout)["throughput_tok_s"] > 0
        losses[impl] = rep["losses"]
    assert len(losses["ours"]) == 3
    assert losses["ours"] == pytest.approx(losses["reference"], rel=1e-5, abs=1e-5)


# ----------------------------------------------------------------------------- conclusions and legacy
def test_gate_windows_conclusion(tmp_path):
    rep = {"initial_parameters": {"global_max_abs": 0.0}, "loss_abs": 0.0, "logits_relative_l2": 0.0,
           "gradients": {"worst_relative_l2": {"relative_l2": 0.0}, "global_relative_l2": 0.0},
           "parameters_after_one_step": {"worst_relative_l2": {"relative_l2": 0.0}, "global_relative_l2": 0.0,
                                         "global_max_abs": 0.0}}
    wins = []
    for off in (0, 8, 16):
        p = tmp_path / f"w{off}.json"
        p.write_text(json.dumps(rep))
        wins.append((off, p))
    with pytest.raises(ValueError, match="at least 3"):
        conclusions.gate_windows(wins[:2])
    out = tmp_path / "conclusion.json"
    res = conclusions.gate_windows(wins, "bf16", output=out)
    assert res["status"] == "gate_passed" and res["original_per_tensor_gate_passed_all_windows"]
    with pytest.raises(ValueError, match="overwrite"):
        conclusions.gate_windows(wins, "bf16", output=out)


def test_synthetic_and_identity_datasets(tmp_path):
    p = tmp_path / "syn.pt"
    d = legacy.save_synthetic(p, num_steps=3, B=2, S=8, effective_vocab=10)
    assert torch.equal(d["labels"], (d["input_ids"] + 1) % 10)
    ident = legacy.make_identity(p, tmp_path / "id.pt")
    assert torch.equal(ident["labels"], ident["input_ids"])


def test_loss_parsing_and_curve_record():
    out = "step    1 | loss 6.9000\nstep    2 | loss 6.5000\nThroughput:      1,000 tok/s\nMFU:             1.50%\n"
    assert legacy.parse_losses(out) == [(1, 6.9), (2, 6.5)]
    assert legacy.parse_report(out) == {"throughput": 1000.0, "mfu": 1.5}
    rec = legacy.loss_curve_record("t", "m", "d", {}, {"ours": [(1, 6.9)]}, "c")
    assert rec["results"]["ours"] == [{"step": 1, "loss": 6.9}]


# ----------------------------------------------------------------------------- command lines
def test_command_lines_end_to_end(tmp_path, capsys, monkeypatch):
    """The harness modules' CLIs: bundle run/validate, paired summary, campaign init/record/validate,
    kernel classification, artifacts, legacy datasets and conclusions."""
    from mini_megatron_b200.harness import artifacts as A
    # no nvidia-smi here: record the preflight of an idle GPU host so the bundles qualify for pairing
    monkeypatch.setattr(B, "gpu_preflight", lambda: {"command": ["nvidia-smi"], "return_code": 0, "stdout": "",
                                                      "stderr": "", "active_processes": []})
    from mini_megatron_b200.harness import kernels as KN
    results = tmp_path / "runs"
    cmd = [sys.executable, "-c", "print('Throughput:      2,000 tok/s')"]
    for pair, order in (("01", ("ours", "reference")), ("02", ("reference", "ours"))):
        for v in order:
            rc = B.main(["run", "--name", f"p{pair}-{v}", "--results-dir", str(results), "--tag", f"variant={v}",
                         "--tag", f"pair={pair}", "--tag", "condition=c", "--allow-dirty", "--allow-active-gpus",
                         "--"] + cmd)
            assert rc == 0
    bundles = sorted(results.iterdir())
    assert len(bundles) == 4 and B.main(["validate", str(bundles[0])]) == 0
    capsys.readouterr()
    out = tmp_path / "paired.json"
    assert paired.main(["--results-dir", str(results), "--min-pairs", "2", "--allow-dirty", "--output",
                        str(out)]) == 0
    rep = json.loads(out.read_text())
    assert rep["paired_ratio_left_over_right"]["mean"] == 1.0
    camp = tmp_path / "camp"
    assert campaign.main(["init", "--campaign-dir", str(camp), "--campaign-id", "t"]) == 0
    assert campaign.main(["record", "--campaign-dir", str(camp), "--kind", "benchmark_summary", "--topology",
                          "tp1-pp1-dp1", "--source", str(out)]) == 0
    assert campaign.main(["validate", "--campaign-dir", str(camp)]) == 0
    rows = tmp_path / "rows.json"
    rows.write_text(json.dumps([{"name": "mmb::adamw_kernel", "total_time_ns": 5, "instances": 1}]))
    assert KN.main([str(rows)]) == 0
    assert A.main(["--output-dir", str(tmp_path / "art"), "--preset", "tiny", "--batches", "2", "--batch-size",
                   "1"]) == 0
    assert legacy.main(["synthetic", str(tmp_path / "syn.pt"), "--num-steps", "2", "--batch-size", "1",
                        "--seq-len", "8"]) == 0
    assert legacy.main(["identity", str(tmp_path / "syn.pt"), str(tmp_path / "id.pt")]) == 0
