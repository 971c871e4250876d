"""bench.py's command-line contract (CPU: parsing and config tables only)."""
import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _parse(mod, argv, monkeypatch):
    monkeypatch.setattr(sys, "argv", ["bench.py"] + argv)
    return mod.parse()


def test_defaults_are_the_headline_config(monkeypatch):
    b = _bench()
    a = _parse(b, [], monkeypatch)
    assert (a.gpus, a.steps, a.warmup, a.impl) == (1, 20, 3, "ours")
    assert a.warmup >= 3
    assert (a.tp, a.pp, a.dp, a.micro_batch_size, a.seq_len, a.num_microbatches) == (1, 1, 1, 16, 1024, 1)
    assert a.model == dict(b.MODEL, max_seq_len=1024) and a.model["vocab_size"] == 50257
    assert b.parallelism_name(a) == "dp1"


@pytest.mark.parametrize("config,gpus,expect", [
    ("gpt125m-dp", 8, "dp8"),
    ("gpt125m-tp2pp2", 8, "tp2pp2dp2-sp"),
    ("gpt1.3b-tp8sp", 8, "tp8-sp"),
    ("gpt6.7b-tp4pp2", 8, "tp4pp2-sp"),
])
def test_baseline_configs(monkeypatch, config, gpus, expect):
    b = _bench()
    a = _parse(b, ["--config", config, "--gpus", str(gpus)], monkeypatch)
    assert a.tp * a.pp * a.dp == gpus
    assert b.parallelism_name(a) == expect


def test_config_shapes_match_baseline_json(monkeypatch):
    b = _bench()
    c = b.CONFIGS
    assert (c["gpt125m-tp2pp2"]["mb"], c["gpt125m-tp2pp2"]["m"], c["gpt125m-tp2pp2"]["seq"]) == (8, 8, 1024)
    assert (c["gpt1.3b-tp8sp"]["mb"], c["gpt1.3b-tp8sp"]["seq"]) == (4, 2048)
    assert (c["gpt6.7b-tp4pp2"]["mb"], c["gpt6.7b-tp4pp2"]["m"], c["gpt6.7b-tp4pp2"]["seq"]) == (2, 16, 2048)
    assert b.M_1_3B["hidden_size"] == 2048 and b.M_6_7B["num_layers"] == 32


def test_gpu_count_must_divide(monkeypatch):
    b = _bench()
    with pytest.raises(SystemExit):
        _parse(b, ["--config", "gpt125m-tp2pp2", "--gpus", "2"], monkeypatch)
