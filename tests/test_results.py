"""Committed result records stay parseable and consistent (no GPU needed).

Mirrors the reference's results-schema test (tests/test_identity_results.py):
the loss-curve file exists, has the expected structure, monotonic integer steps
and non-negative losses.  In addition the two implementations' curves, which
were produced from identical frozen weights and batches, must agree.
"""
import json
from pathlib import Path

RESULTS = Path(__file__).resolve().parents[1] / "results"
CURVES = RESULTS / "convergence_tiny_cpu.json"


def _load():
    return json.loads(CURVES.read_text())


def test_curve_file_exists_and_has_schema():
    assert CURVES.exists(), CURVES
    d = _load()
    for k in ("task", "model", "data", "config", "results", "conclusion"):
        assert k in d
    assert set(d["results"]) == {"mini_megatron_b200", "reference_mini_megatron"}


def test_curves_have_monotonic_steps_and_valid_losses():
    for name, curve in _load()["results"].items():
        assert len(curve) > 10, name
        steps = [p["step"] for p in curve]
        losses = [p["loss"] for p in curve]
        assert all(isinstance(s, int) and s > 0 for s in steps)
        assert steps == sorted(steps) and len(set(steps)) == len(steps)
        assert all(isinstance(x, (int, float)) and x >= 0 for x in losses)


def test_both_implementations_learn_and_agree():
    r = _load()["results"]
    ours = [p["loss"] for p in r["mini_megatron_b200"]]
    ref = [p["loss"] for p in r["reference_mini_megatron"]]
    assert ours[-1] < ours[0] - 5.0 and ref[-1] < ref[0] - 5.0
    assert max(abs(a - b) for a, b in zip(ours, ref)) < 1e-4


def test_reference_hang_records_are_kept():
    logs = sorted((RESULTS / "logs").glob("reference_tp_pp_hang_*.txt"))
    assert logs and all("timeout" in p.read_text().lower() for p in logs)
