"""Frozen conclusions built from checksummed evidence, never rewritten.

* ``gate_windows`` -- combine parity reports measured on several independent
  batch windows (``OFFSET:PATH`` each) into one conclusion: the gate holds
  only if it holds on every window, and the original per-tensor view is
  always reported beside any calibrated view.
* ``profile_index`` -- index the profile bundles of two implementations for
  one topology by path, size and SHA-256; it contains no timing
  interpretation (profiles are diagnostics, not throughput samples).

Both refuse to overwrite an existing output.

Reference: experiments/write_fair_pp_conclusion.py:15-97, experiments/summarize_fair_pp_gate_windows.py,
experiments/summarize_fair_pp_profiles.py:37-81.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

from .bundle import sha256_file, validate
from .parity import GATES, evaluate


def _write_new(path, obj):
    path = Path(path)
    if path.exists():
        raise ValueError(f"refusing to overwrite: {path}")
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps(obj, indent=2, sort_keys=True) + "\n", encoding="utf-8")


def gate_windows(windows, gate_name="bf16", min_windows=3, output=None) -> dict:
    """``windows``: [(offset, path to a harness.parity report)]."""
    if len(windows) < min_windows:
        raise ValueError(f"at least {min_windows} independent windows are required")
    offsets = [o for o, _ in windows]
    if len(set(offsets)) != len(offsets):
        raise ValueError("window offsets must be distinct")
    rows = []
    for off, path in sorted(windows):
        path = Path(path).resolve()
        rep = json.loads(path.read_text(encoding="utf-8"))
        per_tensor = evaluate(rep, dict(GATES["fp32"]))
        chosen = evaluate(rep, GATES[gate_name])
        rows.append({"offset": off, "source_path": str(path), "source_sha256": sha256_file(path),
                     "original_per_tensor_checks": per_tensor, "gate_checks": chosen})
    result = {"schema_version": 1, "gate_name": gate_name, "gate": GATES[gate_name],
              "original_per_tensor_gate_passed_all_windows": all(r["original_per_tensor_checks"]["passed"]
                                                                 for r in rows),
              "gate_passed_all_windows": all(r["gate_checks"]["passed"] for r in rows),
              "windows": rows,
              "caveat": "A gate other than the original per-tensor one is reported beside it, never instead of it."}
    result["status"] = "gate_passed" if result["gate_passed_all_windows"] else "gate_failed"
    if output:
        _write_new(output, result)
    return result


def profile_index(bundles: dict, topology: str, output=None) -> dict:
    """``bundles``: {implementation: profile bundle dir}."""
    impls = {}
    for name, b in bundles.items():
        b = Path(b).resolve()
        errs = validate(b)
        if errs:
            raise ValueError(f"{name}: invalid bundle: " + "; ".join(errs))
        manifest = json.loads((b / "manifest.json").read_text(encoding="utf-8"))
        if manifest.get("kind") not in ("profile", "multi_rank_profile"):
            raise ValueError(f"{name} is not a profile bundle")
        if manifest.get("return_code") != 0:
            raise ValueError(f"{name} profile returned non-zero")
        files = sorted(p for p in (b / "profile").rglob("*") if p.is_file())
        impls[name] = {"bundle": str(b), "manifest_sha256": sha256_file(b / "manifest.json"),
                       "files": [{"relative_path": str(p.relative_to(b)), "size_bytes": p.stat().st_size,
                                  "sha256": sha256_file(p)} for p in files]}
    result = {"schema_version": 1, "topology": topology, "status": "profile_index_complete",
              "claim_scope": "Profiler evidence only; never a throughput sample.", "implementations": impls}
    if output:
        _write_new(output, result)
    return result


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("gate-windows")
    g.add_argument("--window", action="append", required=True, metavar="OFFSET:PATH")
    g.add_argument("--gate", default="bf16", choices=sorted(GATES))
    g.add_argument("--output", required=True)
    p = sub.add_parser("profile-index")
    p.add_argument("--bundle", action="append", required=True, metavar="IMPL=DIR")
    p.add_argument("--topology", required=True)
    p.add_argument("--output", required=True)
    args = ap.parse_args(argv)
    try:
        if args.cmd == "gate-windows":
            wins = []
            for w in args.window:
                off, sep, path = w.partition(":")
                if not sep or not off.isdecimal():
                    ap.error("--window must be OFFSET:PATH")
                wins.append((int(off), path))
            res = gate_windows(wins, args.gate, output=args.output)
        else:
            bundles = dict(b.split("=", 1) for b in args.bundle)
            res = profile_index(bundles, args.topology, output=args.output)
    except ValueError as exc:
        ap.error(str(exc))
    print(json.dumps(res, indent=2, sort_keys=True))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
