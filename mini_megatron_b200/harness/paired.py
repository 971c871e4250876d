"""Paired (ABBA) summaries of two benchmark variants.

Benchmark bundles carry tags ``variant=<name>``, ``pair=<id>`` and
``condition=<what was measured>`` (plus optionally ``topology``).  A pair is
the two variants measured back to back; alternating their order from pair to
pair (ABBA) cancels drift of the host.  Only valid, successful,
non-profile bundles whose GPU preflight saw an idle GPU enter the summary;
dirty-tree bundles only when asked.  The report gives per-variant statistics
and the statistics of the per-pair ratio -- never a "best run".

Reference: experiments/summarize_paired_results.py:18-82.

    python -m mini_megatron_b200.harness.paired --results-dir results/runs --left ours --right reference
"""
from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path

from .bundle import validate


def load_bundles(results_dir, allow_dirty=False, topology=None, condition=None, metric="throughput_tok_s"):
    records = []
    for mpath in sorted(Path(results_dir).glob("*/manifest.json")):
        errors = validate(mpath.parent)
        if errors:
            raise ValueError(f"invalid run bundle {mpath.parent}: " + "; ".join(errors))
        manifest = json.loads(mpath.read_text(encoding="utf-8"))
        if manifest.get("kind") != "benchmark" or manifest.get("return_code") != 0:
            continue
        pre = manifest.get("gpu_preflight") or {}
        if pre.get("return_code") != 0 or pre.get("active_processes") != []:
            continue
        if not manifest.get("source_tree_clean") and not allow_dirty:
            continue
        tags = manifest.get("tags") or {}
        if topology is not None and tags.get("topology") != topology:
            continue
        if condition is not None and tags.get("condition") != condition:
            continue
        value = (manifest.get("metrics") or {}).get(metric)
        if not isinstance(value, (int, float)):
            continue
        env = json.loads((mpath.parent / "environment.json").read_text(encoding="utf-8"))
        records.append({"bundle": str(mpath.parent), metric: float(value), "throughput_tok_s": float(value),
                        "tags": tags, "run_id": manifest.get("run_id"),
                        "source_tree_clean": manifest.get("source_tree_clean"),
                        "git_commit": env.get("git_commit")})
    return records


def _stats(values):
    return {"count": len(values), "mean": statistics.mean(values), "median": statistics.median(values),
            "sample_stddev": statistics.stdev(values) if len(values) > 1 else None,
            "min": min(values), "max": max(values)}


def summarize(records, left, right, min_pairs=5, metric="throughput_tok_s"):
    by_pair = {}
    for rec in records:
        v, p = rec["tags"].get("variant"), rec["tags"].get("pair")
        if v in (left, right) and p:
            if v in by_pair.setdefault(p, {}):
                raise ValueError(f"pair {p} has two {v} samples")
            by_pair[p][v] = rec
    done = []
    for pair in sorted(by_pair):
        d = by_pair[pair]
        if left not in d or right not in d:
            continue
        lc, rc = d[left]["tags"].get("condition"), d[right]["tags"].get("condition")
        if not lc or lc != rc:
            raise ValueError(f"pair {pair} must have the same non-empty condition tag")
        done.append({"pair": pair, "left": d[left], "right": d[right],
                     "ratio": d[left][metric] / d[right][metric]})
    if not done:
        raise ValueError("no completed pairs; tag runs with variant=<name> and pair=<id>")
    if len(done) < min_pairs:
        raise ValueError(f"need at least {min_pairs} completed pairs, found {len(done)}")
    return {
        "metric": metric,
        "left_variant": left,
        "right_variant": right,
        "pairs": done,
        "left": _stats([x["left"][metric] for x in done]),
        "right": _stats([x["right"][metric] for x in done]),
        "paired_ratio_left_over_right": _stats([x["ratio"] for x in done]),
        "source_tree_clean": all(x["left"].get("source_tree_clean") and x["right"].get("source_tree_clean")
                                 for x in done),
        "git_commits": sorted({x["left"].get("git_commit") for x in done} | {x["right"].get("git_commit") for x in done}
                              - {None}),
        "interpretation": "A ratio above 1 favours the left variant, for the recorded configuration only.",
    }


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--results-dir", default="results/runs")
    ap.add_argument("--left", default="ours")
    ap.add_argument("--right", default="reference")
    ap.add_argument("--metric", default="throughput_tok_s")
    ap.add_argument("--min-pairs", type=int, default=5)
    ap.add_argument("--allow-dirty", action="store_true")
    ap.add_argument("--topology")
    ap.add_argument("--condition")
    ap.add_argument("--output")
    args = ap.parse_args(argv)
    if args.min_pairs < 1:
        ap.error("--min-pairs must be positive")
    try:
        rep = summarize(load_bundles(args.results_dir, args.allow_dirty, args.topology, args.condition, args.metric),
                        args.left, args.right, args.min_pairs, args.metric)
    except ValueError as exc:
        ap.error(str(exc))
    rep["selection"] = {"results_dir": args.results_dir, "topology": args.topology, "condition": args.condition,
                        "allow_dirty": args.allow_dirty}
    text = json.dumps(rep, indent=2, sort_keys=True)
    print(text)
    if args.output:
        out = Path(args.output)
        if out.exists():
            ap.error(f"refusing to overwrite aggregate: {out}")
        out.parent.mkdir(parents=True, exist_ok=True)
        out.write_text(text + "\n", encoding="utf-8")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
