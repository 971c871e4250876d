"""Sequential ABBA benchmark queue.

Runs a fixed, pre-declared schedule of benchmark bundles one at a time:
``pairs`` pairs of two variants, the order alternating from pair to pair
(A B, B A, A B, ...), so neither variant always gets the colder or hotter
host.  Before every run the selected GPUs must be idle (no compute process,
read from nvidia-smi); the queue stops at the first failing run and never
retries or skips silently.  Each run becomes a ``harness.bundle`` bundle
tagged ``variant``, ``pair``, ``pair_ordinal``, ``topology`` and
``condition``, which is what ``harness.paired`` consumes.

    python -m mini_megatron_b200.harness.queue --topology tp1-pp1-dp2 --condition gpt125m-b16-s1024 \\
        --variant ours="torchrun ... bench.py --gpus 2" --variant reference="torchrun ... bench.py --gpus 2 --impl reference"

Reference: experiments/run_tp2_preliminary_queue.py, experiments/run_fair_pp_queue.py:20-119,
experiments/fair_parallel_campaign.py:65-75 (schedule).
"""
from __future__ import annotations

import argparse
import json
import shlex
from pathlib import Path

from .bundle import DEFAULT_RESULTS, gpu_preflight, run_bundle


def abba_schedule(left: str, right: str, pairs: int = 5) -> list:
    """[{pair, variant, pair_ordinal, execution_ordinal}] with the order alternating per pair."""
    out = []
    for p in range(1, pairs + 1):
        order = (left, right) if p % 2 else (right, left)
        for ordinal, v in enumerate(order, start=1):
            out.append({"pair": f"{p:02d}", "variant": v, "pair_ordinal": ordinal, "execution_ordinal": len(out) + 1})
    return out


def require_idle(preflight=None):
    pre = preflight if preflight is not None else gpu_preflight()
    if pre.get("return_code") not in (0, None):
        raise RuntimeError("nvidia-smi failed: " + str(pre.get("stderr", "")).strip())
    if pre.get("active_processes"):
        raise RuntimeError("GPU preflight found compute processes: " + "; ".join(pre["active_processes"]))


def run_queue(commands: dict, topology: str, condition: str, pairs=5, results_dir=DEFAULT_RESULTS,
              allow_dirty=False, runner=run_bundle, preflight=require_idle) -> list:
    """Run the ABBA schedule; returns the bundle paths; raises at the first failure."""
    if len(commands) != 2:
        raise ValueError("exactly two variants are needed")
    left, right = list(commands)
    done = []
    for item in abba_schedule(left, right, pairs):
        preflight()
        name = f"{topology}-p{item['pair']}-{item['variant']}"
        tags = {"variant": item["variant"], "pair": item["pair"], "pair_ordinal": str(item["pair_ordinal"]),
                "topology": topology, "condition": condition}
        bundle, manifest = runner(commands[item["variant"]], name, results_dir, tags, allow_dirty=allow_dirty)
        if manifest["return_code"] != 0:
            raise RuntimeError(f"run {name} failed with exit code {manifest['return_code']}: {bundle}")
        done.append(str(bundle))
    return done


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--variant", action="append", required=True, metavar="NAME=COMMAND")
    ap.add_argument("--topology", required=True)
    ap.add_argument("--condition", required=True)
    ap.add_argument("--pairs", type=int, default=5)
    ap.add_argument("--results-dir", default=str(DEFAULT_RESULTS))
    ap.add_argument("--allow-dirty", action="store_true")
    args = ap.parse_args(argv)
    commands = {}
    for v in args.variant:
        name, sep, cmd = v.partition("=")
        if not sep or not name or not cmd:
            ap.error("--variant must be NAME=COMMAND")
        commands[name] = shlex.split(cmd)
    try:
        bundles = run_queue(commands, args.topology, args.condition, args.pairs, Path(args.results_dir),
                            args.allow_dirty)
    except (RuntimeError, ValueError) as exc:
        print(json.dumps({"status": "stopped", "error": str(exc)}))
        return 1
    print(json.dumps({"status": "complete", "bundles": bundles}, indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
