"""Per-rank kernel profiles of a multi-rank job.

Wraps a Python training script so that every torchrun child profiles its own
CUDA activity with the PyTorch profiler (CUPTI) and writes, under
``--out``, ``rank{R}_kernels.json`` (per-kernel total time and launch count,
the row format ``harness.kernels`` classifies) and, with ``--trace``, a
Chrome trace ``rank{R}_trace.json``.  ``ncu`` replays kernels and must never
wrap a multi-rank command, so this is the per-rank tool for multi-GPU jobs.

    python -m torch.distributed.run --nproc-per-node 2 -m mini_megatron_b200.harness.rank_profile \\
        --out prof/ -- main.py --tp 2 --num-steps 5

Profiled durations are for shares only, never throughput claims.

Reference: experiments/profile_rank_with_nsys.py:14-31 (one profiler per
torchrun child, rank-prefixed outputs).
"""
from __future__ import annotations

import argparse
import collections
import json
import os
import runpy
import sys
from pathlib import Path


def kernel_rows(prof) -> list:
    agg = collections.defaultdict(lambda: [0, 0.0])
    for ev in prof.events():
        if ev.device_type is not None and str(ev.device_type).endswith("CUDA") and ev.name:
            a = agg[ev.name]
            a[0] += 1
            a[1] += getattr(ev, "device_time_total", 0.0) or 0.0
    return sorted(({"name": n, "instances": c, "total_time_ns": int(us * 1e3)} for n, (c, us) in agg.items()),
                  key=lambda r: -r["total_time_ns"])


def profile_bundle(nproc, script_args, name, results_dir=None, tags=None, allow_dirty=False, port=29655,
                   timeout=None):
    """A multi-rank profile bundle: the script under torchrun, every rank profiled by this module.

    The bundle's ``profile/`` holds one ``rank{R}_kernels.json`` per rank (listed in the manifest's
    ``profile_reports``); the manifest kind is ``multi_rank_profile``.
    """
    import datetime as dt
    from . import bundle as B
    results_dir = Path(results_dir or B.DEFAULT_RESULTS)
    run_id = dt.datetime.now(dt.timezone.utc).strftime("%Y%m%dT%H%M%SZ") + "-" + name
    target = results_dir.resolve() / run_id
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}", "--master-addr",
           "127.0.0.1", "--master-port", str(port), "-m", "mini_megatron_b200.harness.rank_profile", "--out",
           str(target / "profile"), "--"] + list(script_args)
    bundle, manifest = B.run_bundle(cmd, name, results_dir, tags, allow_dirty=allow_dirty, timeout=timeout,
                                    run_id=run_id)
    reports = sorted(p.relative_to(bundle).as_posix() for p in (bundle / "profile").glob("rank*_kernels.json")) \
        if (bundle / "profile").is_dir() else []
    manifest.update(kind="multi_rank_profile", profile_reports=reports, profiled_ranks=len(reports),
                    profile_report=reports[0] if reports else None,
                    claim_scope="Profiler evidence only; not a throughput sample.")
    (bundle / "manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    B.write_checksums(bundle)
    return bundle, manifest


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--out", required=True)
    ap.add_argument("--trace", action="store_true", help="also export a Chrome trace per rank")
    ap.add_argument("script_and_args", nargs=argparse.REMAINDER)
    args = ap.parse_args(argv)
    rest = args.script_and_args[1:] if args.script_and_args[:1] == ["--"] else args.script_and_args
    if not rest:
        ap.error("give the script to run after --")
    rank = int(os.environ.get("RANK", os.environ.get("LOCAL_RANK", "0")))
    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    import torch
    from torch.profiler import ProfilerActivity, profile
    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
    script = rest[0]
    sys.argv = list(rest)
    code = 0
    with profile(activities=acts) as prof:
        try:
            runpy.run_path(script, run_name="__main__")
        except SystemExit as exc:  # the wrapped script's own exit status
            code = exc.code if isinstance(exc.code, int) else (0 if exc.code is None else 1)
    rows = kernel_rows(prof)
    (out / f"rank{rank}_kernels.json").write_text(json.dumps(rows, indent=1) + "\n", encoding="utf-8")
    if args.trace:
        prof.export_chrome_trace(str(out / f"rank{rank}_trace.json"))
    return code


if __name__ == "__main__":
    raise SystemExit(main())
