"""Run bundles: one command -> one immutable, checksummed evidence directory.

A bundle directory holds::

    manifest.json      what ran, when, exit code, parsed metrics, tags, inputs
    metrics.json       the parsed metrics alone
    environment.json   git state, pip freeze, nvidia-smi, NVLink topology,
                       CUDA/NCCL/TORCH environment variables, tool versions
    command.txt        the command line as executed
    stdout.log / stderr.log
    profile/           (profile bundles) ncu launch list + kernel summary
    checksums.sha256   SHA-256 of every other file

``run`` refuses a dirty git tree and busy GPUs unless told otherwise, and
never overwrites a bundle.  A profile bundle first runs the command plainly
and only re-runs it under ``ncu`` (one-pass launch list,
``--clock-control none``) when that plain run exited 0; profile bundles are
evidence for bottleneck analysis, never throughput samples.

Metrics are parsed from the report lines ``main.py`` prints (``Throughput:``,
``Peak memory:``, ``MFU:``, ``Final loss:``) and from a ``bench.py`` JSON line.

Reference: experiments/run_experiment.py:44-230 (runner, metric regexes,
preflight, environment capture, checksums), experiments/validate_run_bundle.py:8-57.

    python -m mini_megatron_b200.harness.bundle run --name NAME [--tag k=v] [--profile] -- CMD...
    python -m mini_megatron_b200.harness.bundle validate BUNDLE
"""
from __future__ import annotations

import argparse
import datetime as dt
import hashlib
import json
import os
import platform
import re
import shutil
import subprocess
import sys
import time
from pathlib import Path

SCHEMA_VERSION = 1
REPO = Path(__file__).resolve().parents[2]
DEFAULT_RESULTS = REPO / "results" / "runs"

REQUIRED_FILES = ("manifest.json", "metrics.json", "environment.json", "stdout.log", "stderr.log", "command.txt",
                  "checksums.sha256")
REQUIRED_FIELDS = ("schema_version", "run_id", "kind", "claim_scope", "target_command", "executed_command",
                   "started_at_utc", "finished_at_utc", "elapsed_wall_seconds", "return_code", "metrics",
                   "environment_file")
_NAME_RE = re.compile(r"[A-Za-z0-9][A-Za-z0-9._-]*")

# report lines printed by main.py (and by the reference's main.py)
_REPORT_PATTERNS = (
    ("throughput_tok_s", re.compile(r"Throughput:\s+([\d,]+(?:\.\d+)?) tok/s")),
    ("peak_memory_gb", re.compile(r"Peak memory:\s+([\d.]+) GB")),
    ("mfu_percent", re.compile(r"MFU:\s+([\d.]+)%")),
    ("final_loss", re.compile(r"Final loss:\s+([\d.]+)")),
)


# ----------------------------------------------------------------------------- small helpers
def sha256_file(path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def _capture(cmd, cwd=REPO) -> str:
    try:
        return subprocess.run(cmd, cwd=cwd, text=True, capture_output=True, check=True).stdout.strip()
    except (OSError, subprocess.CalledProcessError) as exc:
        detail = getattr(exc, "stdout", "") or ""
        return f"UNAVAILABLE: {exc}\n{detail}".strip()


def _write_json(path, obj):
    Path(path).write_text(json.dumps(obj, indent=2, sort_keys=True) + "\n", encoding="utf-8")


# ----------------------------------------------------------------------------- parsing
def parse_metrics(stdout: str) -> dict:
    """Metrics from a run's stdout: main.py report lines and/or one bench.py JSON line."""
    metrics = {}
    for key, pat in _REPORT_PATTERNS:
        m = pat.search(stdout)
        if m:
            metrics[key] = float(m.group(1).replace(",", ""))
    for line in stdout.splitlines():
        line = line.strip()
        if not (line.startswith("{") and '"metric"' in line):
            continue
        try:
            rec = json.loads(line)
        except ValueError:
            continue
        if "value" in rec:
            if rec.get("unit") == "tok/s":
                metrics["throughput_tok_s"] = float(rec["value"])
            metrics["bench_value"] = rec["value"]
        for k in ("ms_per_step", "n_gpus"):
            if k in rec:
                metrics[k] = rec[k]
        if isinstance(rec.get("e2e"), dict) and "value" in rec["e2e"]:
            metrics["e2e_value"] = rec["e2e"]["value"]
    return metrics


def parse_compute_processes(stdout: str) -> list:
    """Non-empty rows of ``nvidia-smi --query-compute-apps`` output (idle messages dropped)."""
    rows = []
    for line in stdout.splitlines():
        line = line.strip()
        if line and not line.startswith("No running"):
            rows.append(line)
    return rows


def gpu_preflight() -> dict:
    """Which compute processes hold a GPU right now (reads state only)."""
    cmd = ["nvidia-smi", "--query-compute-apps=pid,process_name,gpu_uuid", "--format=csv,noheader"]
    try:
        r = subprocess.run(cmd, cwd=REPO, text=True, capture_output=True)
    except OSError as exc:
        return {"command": cmd, "return_code": None, "stdout": "", "stderr": f"UNAVAILABLE: {exc}",
                "active_processes": []}
    return {"command": cmd, "return_code": r.returncode, "stdout": r.stdout, "stderr": r.stderr,
            "active_processes": parse_compute_processes(r.stdout) if r.returncode == 0 else []}


def capture_environment(preflight=None) -> dict:
    env_keys = ("CUDA", "NCCL", "TORCH", "PYTORCH", "MMB", "OMP")
    return {
        "captured_at_utc": dt.datetime.now(dt.timezone.utc).isoformat(),
        "platform": platform.platform(),
        "python": sys.version,
        "git_commit": _capture(["git", "rev-parse", "HEAD"]),
        "git_status": _capture(["git", "status", "--short"]),
        "git_diff": _capture(["git", "diff"]),
        "pip_freeze": _capture([sys.executable, "-m", "pip", "freeze"]),
        "nvidia_smi": _capture(["nvidia-smi"]),
        "nvidia_topology": _capture(["nvidia-smi", "topo", "-m"]),
        "nvcc_version": _capture(["nvcc", "--version"]),
        "ncu_version": _capture(["ncu", "--version"]),
        "gpu_preflight": preflight,
        "environment_variables": {k: v for k, v in os.environ.items() if k.startswith(env_keys)},
    }


def write_checksums(bundle) -> None:
    bundle = Path(bundle)
    lines = [f"{sha256_file(p)}  {p.relative_to(bundle).as_posix()}" for p in sorted(bundle.rglob("*"))
             if p.is_file() and p.name != "checksums.sha256"]
    (bundle / "checksums.sha256").write_text("\n".join(lines) + "\n", encoding="utf-8")


# ----------------------------------------------------------------------------- validation
def validate(bundle) -> list:
    """Problems with a bundle (empty list = valid): files, manifest fields, checksums."""
    bundle = Path(bundle)
    missing = [n for n in REQUIRED_FILES if not (bundle / n).is_file()]
    if missing:
        return ["missing required files: " + ", ".join(sorted(missing))]
    try:
        manifest = json.loads((bundle / "manifest.json").read_text(encoding="utf-8"))
    except ValueError as exc:
        return [f"invalid manifest.json: {exc}"]
    errors = []
    absent = [f for f in REQUIRED_FIELDS if f not in manifest]
    if absent:
        errors.append("manifest missing fields: " + ", ".join(sorted(absent)))
    if manifest.get("schema_version") != SCHEMA_VERSION:
        errors.append("unsupported schema_version")
    if not isinstance(manifest.get("target_command"), list) or not manifest.get("target_command"):
        errors.append("target_command must be a non-empty list")
    if not isinstance(manifest.get("metrics"), dict):
        errors.append("metrics must be an object")
    if manifest.get("kind") in ("profile", "multi_rank_profile") and not manifest.get("profile_report"):
        errors.append("profile bundle has no profile_report")
    listed = set()
    for line in (bundle / "checksums.sha256").read_text(encoding="utf-8").splitlines():
        if not line.strip():
            continue
        digest, sep, rel = line.partition("  ")
        if not sep:
            errors.append("malformed checksum line: " + line)
            continue
        listed.add(rel)
        target = bundle / rel
        if not target.is_file():
            errors.append("checksummed file missing: " + rel)
        elif sha256_file(target) != digest:
            errors.append("checksum mismatch: " + rel)
    for p in sorted(bundle.rglob("*")):
        rel = p.relative_to(bundle).as_posix()
        if p.is_file() and p.name != "checksums.sha256" and rel not in listed:
            errors.append("file not covered by checksums: " + rel)
    return errors


# ----------------------------------------------------------------------------- profiling
def ncu_kernel_summary(launch_csv) -> list:
    """Aggregate an ``ncu --csv --metrics gpu__time_duration.sum`` launch list into per-kernel rows."""
    import csv
    rows = {}
    with open(launch_csv, newline="", encoding="utf-8", errors="replace") as f:
        lines = [ln for ln in f if ln.startswith('"')]
    for rec in csv.DictReader(lines):
        if rec.get("Metric Name") != "gpu__time_duration.sum":
            continue
        name = rec.get("Kernel Name") or rec.get("Function Name") or "?"
        unit = (rec.get("Metric Unit") or "ns").strip()
        val = float(str(rec.get("Metric Value", "0")).replace(",", ""))
        scale = {"ns": 1.0, "nsecond": 1.0, "us": 1e3, "usecond": 1e3, "ms": 1e6, "msecond": 1e6}.get(unit, 1.0)
        r = rows.setdefault(name, {"name": name, "total_time_ns": 0, "instances": 0})
        r["total_time_ns"] += int(round(val * scale))
        r["instances"] += 1
    return sorted(rows.values(), key=lambda r: -r["total_time_ns"])


def _profile_command(ncu, csv_path, command, skip, count):
    return [ncu, "--metrics", "gpu__time_duration.sum", "--clock-control", "none", "-s", str(skip), "-c", str(count),
            "--csv", "--log-file", str(csv_path)] + list(command)


# ----------------------------------------------------------------------------- runner
def run_bundle(command, name, results_dir=DEFAULT_RESULTS, tags=None, artifacts=(), profile=False, allow_dirty=False,
               allow_active_gpus=False, ncu="ncu", profile_skip=0, profile_count=2000, timeout=None, run_id=None):
    """Run ``command`` into a new bundle; returns (bundle_path, manifest)."""
    if not _NAME_RE.fullmatch(name):
        raise ValueError("name may contain only letters, digits, '.', '_' and '-'")
    if not command:
        raise ValueError("empty command")
    tags = dict(tags or {})
    status = _capture(["git", "status", "--short"])
    dirty = bool(status) and not status.startswith("UNAVAILABLE")
    if dirty and not allow_dirty:
        raise ValueError("working tree is dirty; commit first or pass allow_dirty")
    preflight = gpu_preflight()
    if preflight["active_processes"] and not allow_active_gpus:
        raise ValueError("GPU preflight found active compute processes: " + "; ".join(preflight["active_processes"]))
    if profile and shutil.which(ncu) is None:
        raise ValueError(f"ncu not found: {ncu}")
    inputs = []
    for a in artifacts:
        p = Path(a).expanduser().resolve()
        if not p.is_file():
            raise ValueError(f"artifact is not a readable file: {p}")
        inputs.append({"path": str(p), "size_bytes": p.stat().st_size, "sha256": sha256_file(p)})
    run_id = run_id or dt.datetime.now(dt.timezone.utc).strftime("%Y%m%dT%H%M%SZ") + "-" + name
    bundle = Path(results_dir).expanduser().resolve() / run_id
    if bundle.exists():
        raise ValueError(f"refusing to overwrite bundle: {bundle}")
    bundle.mkdir(parents=True)
    env = capture_environment(preflight)
    _write_json(bundle / "environment.json", env)

    executed = list(command)
    t0 = time.time()
    r = subprocess.run(executed, cwd=REPO, text=True, capture_output=True, timeout=timeout)
    t1 = time.time()
    stdout, stderr, rc = r.stdout, r.stderr, r.returncode
    report = None
    profile_info = None
    if profile:
        pdir = bundle / "profile"
        pdir.mkdir()
        csv_path = pdir / "launches.csv"
        prof_cmd = _profile_command(ncu, csv_path, command, profile_skip, profile_count)
        executed = prof_cmd
        if rc == 0:   # profile only a command that has just exited 0 without the profiler
            pr = subprocess.run(prof_cmd, cwd=REPO, text=True, capture_output=True, timeout=timeout)
            (pdir / "ncu_stdout.log").write_text(pr.stdout, encoding="utf-8")
            (pdir / "ncu_stderr.log").write_text(pr.stderr, encoding="utf-8")
            profile_info = {"return_code": pr.returncode, "command": prof_cmd}
            if pr.returncode == 0 and csv_path.exists():
                summary = ncu_kernel_summary(csv_path)
                _write_json(pdir / "kernel_summary.json", summary)
                report = "profile/launches.csv"
        else:
            profile_info = {"return_code": None, "skipped": "plain run exited non-zero; not profiled"}
    (bundle / "command.txt").write_text(" ".join(executed) + "\n", encoding="utf-8")
    (bundle / "stdout.log").write_text(stdout, encoding="utf-8")
    (bundle / "stderr.log").write_text(stderr, encoding="utf-8")
    metrics = parse_metrics(stdout)
    manifest = {
        "schema_version": SCHEMA_VERSION,
        "run_id": run_id,
        "kind": "profile" if profile else "benchmark",
        "claim_scope": ("Profiler evidence only; not a throughput sample." if profile else
                        "One benchmark replicate; aggregate paired replicates before a claim."),
        "tags": tags,
        "input_artifacts": inputs,
        "source_tree_clean": not dirty,
        "gpu_preflight": preflight,
        "target_command": list(command),
        "executed_command": executed,
        "started_at_utc": dt.datetime.fromtimestamp(t0, dt.timezone.utc).isoformat(),
        "finished_at_utc": dt.datetime.fromtimestamp(t1, dt.timezone.utc).isoformat(),
        "elapsed_wall_seconds": round(t1 - t0, 6),
        "return_code": rc,
        "metrics": metrics,
        "profile_report": report,
        "profile_run": profile_info,
        "environment_file": "environment.json",
        "environment_capture_time": env["captured_at_utc"],
    }
    _write_json(bundle / "metrics.json", metrics)
    _write_json(bundle / "manifest.json", manifest)
    write_checksums(bundle)
    return bundle, manifest


def _parse_tags(items):
    tags = {}
    for item in items:
        k, sep, v = item.partition("=")
        if not sep or not k or not v:
            raise ValueError("--tag must be KEY=VALUE")
        if k in tags:
            raise ValueError("duplicate --tag key: " + k)
        tags[k] = v
    return tags


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run", help="run one command into a new bundle")
    r.add_argument("--name", required=True)
    r.add_argument("--results-dir", default=str(DEFAULT_RESULTS))
    r.add_argument("--tag", action="append", default=[], metavar="KEY=VALUE")
    r.add_argument("--artifact", action="append", default=[], metavar="PATH")
    r.add_argument("--profile", action="store_true", help="add an ncu launch list (after a clean plain run)")
    r.add_argument("--ncu-bin", default="ncu")
    r.add_argument("--profile-skip", type=int, default=0, help="launches to skip before the launch list")
    r.add_argument("--profile-count", type=int, default=2000)
    r.add_argument("--allow-dirty", action="store_true")
    r.add_argument("--allow-active-gpus", action="store_true")
    r.add_argument("command", nargs=argparse.REMAINDER)
    v = sub.add_parser("validate", help="check a bundle's manifest and checksums")
    v.add_argument("bundle")
    args = ap.parse_args(argv)
    if args.cmd == "validate":
        errors = validate(args.bundle)
        if errors:
            print("INVALID RUN BUNDLE")
            print("\n".join("- " + e for e in errors))
            return 1
        print("VALID RUN BUNDLE: " + str(Path(args.bundle).resolve()))
        return 0
    command = args.command[1:] if args.command[:1] == ["--"] else args.command
    try:
        bundle, manifest = run_bundle(command, args.name, args.results_dir, _parse_tags(args.tag), args.artifact,
                                      args.profile, args.allow_dirty, args.allow_active_gpus, args.ncu_bin,
                                      args.profile_skip, args.profile_count)
    except ValueError as exc:
        ap.error(str(exc))
    print(json.dumps({"bundle": str(bundle), "return_code": manifest["return_code"],
                      "metrics": manifest["metrics"]}, indent=2))
    return manifest["return_code"]


if __name__ == "__main__":
    raise SystemExit(main())
