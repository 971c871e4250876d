"""Datasets, convergence comparisons and archived benchmark sweeps.

* ``generate_synthetic`` / ``save_synthetic`` -- a learnable fixed dataset
  ``labels = (input_ids + 1) % effective_vocab`` of shape ``[N, B, S]`` in the
  ``--data-file`` format of ``main.py`` (and of the reference's main.py).
* ``make_identity`` -- the same file with ``labels = input_ids``.
* ``parse_losses`` / ``parse_report`` -- the ``step N | loss X`` lines and the
  final report block that both main.py programs print.
* ``run_main`` -- one training run of this framework's or the reference's
  ``main.py`` through torchrun (127.0.0.1 rendezvous).
* ``compare_convergence`` -- both programs on one data file; loss curves
  side by side, with a pass rule on this framework's loss decrease.
* ``compare_loss`` -- the smoke comparison at TP=1 and TP=2.
* ``loss_curve_record`` -- the ``results/*.json`` loss-curve schema
  (``task``, ``model``, ``data``, ``config``, ``results{name: [{step, loss}]}``,
  ``conclusion``).
* ``save_benchmark_results`` -- alternating A/B rounds of both programs with
  raw logs archived next to a summary JSON.

Reference: experiments/synthetic_data.py:12-45, experiments/make_identity.py,
experiments/compare_convergence.py:25-157, experiments/save_benchmark_results.py:34-183,
eval/compare_loss.py:16-43, results/identity_2000steps.json (schema).
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parents[2]
OURS_MAIN = REPO / "main.py"
REFERENCE_MAIN = REPO / "baseline" / "_ref" / "main.py"
_STEP_RE = re.compile(r"step\s+(\d+)\s+\|\s+loss\s+([\d.]+)")
_REPORT = (("throughput", re.compile(r"Throughput:\s+([\d,]+) tok/s")),
           ("peak_mem", re.compile(r"Peak memory:\s+([\d.]+) GB")),
           ("mfu", re.compile(r"MFU:\s+([\d.]+)%")),
           ("final_loss", re.compile(r"Final loss:\s+([\d.]+)")))


def generate_synthetic(num_steps, B, S, effective_vocab, seed=42):
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(0, effective_vocab, (num_steps, B, S), generator=g)
    return x.clone(), (x + 1) % effective_vocab


def save_synthetic(path, num_steps=100, B=4, S=512, effective_vocab=1024, model_vocab=50304, seed=42):
    ids, labels = generate_synthetic(num_steps, B, S, effective_vocab, seed)
    data = {"input_ids": ids, "labels": labels, "effective_vocab": effective_vocab, "model_vocab": model_vocab,
            "B": B, "S": S, "num_steps": num_steps, "seed": seed}
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    torch.save(data, path)
    return data


def make_identity(src, dst):
    d = torch.load(src, map_location="cpu", weights_only=True)
    d["labels"] = d["input_ids"].clone()
    torch.save(d, dst)
    return d


def parse_losses(stdout: str) -> list:
    return [(int(m.group(1)), float(m.group(2))) for m in _STEP_RE.finditer(stdout)]


def parse_report(stdout: str) -> dict:
    out = {}
    for k, pat in _REPORT:
        m = pat.search(stdout)
        if m:
            out[k] = float(m.group(1).replace(",", ""))
    return out


def run_main(script, nproc=1, args=(), timeout=1200, port=None, env=None) -> dict:
    port = port or 29000 + (os.getpid() % 900)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr", "127.0.0.1", "--master-port", str(port), str(script)] + [str(a) for a in args]
    e = dict(os.environ, **(env or {}))
    e["PYTHONPATH"] = str(Path(script).resolve().parent) + os.pathsep + e.get("PYTHONPATH", "")
    t0 = time.time()
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=e, cwd=str(Path(script).parent))
        out, err, rc = r.stdout, r.stderr, r.returncode
    except subprocess.TimeoutExpired as exc:
        out, err, rc = exc.stdout or "", (exc.stderr or "") + "\nTIMEOUT", None
    return {"command": cmd, "return_code": rc, "elapsed_s": round(time.time() - t0, 2), "stdout": out,
            "stderr": err, "losses": parse_losses(out), "report": parse_report(out)}


def compare_convergence(data_file, steps=100, warmup=10, min_drop=1.0, extra_ours=(), extra_ref=()) -> dict:
    common = ["--tp", "1", "--pp", "1", "--num-steps", str(steps), "--warmup-steps", str(warmup), "--data-file",
              str(data_file), "--log-interval", "1"]
    ours = run_main(OURS_MAIN, 1, common + list(extra_ours))
    ref = run_main(REFERENCE_MAIN, 1, common + ["--amp"] + list(extra_ref)) if REFERENCE_MAIN.exists() else None
    res = {"ours": ours, "reference": ref}
    lo = ours["losses"]
    res["ours_drop"] = (lo[0][1] - lo[-1][1]) if lo else None
    res["passed"] = bool(lo) and res["ours_drop"] > min_drop
    if ref and ref["losses"]:
        lr = ref["losses"]
        res["reference_drop"] = lr[0][1] - lr[-1][1]
        pairs = list(zip(lo, lr))
        res["max_abs_loss_diff"] = max((abs(a[1] - b[1]) for a, b in pairs), default=None)
    return res


def compare_loss(steps=20, warmup=5, batch=4) -> dict:
    """Both programs at TP=1 and TP=2.  Each draws its own random data, so losses are a smoke check only."""
    out = {}
    for tp in (1, 2):
        args = ["--tp", str(tp), "--pp", "1", "--num-steps", str(steps), "--warmup-steps", str(warmup),
                "--micro-batch-size", str(batch)]
        o = run_main(OURS_MAIN, tp, args)
        r = run_main(REFERENCE_MAIN, tp, args) if REFERENCE_MAIN.exists() else None
        out[f"tp{tp}"] = {"ours": o["losses"], "reference": r["losses"] if r else None}
    return out


def loss_curve_record(task, model, data, config, results: dict, conclusion) -> dict:
    return {"task": task, "model": model, "data": data, "config": config,
            "results": {k: [{"step": int(s), "loss": float(l)} for s, l in v] for k, v in results.items()},
            "conclusion": conclusion}


def save_benchmark_results(out_dir, configs, rounds=2, steps=50, warmup=10) -> dict:
    """``configs``: {name: (which, nproc, extra args)} with which in {"ours", "reference"}.

    Runs every config once per round, reversing the order in alternate rounds,
    archives each raw stdout under ``out_dir/logs`` and returns the summary
    (also written to ``out_dir/benchmarks.json``).
    """
    out_dir = Path(out_dir)
    (out_dir / "logs").mkdir(parents=True, exist_ok=True)
    summary = {"generated_utc": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
               "method": "alternating A/B rounds, raw logs archived", "runs": {}}
    names = list(configs)
    for rnd in range(1, rounds + 1):
        order = names if rnd % 2 else list(reversed(names))
        rr = {}
        for name in order:
            which, nproc, extra = configs[name]
            script = OURS_MAIN if which == "ours" else REFERENCE_MAIN
            res = run_main(script, nproc, ["--num-steps", str(steps), "--warmup-steps", str(warmup)] + list(extra))
            log = out_dir / "logs" / f"r{rnd}_{name}.log"
            log.write_text("CMD: " + " ".join(res["command"]) + "\n\n" + res["stdout"] +
                           ("\n\nSTDERR:\n" + res["stderr"] if res["stderr"] else ""), encoding="utf-8")
            rr[name] = dict(res["report"], return_code=res["return_code"], elapsed_s=res["elapsed_s"],
                            log=str(log.relative_to(out_dir)))
        summary["runs"][f"round{rnd}"] = rr
    (out_dir / "benchmarks.json").write_text(json.dumps(summary, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    return summary


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    s = sub.add_parser("synthetic")
    s.add_argument("path")
    s.add_argument("--num-steps", type=int, default=100)
    s.add_argument("--batch-size", type=int, default=4)
    s.add_argument("--seq-len", type=int, default=512)
    s.add_argument("--effective-vocab", type=int, default=1024)
    s.add_argument("--seed", type=int, default=42)
    i = sub.add_parser("identity")
    i.add_argument("src")
    i.add_argument("dst")
    c = sub.add_parser("convergence")
    c.add_argument("--data-file", required=True)
    c.add_argument("--steps", type=int, default=100)
    c.add_argument("--warmup", type=int, default=10)
    c.add_argument("--output")
    lc = sub.add_parser("compare-loss")
    lc.add_argument("--steps", type=int, default=20)
    args = ap.parse_args(argv)
    if args.cmd == "synthetic":
        save_synthetic(args.path, args.num_steps, args.batch_size, args.seq_len, args.effective_vocab,
                       seed=args.seed)
        print(f"saved {args.path}: [{args.num_steps}, {args.batch_size}, {args.seq_len}], (x+1)%{args.effective_vocab}")
        return 0
    if args.cmd == "identity":
        make_identity(args.src, args.dst)
        print(f"saved {args.dst}")
        return 0
    if args.cmd == "compare-loss":
        print(json.dumps(compare_loss(args.steps), indent=2))
        return 0
    res = compare_convergence(args.data_file, args.steps, args.warmup)
    slim = {k: v for k, v in res.items() if k not in ("ours", "reference")}
    slim["ours_losses"] = res["ours"]["losses"]
    slim["reference_losses"] = res["reference"]["losses"] if res["reference"] else None
    slim["ours_report"] = res["ours"]["report"]
    slim["reference_report"] = res["reference"]["report"] if res["reference"] else None
    text = json.dumps(slim, indent=2)
    print(text)
    if args.output:
        Path(args.output).write_text(text + "\n", encoding="utf-8")
    return 0 if res["passed"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
