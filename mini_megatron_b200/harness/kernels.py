"""Kernel-time classification of a launch list.

Input rows are ``{"name", "total_time_ns", "instances"}`` -- from
``bundle.ncu_kernel_summary`` (an ``ncu`` one-pass launch list), from
``utils.step_profile`` (PyTorch profiler), or from any CSV with the columns
``Name``, ``Total Time (ns)``, ``Instances``.  Each kernel is put in the first
category whose pattern matches its name; anything unmatched stays visible as
``unclassified`` (no guessing from neighbouring launches).  Collective-fused
kernels of this framework get their own categories so that their share of
the step is explicit.

Reference: experiments/analyze_nsys_kernel_summary.py:21-78 (conservative
regex buckets, unclassified kept).
"""
from __future__ import annotations

import argparse
import csv
import json
import re
from pathlib import Path

# order matters: first match wins
CLASSIFIERS = (
    ("fused_dp_optimizer", re.compile(r"dp_rs_adamw_ag", re.I)),
    ("fused_tp_collective", re.compile(r"tp_rs_reduce|tp_ag_push|ln_fwd_push|EPI_PUSH|, 7>", re.I)),
    ("fused_adamw", re.compile(r"adamw_kernel|FusedAdamMathFunctor|multi_tensor_apply_kernel", re.I)),
    ("attention", re.compile(r"flash|fmha|scaled_dot_product|attn_", re.I)),
    ("gemm", re.compile(r"gemm|cutlass|cublas|nvjet|matmul|sm100_xmma|sm90_xmma", re.I)),
    ("layernorm", re.compile(r"ln_fwd|ln_bwd|ln_param|layer_norm|LayerNorm|GammaBeta", re.I)),
    ("cross_entropy", re.compile(r"ce_fwd|ce_bwd|cross_entropy|SoftMax|softmax|nll_loss", re.I)),
    ("embedding", re.compile(r"emb_|embedding|gather_kernel|index_select", re.I)),
    ("nccl", re.compile(r"nccl", re.I)),
    ("copy_cast", re.compile(r"bfloat16_copy|copy_kernel|f32_to_bf16|cast|Memcpy|Memset|CatArray", re.I)),
)


def classify(name: str) -> str:
    for cat, pat in CLASSIFIERS:
        if pat.search(name):
            return cat
    return "unclassified"


def _int(v):
    return int(str(v).replace(",", ""))


def read_rows(path) -> list:
    """Rows from a kernel-summary CSV (Name / Total Time (ns) / Instances) or a JSON list of rows."""
    path = Path(path)
    if path.suffix == ".json":
        data = json.loads(path.read_text(encoding="utf-8"))
        return [{"name": r["name"], "total_time_ns": _int(r["total_time_ns"]), "instances": _int(r["instances"])}
                for r in data]
    with path.open(newline="", encoding="utf-8-sig") as f:
        return [{"name": r["Name"], "total_time_ns": _int(r["Total Time (ns)"]), "instances": _int(r["Instances"])}
                for r in csv.DictReader(f)]


def analyze(rows) -> dict:
    total = sum(r["total_time_ns"] for r in rows)
    cats = {}
    for r in rows:
        c = cats.setdefault(classify(r["name"]), {"total_time_ns": 0, "instances": 0, "kernels": []})
        c["total_time_ns"] += r["total_time_ns"]
        c["instances"] += r["instances"]
        c["kernels"].append(r)
    for c in cats.values():
        c["percent_kernel_time"] = 100.0 * c["total_time_ns"] / total if total else 0.0
        c["kernels"].sort(key=lambda r: -r["total_time_ns"])
    return {"total_kernel_time_ns": total, "total_kernel_instances": sum(r["instances"] for r in rows),
            "categories": cats, "top_kernels": sorted(rows, key=lambda r: -r["total_time_ns"])[:30],
            "classification_rules": [{"category": c, "regex": p.pattern} for c, p in CLASSIFIERS],
            "method_notes": ["Percentages are of total kernel time, not wall-clock time.",
                             "Unmatched kernel time is kept as unclassified."]}


def analyze_bundle(bundle) -> dict:
    """Classify a profile bundle's kernel summary and store profile/analysis.json (re-checksummed)."""
    from .bundle import sha256_file, write_checksums
    bundle = Path(bundle)
    src = bundle / "profile" / "kernel_summary.json"
    if not src.is_file():
        raise ValueError(f"no profile/kernel_summary.json in {bundle}")
    res = analyze(read_rows(src))
    res.update({"schema_version": 1, "source": "profile/kernel_summary.json", "source_sha256": sha256_file(src)})
    (bundle / "profile" / "analysis.json").write_text(json.dumps(res, indent=2, sort_keys=True) + "\n",
                                                      encoding="utf-8")
    write_checksums(bundle)
    return res


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("source", help="a profile bundle directory, a kernel-summary CSV or a JSON list of rows")
    args = ap.parse_args(argv)
    p = Path(args.source)
    res = analyze_bundle(p) if p.is_dir() else analyze(read_rows(p))
    print(json.dumps({"total_kernel_time_ns": res["total_kernel_time_ns"],
                      "categories": {k: {"percent_kernel_time": round(v["percent_kernel_time"], 2),
                                         "instances": v["instances"]} for k, v in res["categories"].items()}},
                     indent=2, sort_keys=True))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
