"""Append-only evidence ledger for a comparison campaign.

``init`` writes an immutable plan (``campaign.json``): the model contract,
the fairness requirements and numerical gate, the measurement plan with its
fixed ABBA schedule, and the topologies to cover.  ``record`` appends one
ledger entry that references an evidence file by absolute path, size and
SHA-256 (kinds: artifact, numerical_parity, benchmark_summary, profile,
diagnostic); entries are numbered files that are never rewritten.
``validate`` re-hashes every referenced file and reports, per topology,
whether the evidence chain is complete and whether it supports an
unconditional claim: a topology is publishable only when artifact,
numerical_parity, benchmark_summary and profile entries all exist and are
all marked ``ordinary``.

Reference: experiments/fair_parallel_campaign.py:16-195.

    python -m mini_megatron_b200.harness.campaign init --campaign-dir D --campaign-id ID
    python -m mini_megatron_b200.harness.campaign record --campaign-dir D --kind profile --topology tp1-pp1-dp1 --source F
    python -m mini_megatron_b200.harness.campaign validate --campaign-dir D
"""
from __future__ import annotations

import argparse
import datetime as dt
import json
from pathlib import Path

from .bundle import sha256_file
from .parity import GATES
from .queue import abba_schedule

SCHEMA_VERSION = 1
KINDS = ("artifact", "numerical_parity", "benchmark_summary", "profile", "diagnostic")
REQUIRED = ("artifact", "numerical_parity", "benchmark_summary", "profile")
CLAIM_STATUSES = ("ordinary", "conditional_exploratory", "diagnostic")

CONTRACT = {
    "model": "bias-free GPT next-token training",
    "layers": 12, "hidden_size": 768, "attention_heads": 12, "ffn_hidden_size": 3072,
    "sequence_length": 1024, "vocab_size": 50257, "precision": "bf16 tensor-core operands, fp32 master + AdamW",
    "optimizer": "AdamW(lr=6e-4, betas=(0.9, 0.999), weight_decay=0.1)", "dropout": 0.0,
    "position_embedding": "learned_absolute",
}
# B200 single-node matrix: the headline DP sweep plus the TP / PP mixes
TOPOLOGIES = (
    {"id": "tp1-pp1-dp1", "tp": 1, "pp": 1, "dp": 1, "status": "planned"},
    {"id": "tp1-pp1-dp2", "tp": 1, "pp": 1, "dp": 2, "status": "planned"},
    {"id": "tp1-pp1-dp4", "tp": 1, "pp": 1, "dp": 4, "status": "planned"},
    {"id": "tp1-pp1-dp8", "tp": 1, "pp": 1, "dp": 8, "status": "planned"},
    {"id": "tp2-pp1-dp1", "tp": 2, "pp": 1, "dp": 1, "status": "planned"},
    {"id": "tp1-pp2-dp1", "tp": 1, "pp": 2, "dp": 1, "status": "planned"},
    {"id": "tp2-pp2-dp2", "tp": 2, "pp": 2, "dp": 2, "status": "planned"},
)


def _now():
    return dt.datetime.now(dt.timezone.utc).isoformat()


def _write_new(path, obj):
    """Create ``path`` holding ``obj`` as JSON; ledger entries are write-once, so an existing file is an error."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    try:
        with open(path, "x", encoding="utf-8") as f:   # exclusive create: never replaces an entry
            json.dump(obj, f, indent=2, sort_keys=True)
            f.write("\n")
    except FileExistsError:
        raise ValueError(f"ledger entry {path} already exists; entries are never rewritten") from None


def load(campaign_dir) -> dict:
    f = Path(campaign_dir) / "campaign.json"
    if not f.is_file():
        raise ValueError(f"campaign.json not found: {f}")
    c = json.loads(f.read_text(encoding="utf-8"))
    if c.get("schema_version") != SCHEMA_VERSION:
        raise ValueError("unsupported campaign schema")
    return c


def init(campaign_dir, campaign_id, left="ours", right="reference", topologies=TOPOLOGIES) -> dict:
    d = Path(campaign_dir).resolve()
    if d.exists():
        raise ValueError(f"campaign directory already exists: {d}")
    plan = {
        "schema_version": SCHEMA_VERSION, "campaign_id": campaign_id, "created_at_utc": _now(),
        "archive_root": str(d), "purpose": f"{left} vs {right} on B200",
        "contract": CONTRACT,
        "fairness_requirements": {
            "same_logical_model": True, "same_source_weights": True, "same_immutable_batches": True,
            "same_global_tokens_per_optimizer_update": True, "numerical_gate": GATES["bf16"],
            "throughput_pairs": 5, "profile_is_not_throughput_sample": True,
            "device_timed_max_over_ranks": True,
        },
        "measurement_plan": {"warmup_optimizer_steps": 3, "measured_optimizer_steps": 20,
                             "execution_schedule": abba_schedule(left, right, 5)},
        "topologies": [dict(t) for t in topologies],
        "publication_rule": ("A topology is publishable only when its artifact, numerical_parity, benchmark_summary "
                             "and profile entries all validate and are all marked ordinary."),
    }
    d.mkdir(parents=True)
    _write_new(d / "campaign.json", plan)
    for sub in ("ledger", "artifacts", "parity", "benchmarks", "profiles", "reports"):
        (d / sub).mkdir()
    return plan


def record(campaign_dir, kind, topology, source, note=None, claim_status="ordinary") -> Path:
    c = load(campaign_dir)
    if kind not in KINDS:
        raise ValueError(f"unknown kind: {kind}")
    if claim_status not in CLAIM_STATUSES:
        raise ValueError(f"unknown claim status: {claim_status}")
    if topology not in {t["id"] for t in c["topologies"]}:
        raise ValueError(f"unknown topology: {topology}")
    src = Path(source).resolve()
    if not src.is_file():
        raise ValueError(f"source evidence is not a file: {src}")
    entry = {"schema_version": SCHEMA_VERSION, "kind": kind, "topology": topology, "recorded_at_utc": _now(),
             "source_path": str(src), "source_sha256": sha256_file(src), "source_size_bytes": src.stat().st_size,
             "campaign_id": c["campaign_id"], "claim_status": claim_status}
    if note:
        entry["note"] = note
    ledger = Path(campaign_dir) / "ledger"
    dest = ledger / f"{len(list(ledger.glob('*.json'))) + 1:04d}-{kind}-{topology}.json"
    _write_new(dest, entry)
    return dest


def validate(campaign_dir) -> dict:
    d = Path(campaign_dir).resolve()
    c = load(d)
    errors, entries = [], []
    for p in sorted((d / "ledger").glob("*.json")):
        try:
            e = json.loads(p.read_text(encoding="utf-8"))
        except ValueError as exc:
            errors.append(f"invalid ledger entry {p.name}: {exc}")
            continue
        entries.append(e)
        src = Path(e.get("source_path", ""))
        if not src.is_file():
            errors.append(f"{p.name}: source missing: {src}")
        elif sha256_file(src) != e.get("source_sha256"):
            errors.append(f"{p.name}: source checksum mismatch")
    status = {}
    for t in c["topologies"]:
        mine = [e for e in entries if e.get("topology") == t["id"]]
        kinds = {e.get("kind") for e in mine}
        claims = sorted({e.get("claim_status", "legacy_unspecified") for e in mine if e.get("kind") in REQUIRED})
        complete = set(REQUIRED) <= kinds
        status[t["id"]] = {"recorded_kinds": sorted(k for k in kinds if k),
                           "missing_publishable_evidence": sorted(set(REQUIRED) - kinds),
                           "claim_statuses": claims, "evidence_chain_complete": complete,
                           "unconditional_publishable": complete and claims == ["ordinary"],
                           "conditional_conclusion_required": complete and claims != ["ordinary"]}
    return {"campaign_id": c["campaign_id"], "valid": not errors, "errors": errors, "topologies": status}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    i = sub.add_parser("init")
    i.add_argument("--campaign-dir", required=True)
    i.add_argument("--campaign-id", required=True)
    r = sub.add_parser("record")
    r.add_argument("--campaign-dir", required=True)
    r.add_argument("--kind", required=True, choices=KINDS)
    r.add_argument("--topology", required=True)
    r.add_argument("--source", required=True)
    r.add_argument("--note")
    r.add_argument("--claim-status", default="ordinary", choices=CLAIM_STATUSES)
    v = sub.add_parser("validate")
    v.add_argument("--campaign-dir", required=True)
    args = ap.parse_args(argv)
    try:
        if args.cmd == "init":
            print(json.dumps(init(args.campaign_dir, args.campaign_id), indent=2, sort_keys=True))
            return 0
        if args.cmd == "record":
            print(record(args.campaign_dir, args.kind, args.topology, args.source, args.note, args.claim_status))
            return 0
        res = validate(args.campaign_dir)
        print(json.dumps(res, indent=2, sort_keys=True))
        return 0 if res["valid"] else 1
    except ValueError as exc:
        ap.error(str(exc))


if __name__ == "__main__":
    raise SystemExit(main())
