"""Frozen, shared inputs for fair comparisons.

``freeze`` writes one directory that every implementation of a comparison
loads, so that no benchmark compares unrelated random initialisations or
different data:

    source_full.pt            unsharded weights in the shared layout (exact vocabulary)
    ours_tp{T}_pp{P}_rank{R}.pt   this framework's chunk for global rank R (vocabulary padded)
    reference_tp{T}_pp{P}_rank{R}.pt   the reference's chunk (its own names and shards)
    next_token_batches.pt     [N, B, S] tokens; labels = next token, last = -100
    manifest.json             contract, seeds, shapes, SHA-256 of every file

It refuses to write into an existing directory.  Global ranks follow the
topology rule ``rank = dp_rank * tp * pp + pp_rank * tp + tp_rank``; chunks
are written for dp_rank 0 (replicas share weights).

Reference: experiments/create_fair_tp1_artifacts.py:22-68,
experiments/create_fair_tp2_artifacts.py, experiments/create_fair_pp_artifacts.py:60-207.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

from .bundle import sha256_file
from .contract import CONTRACT, from_reference_state, full_parameter_names, shard_state

SCHEMA_VERSION = 1


def _model_dict(c):
    keys = ("num_layers", "hidden_size", "num_attention_heads", "ffn_hidden_size", "max_seq_len", "vocab_size")
    return {k: (c[k] if isinstance(c, dict) else getattr(c, k)) for k in keys}


def canonical_weights(model_config, seed) -> dict:
    """Unsharded N(0, 0.02) weights (LayerNorm weight 1, bias 0) from an explicit CPU generator."""
    mc = _model_dict(model_config)
    g = torch.Generator().manual_seed(seed)
    H, F, V, S = mc["hidden_size"], mc["ffn_hidden_size"], mc["vocab_size"], mc["max_seq_len"]
    shapes = {"embedding.token_embedding.weight": (V, H), "embedding.position_embedding.weight": (S, H),
              "attn.qkv.weight": (3 * H, H), "attn.o.weight": (H, H), "mlp.fc1.weight": (F, H),
              "mlp.fc2.weight": (H, F), "lm_head.weight": (V, H)}
    out = {}
    for n in full_parameter_names(mc):
        if n.endswith(("ln1.weight", "ln2.weight")) or n == "ln_f.weight":
            out[n] = torch.ones(H)
        elif n.endswith(("ln1.bias", "ln2.bias")) or n == "ln_f.bias":
            out[n] = torch.zeros(H)
        else:
            key = n if n in shapes else ".".join(n.split(".")[-3:])
            out[n] = torch.randn(shapes[key], generator=g) * 0.02
    return out


def next_token_batches(num_batches, batch_size, seq_len, vocab, seed, pattern="next_token", effective_vocab=None):
    """Fixed batches.  ``next_token``: uniform tokens, labels = the next token (last = -100);
    ``shift``: labels = (token + 1) % effective_vocab (a learnable task); ``identity``: labels = tokens."""
    g = torch.Generator().manual_seed(seed)
    hi = effective_vocab or vocab
    tokens = torch.randint(0, hi, (num_batches, batch_size, seq_len), generator=g, dtype=torch.long)
    if pattern == "shift":
        return tokens, (tokens + 1) % hi
    if pattern == "identity":
        return tokens, tokens.clone()
    if pattern != "next_token":
        raise ValueError(f"unknown pattern {pattern}")
    labels = torch.roll(tokens, -1, dims=-1)
    labels[..., -1] = -100
    return tokens, labels


def freeze(out_dir, model_config, tp=1, pp=1, num_batches=64, batch_size=4, seed=20260818, padded_vocab=None,
           pattern="next_token", effective_vocab=None):
    out_dir = Path(out_dir)
    if out_dir.exists():
        raise ValueError(f"refusing to overwrite artifact directory: {out_dir}")
    mc = _model_dict(model_config)
    if padded_vocab is None:
        mult = 128 * tp
        padded_vocab = (mc["vocab_size"] + mult - 1) // mult * mult
    out_dir.mkdir(parents=True)
    full = canonical_weights(mc, seed)
    files = {"source": out_dir / "source_full.pt"}
    torch.save({"schema_version": SCHEMA_VERSION, "contract": CONTRACT, "seed": seed, "model": mc,
                "state_dict": full}, files["source"])
    ours_full = from_reference_state(full, padded_vocab)
    for pp_rank in range(pp):
        for tp_rank in range(tp):
            rank = pp_rank * tp + tp_rank
            meta = {"schema_version": SCHEMA_VERSION, "contract": CONTRACT, "seed": seed, "model": mc,
                    "topology": {"tp": tp, "pp": pp}, "tp_rank": tp_rank, "pp_rank": pp_rank}
            p = out_dir / f"ours_tp{tp}_pp{pp}_rank{rank}.pt"
            torch.save(dict(meta, padded_vocab=padded_vocab,
                            state_dict=shard_state(ours_full, mc, tp, tp_rank, pp, pp_rank)), p)
            files[f"ours_rank{rank}"] = p
            if mc["vocab_size"] % tp == 0:   # the reference shards the exact vocabulary (V % tp == 0 required)
                p = out_dir / f"reference_tp{tp}_pp{pp}_rank{rank}.pt"
                torch.save(dict(meta, state_dict=shard_state(full, mc, tp, tp_rank, pp, pp_rank)), p)
                files[f"reference_rank{rank}"] = p
    tokens, labels = next_token_batches(num_batches, batch_size, mc["max_seq_len"], mc["vocab_size"], seed + 1,
                                        pattern, effective_vocab)
    files["batches"] = out_dir / "next_token_batches.pt"
    torch.save({"schema_version": SCHEMA_VERSION, "contract": CONTRACT, "seed": seed + 1, "input_ids": tokens,
                "labels": labels, "pattern": pattern}, files["batches"])
    manifest = {"schema_version": SCHEMA_VERSION, "contract": CONTRACT, "seed": seed, "model": mc,
                "topology": {"tp": tp, "pp": pp}, "padded_vocab": padded_vocab,
                "reference_chunks": mc["vocab_size"] % tp == 0,
                "batch_shape": list(tokens.shape), "pattern": pattern, "effective_vocab": effective_vocab,
                "files": {k: {"path": v.name, "sha256": sha256_file(v), "bytes": v.stat().st_size}
                          for k, v in files.items()}}
    (out_dir / "manifest.json").write_text(json.dumps(manifest, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    return manifest


def verify(out_dir) -> list:
    """Checksum problems of a frozen artifact directory (empty = intact)."""
    out_dir = Path(out_dir)
    try:
        manifest = json.loads((out_dir / "manifest.json").read_text(encoding="utf-8"))
    except (OSError, ValueError) as exc:
        return [f"cannot read manifest: {exc}"]
    errors = []
    for key, f in manifest["files"].items():
        p = out_dir / f["path"]
        if not p.is_file():
            errors.append(f"{key}: missing {f['path']}")
        elif sha256_file(p) != f["sha256"]:
            errors.append(f"{key}: checksum mismatch {f['path']}")
    return errors


def load_chunk(out_dir, impl, rank, tp, pp):
    """(state_dict, meta) of one rank's chunk after verifying the whole artifact."""
    errors = verify(out_dir)
    if errors:
        raise ValueError("artifact verification failed: " + "; ".join(errors))
    obj = torch.load(Path(out_dir) / f"{impl}_tp{tp}_pp{pp}_rank{rank}.pt", map_location="cpu", weights_only=True)
    if obj.get("contract") != CONTRACT:
        raise ValueError("artifact contract mismatch")
    return obj["state_dict"], obj


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--output-dir", required=True)
    ap.add_argument("--preset", default="gpt-125m")
    ap.add_argument("--seq-len", type=int)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--pp", type=int, default=1)
    ap.add_argument("--batches", type=int, default=64)
    ap.add_argument("--batch-size", type=int, default=4)
    ap.add_argument("--seed", type=int, default=20260818)
    ap.add_argument("--pattern", default="next_token", choices=("next_token", "shift", "identity"))
    ap.add_argument("--effective-vocab", type=int, default=None)
    args = ap.parse_args(argv)
    from ..config import PRESETS
    mc = _model_dict(PRESETS[args.preset])
    if args.seq_len:
        mc["max_seq_len"] = args.seq_len
    try:
        m = freeze(args.output_dir, mc, args.tp, args.pp, args.batches, args.batch_size, args.seed,
                   pattern=args.pattern, effective_vocab=args.effective_vocab)
    except ValueError as exc:
        ap.error(str(exc))
    print(json.dumps(m, indent=2, sort_keys=True))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
