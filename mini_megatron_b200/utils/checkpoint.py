"""Checkpointing.

``save_checkpoint`` / ``load_checkpoint`` keep the reference's single-file
layout exactly (checkpoint.py:5-21): ``{"model_state", "optimizer_state",
"scheduler_state", "step"}`` via ``torch.save`` / ``torch.load(weights_only=True)``.

``save_distributed_checkpoint`` / ``load_distributed_checkpoint`` add what a
(dp, pp, tp) run needs: one file per (tp, pp) model shard written by DP rank
0, one optimizer file per DP rank when the optimizer state is sharded
(ZeRO-1), a JSON manifest with the topology and a SHA-256 of every file.  The
loader validates the topology and the checksums and raises
``CheckpointError`` on any mismatch or truncated file.  Writes go to a
temporary name and are renamed into place, so a crash never leaves a
half-written file under the final name.  The bf16 GEMM shadows are rebuilt
on load, never saved.
"""
from __future__ import annotations

import hashlib
import json
import os

import torch
import torch.distributed as dist

SCHEMA_VERSION = 1


class CheckpointError(RuntimeError):
    pass


def save_checkpoint(model, optimizer, scheduler, step, path):
    d = os.path.dirname(path)
    os.makedirs(d if d else ".", exist_ok=True)
    state = {
        "model_state": model.state_dict(),
        "optimizer_state": optimizer.state_dict(),
        "scheduler_state": scheduler.state_dict(),
        "step": step,
    }
    _atomic_save(state, path)


def load_checkpoint(model, optimizer, scheduler, path, device):
    state = torch.load(path, map_location=device, weights_only=True)
    model.load_state_dict(state["model_state"])
    optimizer.load_state_dict(state["optimizer_state"])
    scheduler.load_state_dict(state["scheduler_state"])
    _refresh_shadows(model)
    return state["step"]


def _refresh_shadows(model):
    seen = set()
    for p in model.parameters():
        buf = getattr(p, "_mmb_buffer", None)
        if buf is not None and id(buf) not in seen:
            seen.add(id(buf))
            buf.refresh_bf16()


def _atomic_save(obj, path):
    tmp = path + ".tmp"
    torch.save(obj, tmp)
    os.replace(tmp, path)


def _sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def _names(mpu):
    tp, pp, dp = (mpu["tp_rank"], mpu["pp_rank"], mpu["dp_rank"]) if mpu else (0, 0, 0)
    return f"model_tp{tp:02d}_pp{pp:03d}.pt", f"optim_tp{tp:02d}_pp{pp:03d}_dp{dp:03d}.pt"


def _topology(mpu):
    if not mpu:
        return {"tp": 1, "pp": 1, "dp": 1}
    return {"tp": mpu["tp_size"], "pp": mpu["pp_size"], "dp": mpu["dp_size"]}


def save_distributed_checkpoint(directory, model, optimizer, scheduler, step, mpu=None, sharded_optimizer=False):
    """Write this rank's part of a distributed checkpoint.

    The optimizer file is written per DP rank when ``sharded_optimizer`` is set
    or when the optimizer itself reports that each DP rank holds only its own
    slice of the state (``optimizer.state_is_sharded``: ZeRO-1 and the fused-DP
    optimizer with dp > 1); otherwise DP rank 0 writes the one shared copy.
    """
    os.makedirs(directory, exist_ok=True)
    sharded_optimizer = bool(sharded_optimizer or getattr(optimizer, "state_is_sharded", False))
    model_name, optim_name = _names(mpu)
    dp_rank = mpu["dp_rank"] if mpu else 0
    written = {}
    if dp_rank == 0:
        p = os.path.join(directory, model_name)
        _atomic_save({"model_state": model.state_dict(), "step": step, "schema_version": SCHEMA_VERSION,
                      "topology": _topology(mpu)}, p)
        written[model_name] = _sha256(p)
    if dp_rank == 0 or sharded_optimizer:
        p = os.path.join(directory, optim_name)
        _atomic_save({"optimizer_state": optimizer.state_dict(), "scheduler_state": scheduler.state_dict(),
                      "step": step}, p)
        written[optim_name] = _sha256(p)
    # gather every rank's file hashes into one manifest written by global rank 0
    if dist.is_initialized() and dist.get_world_size() > 1:
        allw = [None] * dist.get_world_size()
        dist.all_gather_object(allw, written)
        written = {k: v for w in allw for k, v in w.items()}
    if not dist.is_initialized() or dist.get_rank() == 0:
        manifest = {"schema_version": SCHEMA_VERSION, "step": step, "topology": _topology(mpu),
                    "sharded_optimizer": bool(sharded_optimizer), "files": written}
        tmp = os.path.join(directory, "manifest.json.tmp")
        with open(tmp, "w") as f:
            json.dump(manifest, f, indent=1, sort_keys=True)
        os.replace(tmp, os.path.join(directory, "manifest.json"))
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def load_distributed_checkpoint(directory, model, optimizer, scheduler, mpu=None, device="cpu"):
    mpath = os.path.join(directory, "manifest.json")
    try:
        with open(mpath) as f:
            manifest = json.load(f)
    except (OSError, ValueError) as exc:
        raise CheckpointError(f"cannot read checkpoint manifest {mpath}: {exc}") from exc
    if manifest.get("schema_version") != SCHEMA_VERSION:
        raise CheckpointError(f"unsupported checkpoint schema {manifest.get('schema_version')}")
    if manifest["topology"] != _topology(mpu):
        raise CheckpointError(f"checkpoint topology {manifest['topology']} != current {_topology(mpu)}")
    model_name, optim_name = _names(mpu)
    if not manifest["sharded_optimizer"]:
        optim_name = optim_name.rsplit("_dp", 1)[0] + "_dp000.pt"
    states = []
    for name in (model_name, optim_name):
        path = os.path.join(directory, name)
        want = manifest["files"].get(name)
        if want is None or not os.path.exists(path):
            raise CheckpointError(f"checkpoint file {name} missing")
        if _sha256(path) != want:
            raise CheckpointError(f"checkpoint file {name} is corrupt (checksum mismatch)")
        try:
            states.append(torch.load(path, map_location=device, weights_only=True))
        except Exception as exc:  # noqa: BLE001 - any unpickling failure is a corrupt file
            raise CheckpointError(f"checkpoint file {name} cannot be loaded: {exc}") from exc
    mstate, ostate = states
    model.load_state_dict(mstate["model_state"])
    optimizer.load_state_dict(ostate["optimizer_state"])
    scheduler.load_state_dict(ostate["scheduler_state"])
    _refresh_shadows(model)
    return manifest["step"]
