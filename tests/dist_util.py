"""Helpers for multi-process gloo tests on CPU (spawn + file rendezvous)."""
import os
import tempfile
import traceback

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _entry(rank, world, init_file, fn, args, out_dir, timeout_s):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if root not in sys.path:
        sys.path.insert(0, root)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, init_method=f"file://{init_file}",
                                timeout=datetime.timedelta(seconds=timeout_s))
        result = fn(rank, world, *args)
        torch.save(result, os.path.join(out_dir, f"r{rank}.pt"))
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        with open(os.path.join(out_dir, f"err{rank}.txt"), "w") as f:
            f.write(traceback.format_exc())
        raise


def run_ranks(fn, world, *args, timeout_s=120, expect_fail=False):
    """Run ``fn(rank, world, *args)`` in ``world`` gloo processes; return their results by rank."""
    with tempfile.TemporaryDirectory() as d:
        init_file = os.path.join(d, "rdzv")
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_entry, args=(r, world, init_file, fn, args, d, timeout_s)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout_s + 60)
            if p.is_alive():
                p.kill()
        errs = {}
        for r in range(world):
            e = os.path.join(d, f"err{r}.txt")
            if os.path.exists(e):
                errs[r] = open(e).read()
        if expect_fail:
            return errs, [p.exitcode for p in procs]
        assert not errs, "\n".join(f"rank {r}:\n{t}" for r, t in errs.items())
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        return [torch.load(os.path.join(d, f"r{r}.pt"), weights_only=False) for r in range(world)]
