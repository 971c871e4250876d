"""Per-kernel time shares of one training step (CUPTI via torch.profiler).

    python -m mini_megatron_b200.utils.step_profile --model gpt-125m --micro-batch-size 16 --seq-len 1024

Runs a few warm-up steps, then profiles ``--steps`` steps and prints, per
kernel name, the number of launches and the share of total kernel time.
Profiled durations are only used for these shares; reported throughput
numbers come from CUDA-event timing without a profiler (bench.py).
"""
import argparse
import collections
import json
import os

import torch
import torch.distributed as dist


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="gpt-125m")
    ap.add_argument("--micro-batch-size", type=int, default=16)
    ap.add_argument("--seq-len", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--json", default=None)
    args = ap.parse_args()
    from mini_megatron_b200.config import PRESETS
    from mini_megatron_b200.training import TrainConfig, Trainer, synthetic_batch
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29577")
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
    cfg = TrainConfig(model=PRESETS[args.model], micro_batch_size=args.micro_batch_size, seq_len=args.seq_len)
    t = Trainer(cfg)
    tok, lab = synthetic_batch(1, args.micro_batch_size, args.seq_len, cfg.model.vocab_size, seed=0)
    tok, lab = tok.cuda(), lab.cuda()
    for _ in range(3):
        t.train_step(tok, lab)
    torch.cuda.synchronize()
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.steps):
            t.train_step(tok, lab)
        torch.cuda.synchronize()
    agg = collections.defaultdict(lambda: [0, 0.0])
    for ev in prof.events():
        if ev.device_type is not None and str(ev.device_type).endswith("CUDA"):
            name = ev.name
            agg[name][0] += 1
            agg[name][1] += ev.device_time_total if hasattr(ev, "device_time_total") else ev.cuda_time_total
    total = sum(v[1] for v in agg.values())
    rows = sorted(agg.items(), key=lambda kv: -kv[1][1])
    out = []
    for name, (n, us) in rows:
        out.append({"kernel": name[:110], "launches_per_step": n / args.steps, "us_per_step": us / args.steps,
                    "share": us / total})
    print(f"total kernel time per step: {total / args.steps / 1e3:.3f} ms")
    for r in out[:40]:
        print(f"{r['share'] * 100:6.2f}%  {r['us_per_step']:9.1f} us  x{r['launches_per_step']:5.1f}  {r['kernel']}")
    if args.json:
        with open(args.json, "w") as f:
            json.dump(out, f, indent=1)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
