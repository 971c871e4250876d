"""Command-line training driver (flag-compatible with the reference's main.py).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 main.py --tp T --pp P [--amp] ...

Reference flags kept verbatim (main.py:70-83 of the reference):
``--num-steps --warmup-steps --micro-batch-size --tp --pp --schedule {1f1b,serial}
--log-interval --amp --fused --compile --data-file``.  ``--amp`` selects the bf16
compute path (the only compute dtype of the native kernels; fp32 master
weights and optimizer state are always kept), ``--fused`` and ``--compile`` are
accepted for compatibility (the optimizer is always the fused flat AdamW and
nothing is traced by a compiler).

Extra flags: model shape (``--model`` preset or ``--num-layers`` ...), ``--seq-len``,
``--num-microbatches``, ``--sequence-parallel``, ``--zero1``, ``--recompute``,
``--no-dp-overlap``, ``--save``/``--load`` (distributed checkpoint directory),
``--reference-pp-semantics`` (one optimizer step over ``--num-steps``
microbatches with summed losses, like the reference's PP path).

Report lines keep the reference's format (``step N | loss X``, ``Throughput:``,
``Peak memory:``, ``MFU:``, ``Final loss:``) so log parsers keep working;
throughput is reported both per data-parallel replica (the reference's
definition) and for the whole job.
"""
from __future__ import annotations

import argparse
import dataclasses
import datetime
import json
import os
import time

import torch
import torch.distributed as dist

from mini_megatron_b200 import config as cfgmod
from mini_megatron_b200.config import PRESETS, GPTConfig
from mini_megatron_b200.training import TrainConfig, Trainer, compute_mfu
from mini_megatron_b200.utils.checkpoint import load_distributed_checkpoint, save_distributed_checkpoint


def parse_args(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--num-steps", type=int, default=cfgmod.MAX_TRAIN_STEPS)
    p.add_argument("--warmup-steps", type=int, default=cfgmod.WARMUP_STEPS)
    p.add_argument("--micro-batch-size", type=int, default=cfgmod.MICRO_BATCH_SIZE)
    p.add_argument("--tp", type=int, default=1)
    p.add_argument("--pp", type=int, default=1)
    p.add_argument("--schedule", type=str, default="1f1b", choices=["1f1b", "serial"])
    p.add_argument("--log-interval", type=int, default=10)
    p.add_argument("--amp", action="store_true", help="bf16 compute (always on for the native kernels)")
    p.add_argument("--fused", action="store_true", help="accepted for compatibility; AdamW is always fused")
    p.add_argument("--compile", action="store_true", help="accepted for compatibility; no tracing compiler is used")
    p.add_argument("--data-file", type=str, default=None, help=".pt with input_ids/labels [N, B, S]")
    # extras
    p.add_argument("--model", type=str, default="reference-125m", choices=sorted(PRESETS))
    p.add_argument("--num-layers", type=int)
    p.add_argument("--hidden-size", type=int)
    p.add_argument("--num-attention-heads", type=int)
    p.add_argument("--ffn-hidden-size", type=int)
    p.add_argument("--vocab-size", type=int)
    p.add_argument("--seq-len", type=int)
    p.add_argument("--vocab-pad", type=int, default=None,
                   help="pad the vocabulary tables to a multiple of this times tp (default 128)")
    p.add_argument("--num-microbatches", type=int, default=1)
    p.add_argument("--sequence-parallel", action="store_true")
    p.add_argument("--zero1", action="store_true")
    p.add_argument("--recompute", action="store_true")
    p.add_argument("--no-dp-overlap", action="store_true")
    p.add_argument("--tp-impl", choices=["auto", "fused", "nccl"], default="auto",
                   help="TP collectives: fused into the LN/GEMM kernels (implies SP) or NCCL")
    p.add_argument("--dp-impl", choices=["auto", "fused", "nccl"], default="auto",
                   help="DP gradient sync: fused RS+AdamW+AG kernel over NVLink or NCCL")
    p.add_argument("--kernels", choices=["native", "nccl"], default="native",
                   help="nccl = every collective through NCCL (same as --tp-impl nccl --dp-impl nccl)")
    p.add_argument("--nvtx", action="store_true", help="NVTX ranges per training phase")
    p.add_argument("--json-metrics", action="store_true",
                   help="also print one JSON line: global tok/s (device-timed, max over ranks), per-rank ms")
    p.add_argument("--lr", type=float, default=cfgmod.LEARNING_RATE)
    p.add_argument("--weight-decay", type=float, default=cfgmod.WEIGHT_DECAY)
    p.add_argument("--save", type=str, default=None)
    p.add_argument("--load", type=str, default=None)
    p.add_argument("--identity-labels", action="store_true", help="labels = tokens (the reference's default task)")
    p.add_argument("--reference-pp-semantics", action="store_true")
    return p.parse_args(argv)


def model_config(args) -> GPTConfig:
    base = dataclasses.replace(PRESETS[args.model])
    for f in ("num_layers", "hidden_size", "num_attention_heads", "ffn_hidden_size", "vocab_size"):
        v = getattr(args, f)
        if v is not None:
            setattr(base, f, v)
    if args.seq_len is not None:
        base.max_seq_len = max(base.max_seq_len, args.seq_len)
    if args.vocab_pad is not None:
        if args.vocab_pad < 1:
            raise SystemExit("--vocab-pad must be positive")
        base.vocab_pad_multiple = args.vocab_pad
    return base


def data_iterator(args, B, S, V, dp_rank, m):
    """Yields [m, B, S] token/label batches: preloaded file first, then random (seed 42 + dp_rank*10000)."""
    if args.data_file:
        d = torch.load(args.data_file, map_location="cpu", weights_only=True)
        ids, labels = d["input_ids"], d["labels"]
        for i in range(0, ids.size(0) - m + 1, m):
            yield ids[i:i + m].contiguous(), labels[i:i + m].contiguous()
    g = torch.Generator().manual_seed(42 + dp_rank * 10000)
    while True:
        if args.identity_labels:
            tok = torch.randint(0, V, (m, B, S), generator=g)
            yield tok, tok.clone()
        else:
            tok = torch.randint(0, V, (m, B, S + 1), generator=g)
            yield tok[..., :-1].contiguous(), tok[..., 1:].contiguous()


def main(argv=None):
    args = parse_args(argv)
    cfgmod.enable_tf32()
    if "RANK" not in os.environ:
        os.environ.update(RANK="0", LOCAL_RANK="0", WORLD_SIZE="1", MASTER_ADDR="127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29599")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
        device = torch.device("cuda", local)
    else:
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
        device = torch.device("cpu")
    rank = dist.get_rank()
    mcfg = model_config(args)
    S = args.seq_len or mcfg.max_seq_len
    m = args.num_microbatches
    steps = args.num_steps
    if args.reference_pp_semantics and args.pp > 1:
        m, steps = args.num_steps, 1
    tcfg = TrainConfig(model=mcfg, micro_batch_size=args.micro_batch_size, seq_len=S, num_microbatches=m,
                       tp=args.tp, pp=args.pp, sequence_parallel=args.sequence_parallel, zero1=args.zero1,
                       schedule=args.schedule, lr=args.lr, weight_decay=args.weight_decay,
                       warmup_steps=args.warmup_steps, num_steps=steps + args.warmup_steps,
                       dp_overlap=not args.no_dp_overlap, recompute=args.recompute,
                       average_microbatches=not args.reference_pp_semantics,
                       tp_impl="nccl" if args.kernels == "nccl" else args.tp_impl,
                       dp_impl="nccl" if args.kernels == "nccl" else args.dp_impl, nvtx=args.nvtx)
    trainer = Trainer(tcfg, device=device)
    mpu = trainer.mpu
    start_step = 0
    if args.load:
        start_step = load_distributed_checkpoint(args.load, *trainer.state_for_checkpoint(), mpu=mpu, device=device)
    it = data_iterator(args, args.micro_batch_size, S, mcfg.vocab_size, mpu["dp_rank"], m)
    is_reporter = mpu["pp_rank"] == mpu["pp_size"] - 1 and mpu["tp_rank"] == 0 and mpu["dp_rank"] == 0
    warm = 0 if args.reference_pp_semantics else args.warmup_steps
    for _ in range(warm):
        trainer.train_step(*next(it))
    if device.type == "cuda":
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
    dist.barrier()
    t0 = time.perf_counter()
    if device.type == "cuda":
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
    losses = []
    for step in range(steps):
        loss = trainer.train_step(*next(it))
        if loss is not None and ((step + 1) % args.log_interval == 0 or step == steps - 1):
            lv = loss.item()
            losses.append(lv)
            if is_reporter and (step + 1) % args.log_interval == 0:
                print(f"step {step + 1:4d} | loss {lv:.4f}", flush=True)
    if device.type == "cuda":
        ev1.record()
        torch.cuda.synchronize()
    dist.barrier()
    elapsed = time.perf_counter() - t0
    device_ms = ev0.elapsed_time(ev1) if device.type == "cuda" else elapsed * 1e3
    per_rank = [None] * dist.get_world_size()
    if args.json_metrics:
        dist.all_gather_object(per_rank, {"rank": rank, "device_ms": device_ms,
                                          "peak_gb": (torch.cuda.max_memory_allocated() / 1024 ** 3
                                                      if device.type == "cuda" else 0.0)})
    if args.save:
        save_distributed_checkpoint(args.save, *trainer.state_for_checkpoint(), start_step + steps, mpu=mpu,
                                    sharded_optimizer=args.zero1 or trainer.dp_impl == "fused")
    if is_reporter:
        B = args.micro_batch_size
        per_replica = B * S * m * steps / elapsed
        peak = torch.cuda.max_memory_allocated() / 1024 ** 3 if device.type == "cuda" else 0.0
        mfu = compute_mfu(dict(num_layers=mcfg.num_layers, hidden_size=mcfg.hidden_size, vocab_size=mcfg.vocab_size),
                          S, B, args.tp, args.pp, elapsed, steps * m)
        print(f"\n{'=' * 60}")
        print(f"Mini-Megatron-B200 Results (TP={args.tp}, PP={args.pp}, DP={mpu['dp_size']}, "
              f"SP={'on' if mpu['sequence_parallel'] else 'off'}, ZeRO-1={'on' if args.zero1 else 'off'}, BF16)")
        print(f"{'=' * 60}")
        print(f"Model:           {mcfg.hidden_size}hid {mcfg.num_layers}lay {mcfg.num_attention_heads}head")
        print(f"Micro batch:     {B}  |  Seq len: {S}  |  Steps: {steps}  |  Micro-batches/step: {m}")
        print(f"{'-' * 60}")
        print(f"Throughput:      {per_replica:,.0f} tok/s")
        print(f"Global tput:     {per_replica * mpu['dp_size']:,.0f} tok/s")
        print(f"Peak memory:     {peak:.2f} GB/GPU")
        print(f"MFU:             {mfu:.2%}")
        if losses:
            print(f"Final loss:      {losses[-1]:.4f}")
        print(f"{'=' * 60}\n", flush=True)
    if args.json_metrics and rank == 0:
        B = args.micro_batch_size
        worst = max(r["device_ms"] for r in per_rank)
        print(json.dumps({"event": "summary", "global_tokens_per_s": B * S * m * steps * mpu["dp_size"] / (worst / 1e3),
                          "device_ms_max_over_ranks": worst, "steps": steps, "micro_batches_per_step": m,
                          "tp": args.tp, "pp": args.pp, "dp": mpu["dp_size"], "tp_impl": trainer.tp_impl,
                          "dp_impl": trainer.dp_impl, "final_loss": losses[-1] if losses else None,
                          "ranks": per_rank}), flush=True)
    trainer.destroy()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
