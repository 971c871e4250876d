"""Compute-only benchmark of one implementation on frozen artifacts.

Both implementations load the same frozen weights (``harness.artifacts``)
and consume the same fixed next-token batches, ``m`` microbatches per
optimizer update (loss / m).  Warm-up updates are untimed; the measured
updates are bracketed by a barrier and ``torch.cuda.synchronize`` and timed
with CUDA events; the reported time is the max over ranks.  With
``--phase-timing`` each phase (forward+loss, backward, optimizer) is also
timed with CUDA events (a diagnostic, never a throughput substitute; only
for pp = 1).  Rank 0 prints a JSON report and the ``Throughput:`` /
``Peak memory:`` / ``Final loss:`` lines that ``harness.bundle`` parses.

    python -m torch.distributed.run --nproc-per-node 2 -m mini_megatron_b200.harness.fair_bench \\
        --implementation ours --artifact-dir A --tp 2 --num-updates 20 --warmup-updates 3

Reference: experiments/run_fair_tp1_benchmark.py:33-114, experiments/run_fair_tp2_benchmark.py:60-182,
experiments/run_fair_pp_benchmark.py:105-176.
"""
from __future__ import annotations

import argparse
import contextlib
import datetime
import io
import json
import os
from pathlib import Path

import torch
import torch.distributed as dist

from .artifacts import load_chunk
from .contract import CONTRACT


def _init(device_type):
    kw = {}
    if "RANK" not in os.environ:
        # a lone process: rendezvous through a private file instead of a TCP port that may be taken
        import tempfile
        os.environ.update(RANK="0", LOCAL_RANK="0", WORLD_SIZE="1")
        fd, path = tempfile.mkstemp(prefix="mmb_fair_bench_rdzv_")
        os.close(fd)
        os.unlink(path)
        kw = dict(init_method=f"file://{path}", rank=0, world_size=1)
    local = int(os.environ["LOCAL_RANK"])
    if device_type == "cuda":
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local), **kw)
        return torch.device("cuda", local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300), **kw)
    return torch.device("cpu")


class _Timer:
    def __init__(self, device, enabled):
        self.enabled = enabled and device.type == "cuda"
        self.records = {}

    @contextlib.contextmanager
    def phase(self, name):
        if not self.enabled:
            yield
            return
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        yield
        e.record()
        self.records.setdefault(name, []).append((s, e))

    def report(self):
        return {k: {"milliseconds_total": sum(s.elapsed_time(e) for s, e in v), "event_pairs": len(v)}
                for k, v in self.records.items()}


def build_ours(args, device, mc, state, timer):
    from ..config import GPTConfig
    from ..training import TrainConfig, Trainer
    cfg = TrainConfig(model=GPTConfig(**mc), micro_batch_size=args.batch_size, seq_len=mc["max_seq_len"],
                      num_microbatches=args.microbatches_per_update, tp=args.tp, pp=args.pp,
                      sequence_parallel=args.sequence_parallel, zero1=args.zero1, lr=6e-4, weight_decay=0.1,
                      warmup_steps=0, num_steps=10 ** 6)
    tr = Trainer(cfg, device=device)
    with torch.no_grad():
        for n, p in tr.model.named_parameters():
            p.copy_(state[n])
    seen = set()
    for p in tr.model.parameters():
        buf = getattr(p, "_mmb_buffer", None)
        if buf is not None and id(buf) not in seen:
            seen.add(id(buf))
            buf.refresh_bf16()
    if hasattr(tr.optimizer, "refresh_from_params"):
        tr.optimizer.refresh_from_params()

    def update(tokens, labels):
        if args.pp > 1 or not timer.enabled:
            return tr.train_step(tokens, labels, (labels != -100).float())
        # same phases as Trainer.train_step, each bracketed by CUDA events
        m = tokens.shape[0]
        masks = (labels != -100).float()
        tr.optimizer.zero_grad()
        tr.grad_sync.reset()
        total = 0.0
        for mb in range(m):
            tr.grad_sync.overlap = cfg.dp_overlap if mb == m - 1 else False
            with timer.phase("forward_loss"):
                _, loss = tr.model(tokens[mb], labels[mb], masks[mb])
            with timer.phase("backward"):
                (loss / m).backward()
            total = total + loss.detach()
        tr.grad_sync.overlap = cfg.dp_overlap
        with timer.phase("optimizer"):
            if not cfg.zero1 and tr.dp_impl != "fused":
                tr.grad_sync.finish()
            if tr.sp_params:
                from ..parallel.data_parallel import allreduce_sequence_parallel_grads
                allreduce_sequence_parallel_grads(tr.sp_params, tr.mpu["tp_group"])
            tr.optimizer.step()
            tr.scheduler.step()
        return total / m

    return update, tr.mpu


def build_reference(args, device, mc, state, timer):
    import sys
    ref = Path(__file__).resolve().parents[2] / "baseline" / "_ref"
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    import config as rcfg
    for k, v in (("NUM_LAYERS", "num_layers"), ("HIDDEN_SIZE", "hidden_size"),
                 ("NUM_ATTENTION_HEADS", "num_attention_heads"), ("FFN_HIDDEN_SIZE", "ffn_hidden_size"),
                 ("MAX_SEQ_LEN", "max_seq_len"), ("VOCAB_SIZE", "vocab_size")):
        setattr(rcfg, k, mc[v])
    from model.embedding import Embedding
    from model.loss import CrossEntropyLoss
    from model.transformer import GPT, Decoder, DecoderLayer
    from parallel.data_parallel import allreduce_grads
    from parallel.pipeline_parallel import train_pipeline_1f1b
    from parallel.process_groups import init_model_parallel, set_model_parallel
    from parallel.tensor_parallel import ColumnParallelLinear
    mpu = init_model_parallel(args.tp, args.pp)
    set_model_parallel(mpu)
    V, H, S = mc["vocab_size"], mc["hidden_size"], mc["max_seq_len"]
    NH, F, L = mc["num_attention_heads"], mc["ffn_hidden_size"], mc["num_layers"]
    amp = torch.autocast(device.type, dtype=torch.bfloat16) if args.amp else contextlib.nullcontext()
    B = args.batch_size
    if args.pp == 1:
        model = GPT(Embedding(V, H, S), Decoder(H, NH, F, L), torch.nn.LayerNorm(H),
                    ColumnParallelLinear(H, V, bias=False, gather_output=True), CrossEntropyLoss()).to(device)
        model.load_state_dict(state, strict=True)
        opt = torch.optim.AdamW(model.parameters(), lr=6e-4, weight_decay=0.1, fused=args.fused)

        def update(tokens, labels):
            m = tokens.shape[0]
            opt.zero_grad(set_to_none=True)
            total = 0.0
            for mb in range(m):
                mask = (labels[mb] != -100).float()
                with timer.phase("forward_loss"), amp:
                    _, loss = model(tokens[mb], labels[mb], mask)
                with timer.phase("backward"):
                    (loss / m).backward()
                total = total + loss.detach()
            with timer.phase("optimizer"):
                allreduce_grads(model, mpu.get("dp_group"))
                opt.step()
            return total / m   # mean microbatch loss, as Trainer.train_step reports
        return update, mpu

    pp_rank = mpu["pp_rank"]
    per = L // args.pp
    start = pp_rank * per
    end = start + per if pp_rank < args.pp - 1 else L
    last = pp_rank == args.pp - 1
    mods = torch.nn.Module()
    if pp_rank == 0:
        mods.embedding = Embedding(V, H, S)
    mods.decoder_layers = torch.nn.ModuleList([DecoderLayer(H, NH, F) for _ in range(start, end)])
    if last:
        mods.ln_f = torch.nn.LayerNorm(H)
        mods.lm_head = ColumnParallelLinear(H, V, bias=False, gather_output=True)
    mods.to(device)
    mods.load_state_dict(state, strict=True)
    opt = torch.optim.AdamW(mods.parameters(), lr=6e-4, weight_decay=0.1, fused=args.fused)
    sched = torch.optim.lr_scheduler.LambdaLR(opt, lambda s: 1.0)
    loss_fn = CrossEntropyLoss().to(device) if last else None

    def update(tokens, labels):
        m = tokens.shape[0]
        it = iter([(tokens[i], labels[i]) for i in range(m)])
        with contextlib.redirect_stdout(io.StringIO()):
            train_pipeline_1f1b(getattr(mods, "embedding", None), mods.decoder_layers, getattr(mods, "ln_f", None),
                                getattr(mods, "lm_head", None), loss_fn, opt, sched, it, B, S, V, device, m, pp_rank,
                                args.pp, dist.get_rank(), H, args.tp, 10 ** 9, mpu.get("dp_group"), amp)
        return None
    return update, mpu


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--implementation", choices=("ours", "reference"), required=True)
    ap.add_argument("--artifact-dir", required=True)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--pp", type=int, default=1)
    ap.add_argument("--sequence-parallel", action="store_true")
    ap.add_argument("--zero1", action="store_true")
    ap.add_argument("--microbatches-per-update", type=int, default=1)
    ap.add_argument("--num-updates", type=int, default=20)
    ap.add_argument("--warmup-updates", type=int, default=3)
    ap.add_argument("--amp", action="store_true", help="bf16 autocast for the reference")
    ap.add_argument("--fused", action="store_true", help="AdamW(fused=True) for the reference")
    ap.add_argument("--phase-timing", action="store_true")
    ap.add_argument("--report-losses", action="store_true")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    args = ap.parse_args(argv)
    device = _init(torch.device(args.device).type)
    world = dist.get_world_size()
    if world % (args.tp * args.pp):
        ap.error("world size must be a multiple of tp * pp")
    dp = world // (args.tp * args.pp)
    rank = dist.get_rank()
    tp_rank, pp_rank = rank % args.tp, (rank // args.tp) % args.pp
    dp_rank = rank // (args.tp * args.pp)
    chunk_rank = pp_rank * args.tp + tp_rank
    state, meta = load_chunk(args.artifact_dir, args.implementation, chunk_rank, args.tp, args.pp)
    if meta["topology"] != {"tp": args.tp, "pp": args.pp}:
        ap.error(f"artifact topology {meta['topology']} != requested tp={args.tp} pp={args.pp}")
    mc = meta["model"]
    data = torch.load(Path(args.artifact_dir) / "next_token_batches.pt", map_location="cpu", weights_only=True)
    if data.get("contract") != CONTRACT:
        raise ValueError("data contract mismatch")
    m = args.microbatches_per_update
    need = (args.warmup_updates + args.num_updates) * m * dp
    if data["input_ids"].size(0) < need:
        raise ValueError(f"artifact has {data['input_ids'].size(0)} batches, {need} needed")
    ids, labs = data["input_ids"], data["labels"]
    args.batch_size = ids.size(1)
    timer = _Timer(device, False)
    build = build_ours if args.implementation == "ours" else build_reference
    update, _ = build(args, device, mc, state, timer)

    def batch(u):
        idx = [(u * m + mb) * dp + dp_rank for mb in range(m)]
        return ids[idx].to(device), labs[idx].to(device)

    losses = []
    for u in range(args.warmup_updates):
        loss = update(*batch(u))
        if loss is not None:
            losses.append(float(loss))
    timer.enabled = args.phase_timing and args.pp == 1 and device.type == "cuda"
    if device.type == "cuda":
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats(device)
    dist.barrier()
    inputs = [batch(u) for u in range(args.warmup_updates, args.warmup_updates + args.num_updates)]
    if device.type == "cuda":
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
    import time
    t0 = time.perf_counter()
    last = None
    for tok, lab in inputs:
        last = update(tok, lab)
        if args.report_losses and last is not None:
            losses.append(float(last))
    if device.type == "cuda":
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e)
    else:
        ms = (time.perf_counter() - t0) * 1e3
    dist.barrier()
    t = torch.tensor([ms], dtype=torch.float64, device=device if device.type == "cuda" else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t)
    final = torch.tensor([float(last) if last is not None else float("nan")], dtype=torch.float64,
                         device=t.device)
    finals = [torch.zeros_like(final) for _ in range(world)]
    dist.all_gather(finals, final)
    final_loss = next((float(x) for x in finals if not torch.isnan(x).any()), float("nan"))
    phases = timer.report() if timer.enabled else None
    gathered = [None] * world
    dist.all_gather_object(gathered, {"rank": rank, "phases": phases,
                                      "peak_memory_gb": (torch.cuda.max_memory_allocated(device) / 2 ** 30
                                                         if device.type == "cuda" else 0.0)})
    if rank == 0:
        tokens_per_update = args.batch_size * mc["max_seq_len"] * m * dp
        tput = tokens_per_update * args.num_updates / (ms / 1e3)
        rep = {"implementation": args.implementation, "contract": CONTRACT,
               "topology": {"tp": args.tp, "pp": args.pp, "dp": dp}, "model": mc,
               "num_updates": args.num_updates, "warmup_updates": args.warmup_updates,
               "microbatches_per_update": m, "micro_batch_size": args.batch_size,
               "tokens_per_update": tokens_per_update, "elapsed_seconds_max_over_ranks": ms / 1e3,
               "throughput_tok_s": tput, "peak_memory_gb": max(g["peak_memory_gb"] for g in gathered),
               "final_loss": final_loss, "amp": args.amp, "fused": args.fused,
               "phase_timing": [g for g in gathered] if args.phase_timing else None,
               "timing": "CUDA events, max over ranks" if device.type == "cuda" else "host clock (CPU)"}
        if args.report_losses:
            rep["losses"] = losses
        print(json.dumps(rep, sort_keys=True))
        print(f"Throughput:      {tput:,.0f} tok/s")
        print(f"Peak memory:     {rep['peak_memory_gb']:.2f} GB/GPU")
        print(f"Final loss:      {final_loss:.6f}")
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
