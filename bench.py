"""Headline benchmark: GPT-125M training tokens/s on N B200s (DP=N, weak scaling).

    python bench.py --gpus N --steps K --warmup W [--impl ours|reference] [--config NAME]

For N > 1 launch one process per GPU:
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N --steps K --warmup W

Config: GPT-125M (12 layers, hidden 768, 12 heads, FFN 3072,
vocab 50257, learned positions, pre-LN, GELU, no bias), TP=1 PP=1 DP=N,
micro-batch 16 per GPU, seq 1024, bf16 compute with fp32 AdamW, synthetic
uniform-random tokens with next-token labels, random N(0, 0.02) init.

``--config`` selects the other BASELINE configs (dp = N / (tp * pp)):
gpt125m-tp2pp2 (125M, TP2 PP2, 8 microbatches of 8 x 1024, sequence parallel),
gpt1.3b-tp8sp (1.3B, TP8 with sequence parallelism, micro-batch 4 x 2048) and
gpt6.7b-tp4pp2 (6.7B, TP4 PP2, 16 microbatches of 2 x 2048, ZeRO-1 when dp > 1).
The reference arm runs the same shapes through its own modules (no sequence
parallelism: the reference does not wire it) and, for pp > 1, its own
``train_pipeline_1f1b``.

Timing: W untimed warm-up steps, then EXACTLY K steps bracketed by a barrier
and torch.cuda.synchronize() on both sides, timed with CUDA events on the
launching stream; the reported time is the MAX over ranks.  A step's working
set (16384 tokens x 50K-vocab logits, 1.6 GB) is far larger than the 126 MB
L2, so no explicit flush is needed between steps.  ``value`` is the
device-timed rate with each step's batch already resident; ``e2e`` is the
same K steps through the public ``Trainer.train_step`` API with the batch
copied from pinned host memory every step and the loss read back to the host
every step.  SM clocks and throttle reasons are sampled with nvidia-smi
during the timed region.  Rank 0 prints ONE JSON line.

``--impl reference`` runs the unmodified reference (copied into
baseline/_ref) through its own modules and main.py's training-loop steps
(AMP bf16 autocast, AdamW(fused=True), LambdaLR, per-parameter DP
all-reduce), with the same model shape, data and timing.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
METRIC = "GPT train tok/s (device-timed, max over ranks) at 1/2/4/8 B200 vs ref's NCCL"
MODEL = dict(num_layers=12, hidden_size=768, num_attention_heads=12, ffn_hidden_size=3072, max_seq_len=1024,
             vocab_size=50257)
BASELINE_VALUE = None  # the reference publishes no B200 number for this config
M_1_3B = dict(num_layers=24, hidden_size=2048, num_attention_heads=16, ffn_hidden_size=8192, max_seq_len=2048,
              vocab_size=50257)
M_6_7B = dict(num_layers=32, hidden_size=4096, num_attention_heads=32, ffn_hidden_size=16384, max_seq_len=2048,
              vocab_size=50257)
# The BASELINE configs.  tp/pp are per config; dp = N / (tp * pp); a step is one
# optimizer step over m microbatches of mb x seq tokens per DP replica.
CONFIGS = {
    "gpt125m-dp": dict(name="GPT-125M", model=MODEL, tp=1, pp=1, mb=16, m=1, seq=1024, sp=False, zero1=False),
    "gpt125m-tp2pp2": dict(name="GPT-125M", model=MODEL, tp=2, pp=2, mb=8, m=8, seq=1024, sp=True, zero1=False),
    "gpt1.3b-tp8sp": dict(name="GPT-1.3B", model=M_1_3B, tp=8, pp=1, mb=4, m=1, seq=2048, sp=True, zero1=False),
    "gpt6.7b-tp4pp2": dict(name="GPT-6.7B", model=M_6_7B, tp=4, pp=2, mb=2, m=16, seq=2048, sp=True, zero1=True),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="gpt125m-dp",
                    help="BASELINE config: gpt125m-dp (headline), gpt125m-tp2pp2, gpt1.3b-tp8sp, gpt6.7b-tp4pp2")
    ap.add_argument("--tp", type=int, default=None, help="override the config's TP size")
    ap.add_argument("--pp", type=int, default=None, help="override the config's PP size")
    ap.add_argument("--micro-batch-size", type=int, default=None)
    ap.add_argument("--num-microbatches", type=int, default=None)
    ap.add_argument("--seq-len", type=int, default=None)
    ap.add_argument("--tp-impl", default="auto", choices=["auto", "fused", "nccl"])
    ap.add_argument("--dp-impl", default="auto", choices=["auto", "fused", "nccl"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-launch-count", action="store_true")
    args = ap.parse_args()
    c = CONFIGS[args.config]
    args.tp = args.tp or c["tp"]
    args.pp = args.pp or c["pp"]
    args.micro_batch_size = args.micro_batch_size or c["mb"]
    args.num_microbatches = args.num_microbatches or c["m"]
    args.seq_len = args.seq_len or c["seq"]
    args.model = dict(c["model"], max_seq_len=args.seq_len)
    args.model_name = c["name"]
    args.sp = c["sp"]
    args.zero1 = c["zero1"]
    if args.gpus % (args.tp * args.pp):
        raise SystemExit(f"--gpus {args.gpus} is not a multiple of tp*pp = {args.tp * args.pp}")
    args.dp = args.gpus // (args.tp * args.pp)
    return args


def synthetic_batch(B, S, vocab, seed, pin=True, m=1):
    """Uniform-random int64 tokens [m, B, S] with next-token labels (host, pinned)."""
    g = torch.Generator().manual_seed(seed)
    toks = torch.randint(0, vocab, (m, B, S + 1), generator=g)
    tokens, labels = toks[..., :-1].contiguous(), toks[..., 1:].contiguous()
    if pin:
        tokens, labels = tokens.pin_memory(), labels.pin_memory()
    return tokens, labels


def init_dist(n):
    if "RANK" not in os.environ:
        if n != 1:
            raise SystemExit("N > 1 must be launched with torch.distributed.run")
        os.environ.update(RANK="0", LOCAL_RANK="0", WORLD_SIZE="1", MASTER_ADDR="127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29500 + os.getpid() % 1000))
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                            device_id=torch.device("cuda", local))
    if dist.get_world_size() != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={dist.get_world_size()}")
    return dist.get_rank(), local


class ClockSampler:
    """nvidia-smi sampling of SM clock / throttle reasons during the timed region (local rank 0)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, enabled):
        self.enabled, self.proc, self.path = enabled, None, None

    def start(self):
        if not self.enabled:
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-f", self.path], stdout=subprocess.DEVNULL,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self, gpus):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9 and parts[0].isdigit() and int(parts[0]) in gpus:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        clocks = [num(r[1]) for r in rows if num(r[1])]
        loaded = [c for c in clocks if c and c > 0.5 * max(clocks)] or clocks
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": num(rows[0][2]), "reasons": sorted(reasons), "samples": len(rows)}


def max_over_ranks(x):
    t = torch.tensor([float(x)], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def time_steps(step_fn, K):
    dist.barrier()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(K):
        step_fn(i)
    e.record()
    dist.barrier()
    torch.cuda.synchronize()
    return max_over_ranks(s.elapsed_time(e))


# ----------------------------------------------------------------------------- our implementation
def build_ours(args, rank):
    sys.path.insert(0, HERE)
    from mini_megatron_b200.config import GPTConfig
    from mini_megatron_b200.training import TrainConfig, Trainer
    m = args.num_microbatches
    cfg = TrainConfig(model=GPTConfig(**args.model), micro_batch_size=args.micro_batch_size, seq_len=args.seq_len,
                      num_microbatches=m, tp=args.tp, pp=args.pp, sequence_parallel=args.sp and args.tp > 1,
                      zero1=args.zero1 and args.dp > 1, lr=6e-4, weight_decay=0.1, warmup_steps=10, num_steps=1000,
                      tp_impl=args.tp_impl, dp_impl=args.dp_impl)
    trainer = Trainer(cfg)
    dp_rank = trainer.mpu["dp_rank"]
    nb = 4 if m == 1 else 2
    batches = [synthetic_batch(args.micro_batch_size, args.seq_len, args.model["vocab_size"],
                               seed=1000 * dp_rank + i, m=m) for i in range(nb)]

    def step_host(i):
        tok, lab = batches[i % nb]
        return trainer.train_step(tok, lab)

    dev = [(t.cuda(), l.cuda()) for t, l in batches]

    def step_dev(i):
        tok, lab = dev[i % nb]
        return trainer.train_step(tok, lab)

    info = {"tp_impl": trainer.tp_impl, "dp_impl": trainer.dp_impl,
            "sequence_parallel": bool(trainer.mpu["sequence_parallel"]), "zero1": bool(cfg.zero1),
            "cuda_graph": bool(trainer.graph_mode)}
    step_dev.trainer = trainer
    return step_dev, step_host, args.micro_batch_size * args.seq_len * m, info


# ----------------------------------------------------------------------------- reference
def build_reference(args, rank):
    ref = os.path.join(HERE, "baseline", "_ref")
    if not os.path.exists(os.path.join(ref, "main.py")):
        return None
    sys.path.insert(0, ref)
    import contextlib
    import io

    import config as rcfg  # the reference's config module
    tp, pp, m = args.tp, args.pp, args.num_microbatches
    # The reference's VocabParallelEmbedding needs V % tp == 0 (tensor_parallel.py:91-92):
    # at tp > 1 it runs its own default vocabulary, 50304 (config.py), the padded size we compute with too.
    vocab = args.model["vocab_size"] if tp == 1 else 50304
    rcfg.NUM_LAYERS, rcfg.HIDDEN_SIZE = args.model["num_layers"], args.model["hidden_size"]
    rcfg.NUM_ATTENTION_HEADS, rcfg.FFN_HIDDEN_SIZE = args.model["num_attention_heads"], args.model["ffn_hidden_size"]
    rcfg.MAX_SEQ_LEN, rcfg.VOCAB_SIZE = args.seq_len, vocab
    from main import make_lr_lambda
    from model.embedding import Embedding
    from model.loss import CrossEntropyLoss
    from model.transformer import GPT, Decoder, DecoderLayer
    from parallel.data_parallel import allreduce_grads
    from parallel.pipeline_parallel import train_pipeline_1f1b
    from parallel.process_groups import init_model_parallel, set_model_parallel
    from parallel.tensor_parallel import ColumnParallelLinear
    rcfg.enable_tf32()
    mpu = init_model_parallel(tp, pp)
    set_model_parallel(mpu)
    torch.manual_seed(42)
    c = rcfg.get_model_config()
    dev = torch.device("cuda", torch.cuda.current_device())
    V, H, S = c["vocab_size"], c["hidden_size"], c["max_seq_len"]
    NH, F, NL = c["num_attention_heads"], c["ffn_hidden_size"], c["num_layers"]
    amp = torch.autocast(device_type="cuda", dtype=torch.bfloat16)
    B = args.micro_batch_size
    dp_rank = mpu["dp_rank"] if mpu else 0
    nb = 4 if m == 1 else 2
    batches = [synthetic_batch(B, S, V, seed=1000 * dp_rank + i, m=m) for i in range(nb)]
    devb = [(t.to(dev), l.to(dev)) for t, l in batches]
    info = {"tp_impl": "reference (NCCL all-reduce, no sequence parallelism)" if tp > 1 else None,
            "dp_impl": "reference (per-parameter NCCL all-reduce)" if args.dp > 1 else None, "vocab": V}

    if pp == 1:
        mask = torch.ones(B, S, dtype=torch.float32, device=dev)
        model = GPT(Embedding(V, H, S).to(dev), Decoder(H, NH, F, NL).to(dev), torch.nn.LayerNorm(H).to(dev),
                    ColumnParallelLinear(H, V, bias=False, gather_output=True).to(dev), CrossEntropyLoss()).to(dev)
        opt = torch.optim.AdamW(model.parameters(), lr=rcfg.LEARNING_RATE, weight_decay=rcfg.WEIGHT_DECAY,
                                fused=True)
        sched = torch.optim.lr_scheduler.LambdaLR(opt, make_lr_lambda(10, 1000))

        def one(tok, lab):
            opt.zero_grad()
            loss = None
            for mb in range(m):
                with amp:
                    _, loss = model(tok[mb], lab[mb], mask)
                loss.backward()
            allreduce_grads(model, mpu.get("dp_group"))
            opt.step()
            sched.step()
            return loss
    else:
        # main.py's PP branch (main.py:116-160): stage modules + train_pipeline_1f1b, one optimizer step per call
        pp_rank = mpu["pp_rank"]
        per = NL // pp
        start = pp_rank * per
        end = start + per if pp_rank < pp - 1 else NL
        embedding = Embedding(V, H, S).to(dev) if pp_rank == 0 else None
        layers = torch.nn.ModuleList([DecoderLayer(H, NH, F).to(dev) for _ in range(start, end)])
        last = pp_rank == pp - 1
        ln_f = torch.nn.LayerNorm(H).to(dev) if last else None
        lm_head = ColumnParallelLinear(H, V, bias=False, gather_output=True).to(dev) if last else None
        loss_fn = CrossEntropyLoss().to(dev) if last else None
        params = (list(embedding.parameters()) if embedding is not None else []) + list(layers.parameters())
        params += (list(ln_f.parameters()) + list(lm_head.parameters())) if last else []
        opt = torch.optim.AdamW(params, lr=rcfg.LEARNING_RATE, weight_decay=rcfg.WEIGHT_DECAY, fused=True)
        sched = torch.optim.lr_scheduler.LambdaLR(opt, make_lr_lambda(10, 1000))
        g_rank = dist.get_rank()

        def one(tok, lab):
            it = iter([(tok[mb], lab[mb]) for mb in range(m)])
            with contextlib.redirect_stdout(io.StringIO()):   # its per-call report lines
                train_pipeline_1f1b(embedding, layers, ln_f, lm_head, loss_fn, opt, sched, it, B, S, V, dev, m,
                                    pp_rank, pp, g_rank, H, tp, 10 ** 9, mpu.get("dp_group"), amp)
            return None

    def step_dev(i):
        return one(*devb[i % nb])

    def step_host(i):
        t, l = batches[i % nb]
        return one(t.to(dev, non_blocking=True), l.to(dev, non_blocking=True))

    return step_dev, step_host, B * S * m, info


def parallelism_name(args):
    parts = [f"tp{args.tp}"] if args.tp > 1 else []
    parts += [f"pp{args.pp}"] if args.pp > 1 else []
    parts += [f"dp{args.dp}"] if args.dp > 1 or not parts else []
    name = "".join(parts)
    if args.sp and args.tp > 1:
        name += "-sp"
    if args.zero1 and args.dp > 1:
        name += "-zero1"
    return name


def count_launches(step_fn):
    """Kernels launched by one step, split into this package's kernels and others (CUPTI, untimed)."""
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn(0)
        torch.cuda.synchronize()
    ours_names = ("gemm_bf16_sm100", "ln_fwd_kernel", "ln_bwd_kernel", "ln_param", "ce_fwd_kernel", "ce_bwd_kernel",
                  "emb_fwd_kernel", "emb_bwd", "adamw_kernel", "f32_to_bf16_kernel", "flash_attn", "mmb_")
    ours = other = 0
    names = {}
    for ev in prof.events():
        if ev.device_type is not None and str(ev.device_type).endswith("CUDA") and ev.name:
            mine = any(k in ev.name for k in ours_names)
            ours += mine
            other += not mine
            key = ev.name[:60]
            names[key] = names.get(key, 0) + 1
    return ours, other, names


def main():
    args = parse()
    rank, local = init_dist(args.gpus)
    N = args.gpus
    if args.impl == "reference" and args.tp > 1 and args.pp > 1:
        # The reference's own 1F1B with tp > 1 and pp > 1 deadlocked on B200 (NCCL collective time-out after
        # 300 s on every rank, 125M TP2 PP2 DP2 and 6.7B TP4 PP2; record in results/logs/); it is not run again.
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference's 1F1B with tp>1 and pp>1 "
                              "deadlocked on B200 (NCCL collective time-out on every rank); not run again",
                              "config": {"bench_config": args.config, "parallelism": parallelism_name(args)}}))
        dist.destroy_process_group()
        return
    if args.impl == "reference":
        built = build_reference(args, rank)
        if built is None:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref/main.py not present"}))
            dist.destroy_process_group()
            return
    else:
        built = build_ours(args, rank)
    step_dev, step_host, tokens_per_replica, info = built
    K, W = args.steps, args.warmup
    for i in range(W):
        step_dev(i)
    torch.cuda.synchronize()
    sampler = ClockSampler(local == 0)
    sampler.start()
    time.sleep(1.0)  # let nvidia-smi start sampling before the timed region
    ms = time_steps(step_dev, K)
    clocks = sampler.stop(list(range(N)))
    tokens = tokens_per_replica * args.dp * K
    value = tokens / (ms / 1e3)
    e2e = None
    if not args.no_e2e:
        def e2e_step(i):
            loss = step_host(i)
            if loss is not None:
                loss.item()   # device -> host read of the step's result
        t0 = time.perf_counter()
        e2e_ms = time_steps(e2e_step, K)
        wall = max_over_ranks(time.perf_counter() - t0)
        B, S, m = args.micro_batch_size, args.seq_len, args.num_microbatches
        e2e = {"value": round(tokens / (e2e_ms / 1e3), 1), "unit": "tok/s", "ms_per_step": round(e2e_ms / K, 3),
               "wall_s": round(wall, 3), "h2d_bytes_per_step": 2 * m * B * S * 8,
               "d2h_bytes_per_step": 4,
               "api": "mini_megatron_b200.training.Trainer.train_step" if args.impl == "ours" else
               "reference modules + main.py loop"}
    launches = None
    if not args.no_launch_count:
        try:
            tr = getattr(step_dev, "trainer", None)
            if tr is not None:   # count the kernels of one step run eagerly (a replayed graph launches the same set)
                with tr.eager():
                    ours, other, names = count_launches(step_dev)
            else:
                ours, other, names = count_launches(step_dev)
            launches = {"ours_per_step": ours, "other_per_step": other}
            if rank == 0 and os.environ.get("BENCH_KERNEL_LIST"):
                with open(os.environ["BENCH_KERNEL_LIST"], "w") as f:
                    json.dump(names, f, indent=1)
        except Exception as exc:  # noqa: BLE001
            launches = {"error": str(exc)[:200]}
    if rank == 0:
        out = {
            "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": N, "steps": K, "warmup": W,
            "ms_per_step": round(ms / K, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": (round(value / BASELINE_VALUE, 4) if BASELINE_VALUE else None),
            "dtype": "bf16", "data": "synthetic (uniform-random tokens, next-token labels; random N(0,0.02) init)",
            "config": {"model": args.model_name, "global_batch": args.micro_batch_size * args.num_microbatches * args.dp,
                       "seq_len": args.seq_len, "micro_batch": args.micro_batch_size,
                       "num_microbatches": args.num_microbatches, "vocab": args.model["vocab_size"],
                       "parallelism": parallelism_name(args), "bench_config": args.config, **{k: v for k, v in
                                                                                             info.items() if v is not None},
                       "l2": "no flush: per-step working set (>= 1 GB of activations and logits) >> 126 MB L2"},
            "clocks": clocks, "e2e": e2e,
        }
        if args.impl == "ours":
            out["gpu_launches"] = (launches or {}).get("ours_per_step", 0) * K if launches and "ours_per_step" in launches else None
            out["launches_per_step"] = launches
        else:
            out["impl"] = "reference"
            out["reference_flags"] = "--amp --fused (bf16 autocast, AdamW(fused=True)), labels = next token"
            out["launches_per_step"] = launches
        print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
