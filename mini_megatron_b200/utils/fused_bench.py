"""Micro-benchmarks of the fused compute+collective kernels, with their rooflines.

Run under torchrun, one process per GPU (all ranks form one TP group for the
``tp`` case, one DP group for the ``dp`` case):

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m mini_megatron_b200.utils.fused_bench tp --model gpt-1.3b --batch 4 --seq 2048
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m mini_megatron_b200.utils.fused_bench dp --params 162000000

Each case is timed with CUDA events after warm-up (median of ``--iters``);
the reported time is the max over ranks.  The roofline of a fused op is the
slower of its FLOPs at the GEMM peak and the bytes it must move over NVLink at
the per-direction link bandwidth (and, for the memory-bound parts, its HBM
bytes at the copy bandwidth); ``frac`` = roofline time / measured time.
Peaks default to this pool's measurements (``MEASURED_PEAKS.json`` when
present: HBM copy, sustained cuBLAS bf16) and 770 GB/s per direction for a
peer copy.

Cases (``tp``, sequence-parallel dataflow as in parallel/fused_tp.py):
  ln_ag        LayerNorm of the local shard + all-gather push into every rank
  ag_gemm      all-gather-waiting Column GEMM (QKV) on the gathered rows
  gemm_rs      Row GEMM (attention out) pushing partial tiles to their owners + the flag-waiting reduce
Case ``dp``: the bucket kernel reduce-scatter + AdamW + all-gather over ``--params`` parameters.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0


def _peaks():
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"]))
    except (OSError, ValueError, KeyError):
        return 6650.0, 1400.0


def _time(fn, iters, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e))
    t = torch.tensor([statistics.median(ts)], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def _report(rank, name, ms, flops=0.0, nvlink_bytes=0.0, hbm_bytes=0.0, extra=None):
    hbm_gbs, tflops = _peaks()
    t_flop = flops / (tflops * 1e12) * 1e3
    t_link = nvlink_bytes / (NVLINK_GBS * 1e9) * 1e3
    t_hbm = hbm_bytes / (hbm_gbs * 1e9) * 1e3
    roof = max(t_flop, t_link, t_hbm)
    if rank == 0:
        rec = {"case": name, "ms": round(ms, 4), "roofline_ms": round(roof, 4), "frac": round(roof / ms, 3),
               "bound": max((("compute", t_flop), ("nvlink", t_link), ("hbm", t_hbm)), key=lambda kv: kv[1])[0],
               "tflops": round(flops / ms / 1e9, 1) if flops else None,
               "nvlink_gbs": round(nvlink_bytes / ms / 1e6, 1) if nvlink_bytes else None,
               "peaks": {"hbm_gbs": hbm_gbs, "bf16_tflops": tflops, "nvlink_gbs": NVLINK_GBS}}
        rec.update(extra or {})
        print(json.dumps(rec), flush=True)


def bench_tp(args):
    from mini_megatron_b200.config import PRESETS
    from mini_megatron_b200.ops import check_errors, native
    from mini_megatron_b200.parallel.fused_tp import TPWorkspace
    C = native()
    world, rank = dist.get_world_size(), dist.get_rank()
    cfg = PRESETS[args.model]
    H, B, S = cfg.hidden_size, args.batch, args.seq
    ws = TPWorkspace(None if world == 1 else dist.group.WORLD, B, S, H, num_fwd_slots=2)
    rows, rows_l = B * S, B * S // world
    torch.manual_seed(rank)
    x = torch.randn(rows_l, H, device="cuda")
    ln = torch.nn.LayerNorm(H).cuda()
    wqkv = (torch.randn(3 * H // world, H, device="cuda") * 0.02).bfloat16()
    wo = (torch.randn(H, H // world, device="cuda") * 0.02).bfloat16()
    ctx = torch.randn(rows, H // world, device="cuda").bfloat16()
    qkv = torch.empty(rows, 3 * H // world, device="cuda", dtype=torch.bfloat16)
    push = rows_l * H * 2 * (world - 1)
    # LayerNorm + all-gather push
    ms = _time(lambda: ws.ln_fwd_ag(x, ln, 0), args.iters)
    _report(rank, "ln_ag", ms, nvlink_bytes=push, hbm_bytes=rows_l * H * 6 + rows * H * 2,
            extra={"world": world, "rows_local": rows_l, "H": H})
    # all-gather -> GEMM (the gather of the same step overlaps the GEMM's first tiles)

    def ag_gemm():
        full, _, _, e = ws.ln_fwd_ag(x, ln, 1)
        ws.gemm_ag(full, e, wqkv, False, qkv)
    ms = _time(ag_gemm, args.iters)
    _report(rank, "ln_ag+ag_gemm(qkv)", ms, flops=2.0 * rows * (3 * H // world) * H, nvlink_bytes=push,
            extra={"world": world, "M": rows, "N": 3 * H // world, "K": H})
    # GEMM -> reduce-scatter (+ reduce with the residual)

    def gemm_rs():
        e = ws.gemm_rs(ctx, wo, False)
        ws.rs_reduce(e, resid=x)
    ms = _time(gemm_rs, args.iters)
    _report(rank, "gemm_rs(o)+rs_reduce", ms, flops=2.0 * rows * H * (H // world),
            nvlink_bytes=rows * H * 2 * (world - 1) / world, hbm_bytes=rows_l * H * (world * 2 + 8),
            extra={"world": world, "M": rows, "N": H, "K": H // world})
    torch.cuda.synchronize()
    check_errors()
    ws.close()


def bench_dp(args):
    from mini_megatron_b200.ops import check_errors
    from mini_megatron_b200.parallel.fused_dp import FusedDPOptimizer
    world, rank = dist.get_world_size(), dist.get_rank()
    n = args.params
    model = torch.nn.Linear(1, 1, bias=False)
    model.weight = torch.nn.Parameter(torch.zeros(n, 1))
    model.cuda()
    opt = FusedDPOptimizer(model, None if world == 1 else dist.group.WORLD, lr=1e-4,
                           bucket_elems=args.bucket_mb * (1 << 20) // 4, overlap=False, defer_done=True)
    opt.buf.grad.normal_()

    def step():
        opt.reset()
        opt.step()
    ms = _time(step, args.iters)
    own = n / world
    # A 2-D weight is a GEMM weight (kind 0): per element, the owner reads 4 B of gradient from each
    # peer and writes 2 B of bf16 shadow into each peer, so every GPU sends (and receives)
    # (world - 1) * own * 6 bytes.  HBM per GPU: its gradients read once (4n), the bf16 shadows
    # written into it (2n), and the owned master and moments read and written (24 B per element).
    _report(rank, "dp_rs_adamw_ag", ms, nvlink_bytes=(world - 1) * own * 6.0,
            hbm_bytes=6.0 * n + 24.0 * own,
            extra={"world": world, "params": n, "buckets": len(opt.buf.buckets)})
    torch.cuda.synchronize()
    check_errors()
    opt.close()


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("case", choices=["tp", "dp"])
    ap.add_argument("--model", default="gpt-1.3b")
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--params", type=int, default=162_000_000)
    ap.add_argument("--bucket-mb", type=int, default=64)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args(argv)
    if "RANK" not in os.environ:
        os.environ.update(RANK="0", LOCAL_RANK="0", WORLD_SIZE="1", MASTER_ADDR="127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29561")
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        (bench_tp if args.case == "tp" else bench_dp)(args)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
