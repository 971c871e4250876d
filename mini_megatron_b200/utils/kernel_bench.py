"""Kernel micro-benchmarks on the training shapes (CUDA-event timed).

Usage::

    python -m mini_megatron_b200.utils.kernel_bench gemm [--model gpt-125m] [--tokens 16384] [--pairs]
    python -m mini_megatron_b200.utils.kernel_bench epi       # every fused GEMM epilogue, pairs vs one CTA
    python -m mini_megatron_b200.utils.kernel_bench attn      # causal attention vs torch SDPA
    python -m mini_megatron_b200.utils.kernel_bench attn_case --d 64   # one fwd + bwd launch (ncu target)

Each kernel is timed with CUDA events on the launching stream after warm-up,
with a device synchronise on both sides; an L2-sized buffer is rewritten
between iterations so every launch starts cold.  Results are printed as JSON
lines: shape, milliseconds, achieved TFLOP/s (or GB/s) and the same for the
library path (cuBLAS via torch.matmul) as a yardstick.
"""
import argparse
import json

import torch

L2_FLUSH_BYTES = 256 << 20


def _timeit(fn, iters=20, warmup=5, flush=None):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush is not None:
            flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def gemm_shapes(h, ffn, vocab, tokens):
    """(name, M, N, K, a_mn, b_mn, epi) for one layer's fwd/dgrad/wgrad + lm_head."""
    shapes = []
    for name, n_out, k_in in (("qkv", 3 * h, h), ("o", h, h), ("fc1", ffn, h), ("fc2", h, ffn), ("lm_head", vocab, h)):
        shapes.append((name + ".fwd", tokens, n_out, k_in, False, False))
        shapes.append((name + ".dgrad", tokens, k_in, n_out, False, True))
        shapes.append((name + ".wgrad", n_out, k_in, tokens, True, True))
    return shapes


def bench_gemm(args):
    from mini_megatron_b200 import _C

    flush = torch.empty(L2_FLUSH_BYTES // 4, device="cuda")
    cfg = {"gpt-125m": (768, 3072, 50304), "gpt-1.3b": (2048, 8192, 50304), "gpt-6.7b": (4096, 16384, 50304)}[args.model]
    for name, M, N, K, a_mn, b_mn in gemm_shapes(*cfg, args.tokens):
        A = torch.randn(K, M, device="cuda").bfloat16() if a_mn else torch.randn(M, K, device="cuda").bfloat16()
        B = torch.randn(K, N, device="cuda").bfloat16() if b_mn else torch.randn(N, K, device="cuda").bfloat16()
        D = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ours = _timeit(lambda: _C.gemm(A, a_mn, B, b_mn, D, _C.EPI_BF16), flush=flush)
        At = A.t() if a_mn else A
        Bt = B if b_mn else B.t()
        lib = _timeit(lambda: torch.matmul(At, Bt, out=D), flush=flush)
        flops = 2.0 * M * N * K
        rec = {"kernel": "gemm_bf16_sm100", "name": name, "M": M, "N": N, "K": K,
               "ms": round(ours, 4), "tflops": round(flops / ours / 1e9, 1),
               "cublas_ms": round(lib, 4), "cublas_tflops": round(flops / lib / 1e9, 1)}
        if args.tile_widths:  # the same GEMM with each output tile width forced
            for bn in (128, 256):
                t = _timeit(lambda: _C.gemm(A, a_mn, B, b_mn, D, _C.EPI_BF16, bn=bn, cg=1), flush=flush)
                rec[f"bn{bn}_ms"] = round(t, 4)
        if args.pairs:  # one CTA per 128 x 256 tile against a CTA pair per 256 x 256 tile
            D1 = torch.empty_like(D)
            t1 = _timeit(lambda: _C.gemm(A, a_mn, B, b_mn, D1, _C.EPI_BF16, bn=256, cg=1), flush=flush)
            t2 = _timeit(lambda: _C.gemm(A, a_mn, B, b_mn, D, _C.EPI_BF16, bn=256, cg=2), flush=flush)
            torch.cuda.synchronize()
            rec["cta1_ms"], rec["pair_ms"] = round(t1, 4), round(t2, 4)
            rec["pair_tflops"] = round(flops / t2 / 1e9, 1)
            rec["pair_vs_cta1_max_abs_diff"] = float((D.float() - D1.float()).abs().max())
        print(json.dumps(rec), flush=True)
    assert _C.get_error() == 0


def bench_epilogues(args):
    """Every fused GEMM epilogue of a GPT-125M layer step, CUDA-event timed, with CTA pairs
    (the default for these shapes) and with one CTA per tile (cg=1)."""
    from mini_megatron_b200 import _C
    torch.manual_seed(0)
    flush = torch.empty(L2_FLUSH_BYTES // 4, device="cuda")
    T, H, F = args.tokens, 768, 3072
    bf = dict(device="cuda", dtype=torch.bfloat16)
    x, act, dy = torch.randn(T, H, **bf), torch.randn(T, F, **bf), torch.randn(T, H, **bf)
    w1, w2, wo = (torch.randn(F, H, **bf) * 0.02, torch.randn(H, F, **bf) * 0.02, torch.randn(H, H, **bf) * 0.02)
    wqkv, dqkv = torch.randn(3 * H, H, **bf) * 0.02, torch.randn(T, 3 * H, **bf)
    out_f, gp, dpre = torch.empty(T, F, **bf), torch.empty(T, F, **bf), torch.empty(T, F, **bf)
    resid, dx = torch.randn(T, H, device="cuda"), torch.empty(T, H, **bf)
    dw1 = torch.zeros(F, H, device="cuda")
    cases = [
        ("fc1.fwd+gelu", 2 * T * F * H, lambda cg: _C.gemm(x, False, w1, False, out_f, _C.EPI_GELU, aux=gp, cg=cg)),
        ("o.fwd+resid", 2 * T * H * H, lambda cg: _C.gemm(x, False, wo, False, resid, _C.EPI_RESID, resid=resid, cg=cg)),
        ("fc2.fwd+resid", 2 * T * H * F, lambda cg: _C.gemm(act, False, w2, False, resid, _C.EPI_RESID, resid=resid,
                                                           cg=cg)),
        ("fc2.dgrad+dgelu", 2 * T * F * H, lambda cg: _C.gemm(dy, False, w2, True, dpre, _C.EPI_DGELU, aux=gp, cg=cg)),
        ("qkv.dgrad", 2 * T * H * 3 * H, lambda cg: _C.gemm(dqkv, False, wqkv, True, dx, _C.EPI_BF16, cg=cg)),
        ("fc1.wgrad+acc", 2 * T * F * H, lambda cg: _C.gemm(dpre, True, x, True, dw1, _C.EPI_F32_ACC, cg=cg)),
    ]
    for name, flops, fn in cases:
        rec = {"kernel": "gemm_bf16_sm100", "case": name, "tokens": T}
        for cg, key in ((0, "default"), (1, "cta1"), (2, "pair")):
            ms = _timeit(lambda: fn(cg), flush=flush)
            rec[key + "_us"] = round(ms * 1e3, 1)
            rec[key + "_tflops"] = round(flops / ms / 1e9, 1)
        print(json.dumps(rec), flush=True)
    torch.cuda.synchronize()
    assert _C.get_error() == 0


def _attn_views(qkv, B, S, nh, d):
    t = qkv.view(B, S, 3, nh, d)
    return (t[:, :, 0].transpose(1, 2), t[:, :, 1].transpose(1, 2), t[:, :, 2].transpose(1, 2))


def bench_attn(args):
    """Causal attention forward and backward against torch SDPA (the reference's op) on the same GPU.

    Shapes: GPT-125M (B=16, S=1024, 12 heads, d=64) and the d=128 long-sequence case
    (B=4, S=2048, 16 heads, d=128).  Causal FLOPs: forward 2 * B * h * S^2 * d,
    backward 2.5x that.
    """
    from mini_megatron_b200 import _C
    import torch.nn.functional as F
    flush = torch.empty(L2_FLUSH_BYTES // 4, device="cuda")
    shapes = [(16, 1024, 12, 64), (4, 2048, 16, 128)]
    for B, S, nh, d in shapes:
        torch.manual_seed(0)
        qkv = (torch.randn(B * S, 3 * nh * d, device="cuda") * 0.5).bfloat16()
        dout = torch.randn(B * S, nh * d, device="cuda").bfloat16()
        fl = 2.0 * B * nh * S * S * d
        rec = {"kernel": "flash_attn", "B": B, "S": S, "heads": nh, "d": d, "fwd_gflop": round(fl / 1e9, 2)}
        rec["fwd_ms"] = _timeit(lambda: _C.flash_attn_fwd(qkv, B, S, nh, d), flush=flush)
        if hasattr(_C, "flash_attn_fwd_v1"):
            rec["fwd_v1_ms"] = _timeit(lambda: _C.flash_attn_fwd_v1(qkv, B, S, nh, d), flush=flush)
        o, lse = _C.flash_attn_fwd(qkv, B, S, nh, d)
        rec["bwd_ms"] = _timeit(lambda: _C.flash_attn_bwd(dout, qkv, o, lse, B, S, nh, d), flush=flush)
        if hasattr(_C, "flash_attn_bwd_v1"):
            rec["bwd_v1_ms"] = _timeit(lambda: _C.flash_attn_bwd_v1(dout, qkv, o, lse, B, S, nh, d), flush=flush)
        q, k, v = _attn_views(qkv, B, S, nh, d)
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        rec["sdpa_fwd_ms"] = _timeit(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True), flush=flush)
        qg, kg, vg = (t.detach().requires_grad_(True) for t in (q, k, v))
        out = F.scaled_dot_product_attention(qg, kg, vg, is_causal=True)
        go = dout.view(B, S, nh, d).transpose(1, 2).contiguous()
        rec["sdpa_bwd_ms"] = _timeit(lambda: torch.autograd.grad(out, (qg, kg, vg), go, retain_graph=True),
                                     flush=flush)
        # numerics of this forward against SDPA's on the same inputs
        ref = out.detach().transpose(1, 2).reshape(B * S, nh * d).float()
        rec["fwd_max_abs_err_vs_sdpa"] = float((o.float() - ref).abs().max())
        for key in ("fwd", "fwd_v1", "sdpa_fwd"):
            if key + "_ms" in rec:
                rec[key + "_tflops"] = round(fl / rec[key + "_ms"] / 1e9, 1)
        for key in ("bwd", "bwd_v1", "sdpa_bwd"):
            if key + "_ms" in rec:
                rec[key + "_tflops"] = round(2.5 * fl / rec[key + "_ms"] / 1e9, 1)
        for k_ in list(rec):
            if k_.endswith("_ms"):
                rec[k_] = round(rec[k_], 4)
        print(json.dumps(rec), flush=True)
    assert _C.get_error() == 0


def attn_case(args):
    """One forward and one backward launch of the attention kernels (a small ncu target)."""
    from mini_megatron_b200 import _C
    B, S, nh, d = (16, 1024, 12, 64) if args.d == 64 else (4, 2048, 16, 128)
    torch.manual_seed(0)
    qkv = (torch.randn(B * S, 3 * nh * d, device="cuda") * 0.5).bfloat16()
    dout = torch.randn(B * S, nh * d, device="cuda").bfloat16()
    for _ in range(2):
        o, lse = _C.flash_attn_fwd(qkv, B, S, nh, d)
        _C.flash_attn_bwd(dout, qkv, o, lse, B, S, nh, d)
        torch.cuda.synchronize()
    assert _C.get_error() == 0
    print("attention case done")


def profile_case(args):
    """One launch of each hot kernel on GPT-125M training shapes (B=16, S=1024): the ncu target.

    Order of launches (use ncu -k to pick one): GEMM fc1 fwd (GELU epilogue),
    GEMM o fwd (residual epilogue), GEMM fc2 dgrad (GELU-backward epilogue),
    GEMM fc1 wgrad (split-K reduce-add), attention fwd, attention bwd, LayerNorm
    fwd/bwd, cross-entropy fwd/bwd, AdamW over 162M parameters.  Everything is
    allocated up front (about 4 GB).
    """
    from mini_megatron_b200 import _C
    torch.manual_seed(0)
    T, H, F, V, nh, S = args.tokens, 768, 3072, 50304, 12, 1024
    B = T // S
    bf = dict(device="cuda", dtype=torch.bfloat16)
    x = torch.randn(T, H, **bf)
    w1 = torch.randn(F, H, **bf) * 0.02
    w2 = torch.randn(H, F, **bf) * 0.02
    wo = torch.randn(H, H, **bf) * 0.02
    act = torch.empty(T, F, **bf)
    gp = torch.empty(T, F, **bf)
    resid = torch.randn(T, H, device="cuda")
    out32 = torch.empty(T, H, device="cuda")
    dy = torch.randn(T, H, **bf)
    dpre = torch.empty(T, F, **bf)
    dw1 = torch.zeros(F, H, device="cuda")
    qkv = torch.randn(T, 3 * H, **bf)
    lnx = torch.randn(T, H, device="cuda")
    g = torch.ones(H, device="cuda")
    bvec = torch.zeros(H, device="cuda")
    lny = torch.empty(T, H, **bf)
    mean = torch.empty(T, device="cuda")
    rstd = torch.empty(T, device="cuda")
    dx = torch.empty(T, H, device="cuda")
    logits = torch.randn(T, V, **bf)
    labels = torch.randint(0, 50257, (T,), device="cuda")
    n_par = 162_000_000
    p = torch.randn(n_par, device="cuda")
    gr = torch.randn(n_par, device="cuda")
    m = torch.zeros(n_par, device="cuda")
    v = torch.zeros(n_par, device="cuda")
    pb = torch.empty(n_par, **bf)
    for _ in range(2):  # warm-up pass, then the profiled pass
        _C.gemm(x, False, w1, False, act, _C.EPI_GELU, aux=gp)
        _C.gemm(x, False, wo, False, out32, _C.EPI_RESID, resid=resid)
        _C.gemm(dy, False, w2, True, dpre, _C.EPI_DGELU, aux=gp)
        _C.gemm(dpre, True, x, True, dw1, _C.EPI_F32_ACC)
        o, lse = _C.flash_attn_fwd(qkv, B, S, nh, 64)
        _C.flash_attn_bwd(dy, qkv, o, lse, B, S, nh, 64)
        _C.layernorm_fwd(lnx, g, bvec, lny, mean, rstd, 1e-5)
        _C.layernorm_bwd(dy, lnx, mean, rstd, g, resid, dx, g.clone(), bvec.clone())
        mx, se, tg = _C.ce_fwd_stats(logits, labels, 0, 50257)
        _C.ce_bwd(logits, labels, 0, 50257, (mx + torch.log(se)).contiguous(), torch.full((T,), 1.0 / T, device="cuda"))
        _C.adamw_flat(p, gr, m, v, pb, 1e-3, 0.9, 0.999, 1e-8, 0.1, 1, 1.0)
        torch.cuda.synchronize()
    assert _C.get_error() == 0
    print("profile case done")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["gemm", "epi", "profile", "attn", "attn_case"])
    ap.add_argument("--model", default="gpt-125m")
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--d", type=int, default=64)
    ap.add_argument("--tile-widths", action="store_true", help="gemm: also time 128- and 256-wide output tiles")
    ap.add_argument("--pairs", action="store_true",
                    help="gemm: also time one CTA per 128x256 tile against a CTA pair per 256x256 tile")
    args = ap.parse_args()
    {"gemm": bench_gemm, "epi": bench_epilogues, "profile": profile_case, "attn": bench_attn,
     "attn_case": attn_case}[args.kernel](args)


if __name__ == "__main__":
    main()
