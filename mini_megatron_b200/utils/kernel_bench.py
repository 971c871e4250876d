"""Kernel micro-benchmarks on the training shapes (CUDA-event timed).

Usage::

    python -m mini_megatron_b200.utils.kernel_bench gemm [--model gpt-125m] [--tokens 16384]

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
        print(json.dumps({"kernel": "gemm_bf16_sm100", "name": name, "M": M, "N": N, "K": K,
                          "ms": round(ours, 4), "tflops": round(flops / ours / 1e9, 1),
                          "cublas_ms": round(lib, 4), "cublas_tflops": round(flops / lib / 1e9, 1)}))
    assert _C.get_error() == 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["gemm"])
    ap.add_argument("--model", default="gpt-125m")
    ap.add_argument("--tokens", type=int, default=16384)
    args = ap.parse_args()
    {"gemm": bench_gemm}[args.kernel](args)


if __name__ == "__main__":
    main()
