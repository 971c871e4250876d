"""Numerics of the tcgen05 GEMM against an fp32 PyTorch reference.

Covers the three operand layouts a linear layer needs (forward, dgrad,
wgrad), ragged M/N/K tails, both tile widths, and every fused epilogue.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from mini_megatron_b200 import _C
    return _C


def _operands(M, N, K, a_mn, b_mn, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    b = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    A = a.t().contiguous() if a_mn else a
    B = b.t().contiguous() if b_mn else b
    ref = a.float() @ b.float().t()
    return A, B, ref


def _check_close(out, ref, rtol):
    err = (out.float() - ref).abs().max().item()
    scale = ref.abs().max().item() + 1e-6
    assert err <= rtol * scale, f"max abs err {err} vs scale {scale}"


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (256, 384, 320), (300, 392, 200), (1024, 2304, 768)])
@pytest.mark.parametrize("bn", [128, 256])
def test_gemm_layouts_fp32_out(a_mn, b_mn, M, N, K, bn):
    C = _C()
    if a_mn and M % 8:
        pytest.skip("MN-major A needs M % 8 == 0 (TMA row stride)")
    A, B, ref = _operands(M, N, K, a_mn, b_mn)
    D = torch.full((M, N), float("nan"), device="cuda")
    C.gemm(A, a_mn, B, b_mn, D, C.EPI_F32, bn=bn)
    torch.cuda.synchronize()
    assert C.get_error() == 0
    _check_close(D, ref, 1e-3)


@pytest.mark.parametrize("bn", [128, 256])
def test_gemm_bf16_out_and_alpha(bn):
    C = _C()
    M, N, K = 512, 768, 768
    A, B, ref = _operands(M, N, K, False, False, seed=1)
    D = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm(A, False, B, False, D, C.EPI_BF16, alpha=0.5, bn=bn)
    torch.cuda.synchronize()
    _check_close(D, 0.5 * ref, 1e-2)


def test_gemm_accumulate():
    C = _C()
    M, N, K = 384, 256, 512
    A, B, ref = _operands(M, N, K, True, True, seed=2)
    D = torch.randn(M, N, device="cuda")
    D0 = D.clone()
    C.gemm(A, True, B, True, D, C.EPI_F32_ACC)
    torch.cuda.synchronize()
    _check_close(D, D0 + ref, 1e-3)


def test_gemm_gelu_and_dgelu():
    C = _C()
    M, N, K = 512, 1024, 256
    A, B, ref = _operands(M, N, K, False, False, seed=3)
    D = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    gp = torch.empty_like(D)
    C.gemm(A, False, B, False, D, C.EPI_GELU, aux=gp)
    torch.cuda.synchronize()
    x = ref.clone().requires_grad_(True)
    y = torch.nn.functional.gelu(x)
    y.backward(torch.ones_like(y))
    _check_close(D, y.detach(), 1e-2)
    _check_close(gp, x.grad, 1e-2)
    # dgelu: out = acc * gelu'(pre), with gelu'(pre) as stored by the forward epilogue
    D2 = torch.empty_like(D)
    C.gemm(A, False, B, False, D2, C.EPI_DGELU, aux=gp)
    torch.cuda.synchronize()
    _check_close(D2, ref * gp.float(), 1e-2)


def test_gemm_residual_inplace():
    C = _C()
    M, N, K = 256, 768, 3072
    A, B, ref = _operands(M, N, K, False, False, seed=4)
    R = torch.randn(M, N, device="cuda")
    expect = R + ref
    C.gemm(A, False, B, False, R, C.EPI_RESID, resid=R)
    torch.cuda.synchronize()
    _check_close(R, expect, 1e-3)


def test_gemm_strided_views():
    """Operands that are column slices of a wider buffer (e.g. q/k/v of a fused qkv)."""
    C = _C()
    M, K = 256, 192
    big = torch.randn(M, 3 * K, device="cuda").bfloat16()
    a = big[:, K:2 * K]
    b = torch.randn(320, K, device="cuda").bfloat16()
    D = torch.empty(M, 320, device="cuda")
    C.gemm(a, False, b, False, D, C.EPI_F32)
    torch.cuda.synchronize()
    _check_close(D, a.float() @ b.float().t(), 1e-3)


@pytest.mark.parametrize("M,N", [(8232, 832), (200, 96), (4096, 768)])
def test_gemm_side_input_epilogues_ragged(M, N):
    """RESID / DGELU epilogues read a side input one chunk ahead: ragged M/N and several tiles per CTA."""
    C = _C()
    K = 256
    A, B, ref = _operands(M, N, K, False, False, seed=11)
    R = torch.randn(M, N, device="cuda")
    expect = R + ref
    C.gemm(A, False, B, False, R, C.EPI_RESID, resid=R)
    gp = torch.randn(M, N, device="cuda").bfloat16()
    D2 = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm(A, False, B, False, D2, C.EPI_DGELU, aux=gp)
    torch.cuda.synchronize()
    _check_close(R, expect, 1e-3)
    _check_close(D2, ref * gp.float(), 1e-2)


# ----------------------------------------------------------------------------- CTA pairs
# cg=2: a 2-CTA cluster computes a 256 x 256 output tile with pair MMAs, each CTA
# holding 128 rows of A and 128 rows of B.  An odd number of 128-row m-tiles
# leaves the second CTA of the last pair outside the matrix.

@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (296, 392, 200), (384, 512, 320), (1024, 2304, 768)])
def test_gemm_cta_pair_layouts(a_mn, b_mn, M, N, K):
    C = _C()
    A, B, ref = _operands(M, N, K, a_mn, b_mn, seed=21)
    D = torch.full((M, N), float("nan"), device="cuda")
    C.gemm(A, a_mn, B, b_mn, D, C.EPI_F32, bn=256, cg=2)
    torch.cuda.synchronize()
    assert C.get_error() == 0
    _check_close(D, ref, 1e-3)


def test_gemm_cta_pair_epilogues():
    C = _C()
    M, N, K = 8232, 832, 256          # 65 m-tiles, 4 n-tiles: several tiles per pair, ragged edges
    A, B, ref = _operands(M, N, K, False, False, seed=22)
    D = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C.gemm(A, False, B, False, D, C.EPI_BF16, alpha=0.5, bn=256, cg=2)
    gp = torch.empty_like(D)
    act = torch.empty_like(D)
    C.gemm(A, False, B, False, act, C.EPI_GELU, aux=gp, bn=256, cg=2)
    R = torch.randn(M, N, device="cuda")
    expect = R + ref
    C.gemm(A, False, B, False, R, C.EPI_RESID, resid=R, bn=256, cg=2)
    D2 = torch.empty_like(D)
    C.gemm(A, False, B, False, D2, C.EPI_DGELU, aux=gp, bn=256, cg=2)
    torch.cuda.synchronize()
    assert C.get_error() == 0
    _check_close(D, 0.5 * ref, 1e-2)
    x = ref.clone().requires_grad_(True)
    y = torch.nn.functional.gelu(x)
    y.backward(torch.ones_like(y))
    _check_close(act, y.detach(), 1e-2)
    _check_close(gp, x.grad, 1e-2)
    _check_close(R, expect, 1e-3)
    _check_close(D2, ref * gp.float(), 1e-2)


@pytest.mark.parametrize("M,N,K", [(768, 768, 16384), (384, 2304, 4096)])
def test_gemm_cta_pair_split_k_accumulate(M, N, K):
    """Weight-gradient shapes: few output tiles, long K -> K splits with the atomic epilogue."""
    C = _C()
    A, B, ref = _operands(M, N, K, True, True, seed=23)
    D = torch.randn(M, N, device="cuda")
    D0 = D.clone()
    C.gemm(A, True, B, True, D, C.EPI_F32_ACC, cg=2)
    torch.cuda.synchronize()
    assert C.get_error() == 0
    _check_close(D, D0 + ref, 1e-3)
