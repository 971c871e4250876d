"""Numerics of the memory-bound sm_100a kernels against fp32 PyTorch references."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from mini_megatron_b200 import _C
    return _C


@pytest.mark.parametrize("H", [64, 768, 1024, 2048, 4096])
def test_layernorm_fwd_bwd(H):
    C = _C()
    torch.manual_seed(0)
    rows = 1000
    x = torch.randn(rows, H, device="cuda") * 3 + 1
    g = torch.randn(H, device="cuda")
    b = torch.randn(H, device="cuda")
    y = torch.empty(rows, H, device="cuda", dtype=torch.bfloat16)
    mean = torch.empty(rows, device="cuda")
    rstd = torch.empty(rows, device="cuda")
    C.layernorm_fwd(x, g, b, y, mean, rstd, 1e-5)
    xr = x.clone().requires_grad_(True)
    gr = g.clone().requires_grad_(True)
    br = b.clone().requires_grad_(True)
    ref = torch.nn.functional.layer_norm(xr, (H,), gr, br, 1e-5)
    assert (y.float() - ref).abs().max().item() < 0.05 * ref.abs().max().item()
    dy = torch.randn(rows, H, device="cuda").bfloat16()
    dres = torch.randn(rows, H, device="cuda")
    ref.backward(dy.float())
    dx = torch.empty_like(x)
    dg = torch.ones(H, device="cuda")   # accumulate on top of existing grads
    db = torch.ones(H, device="cuda")
    C.layernorm_bwd(dy, x, mean, rstd, g, dres, dx, dg, db)
    torch.cuda.synchronize()
    torch.testing.assert_close(dx, xr.grad + dres, rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(dg, gr.grad + 1, rtol=2e-3, atol=2e-2)
    torch.testing.assert_close(db, br.grad + 1, rtol=2e-3, atol=2e-2)


@pytest.mark.parametrize("V,n_valid,start", [(50304, 50257, 0), (1024, 1024, 0), (6288, 6000, 6288)])
def test_cross_entropy_stats_and_grad(V, n_valid, start):
    C = _C()
    torch.manual_seed(1)
    rows = 300
    logits = (torch.randn(rows, V, device="cuda") * 4).bfloat16()
    labels = torch.randint(start, start + n_valid, (rows,), device="cuda")
    labels[::7] = start + n_valid + 5 if start > 0 else labels[::7]   # some labels outside this shard
    mx, se, tg = C.ce_fwd_stats(logits, labels, start, n_valid)
    lf = logits.float()[:, :n_valid]
    rmx = lf.max(-1).values
    torch.testing.assert_close(mx, rmx)
    torch.testing.assert_close(se, torch.exp(lf - rmx[:, None]).sum(-1), rtol=1e-4, atol=1e-4)
    local = labels - start
    inside = (local >= 0) & (local < n_valid)
    rtg = torch.where(inside, lf.gather(1, local.clamp(0, n_valid - 1)[:, None])[:, 0], torch.zeros_like(rmx))
    torch.testing.assert_close(tg, rtg)
    lse = (rmx + torch.log(se)).contiguous()
    scale = torch.rand(rows, device="cuda")
    g = logits.clone()
    C.ce_bwd(g, labels, start, n_valid, lse, scale)
    p = torch.softmax(lf, -1)
    onehot = torch.zeros_like(p)
    onehot[inside, local[inside]] = 1
    ref = torch.zeros(rows, V, device="cuda")
    ref[:, :n_valid] = (p - onehot) * scale[:, None]
    assert (g.float() - ref).abs().max().item() < 1e-2


def test_embedding_fwd_bwd():
    C = _C()
    torch.manual_seed(2)
    B, S, H, V = 4, 64, 768, 5000
    ids = torch.randint(0, V, (B, S), device="cuda")
    wte = torch.randn(V, H, device="cuda")
    wpe = torch.randn(S, H, device="cuda")
    out = torch.empty(B * S, H, device="cuda")
    C.embedding_fwd(ids.view(-1), wte, wpe, out, S, 0, V)
    ref = wte[ids] + wpe[None]
    torch.testing.assert_close(out.view(B, S, H), ref)
    # vocab shard [1000, 3000)
    wsh = wte[1000:3000].contiguous()
    out2 = torch.empty_like(out)
    C.embedding_fwd(ids.view(-1), wsh, None, out2, S, 1000, 3000)
    inside = (ids >= 1000) & (ids < 3000)
    ref2 = torch.where(inside[..., None], wte[ids], torch.zeros_like(ref))
    torch.testing.assert_close(out2.view(B, S, H), ref2)
    dout = torch.randn(B * S, H, device="cuda")
    dwte = torch.zeros(V, H, device="cuda")
    dwpe = torch.zeros(S, H, device="cuda")
    C.embedding_bwd(ids.view(-1), dout, dwte, dwpe, B, S, 0, V)
    rwte = torch.zeros(V, H, device="cuda").index_add_(0, ids.view(-1), dout)
    torch.testing.assert_close(dwte, rwte, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(dwpe, dout.view(B, S, H).sum(0), rtol=1e-4, atol=1e-4)


def test_embedding_bwd_deterministic():
    """The token-table gradient is summed in one fixed order (per-row ownership, no atomics): repeated
    launches give bit-identical results, on a skewed id distribution where many positions share a
    row, into a vocabulary shard, accumulating onto an existing gradient, and match an fp32 sum."""
    C = _C()
    torch.manual_seed(5)
    B, S, H, V = 8, 1024, 768, 50304
    ids = (torch.randn(B, S, device="cuda").abs() * 300).long().clamp_(0, V - 1)  # heavy reuse of low ids
    dout = torch.randn(B * S, H, device="cuda")
    base = torch.randn(2000, H, device="cuda")
    outs = []
    for _ in range(3):
        dwte = base.clone()
        C.embedding_bwd(ids.view(-1), dout, dwte, None, B, S, 100, 2100)
        outs.append(dwte)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    inside = (ids.view(-1) >= 100) & (ids.view(-1) < 2100)
    ref = base.double().index_add_(0, ids.view(-1)[inside] - 100, dout[inside].double())
    torch.testing.assert_close(outs[0].double(), ref, rtol=1e-5, atol=1e-4)


def test_adamw_matches_torch():
    C = _C()
    torch.manual_seed(3)
    n = 100_003
    p = torch.randn(n, device="cuda")
    ref = p.clone().requires_grad_(True)
    opt = torch.optim.AdamW([ref], lr=1e-3, weight_decay=0.1, foreach=False)
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    pb = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    for step in range(1, 4):
        g = torch.randn(n, device="cuda")
        ref.grad = g.clone()
        opt.step()
        C.adamw_flat(p, g * 2.0, m, v, pb, 1e-3, 0.9, 0.999, 1e-8, 0.1, step, 0.5)
    torch.cuda.synchronize()
    torch.testing.assert_close(p, ref.detach(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(pb.float(), p.bfloat16().float())


def test_gelu_math_matches_exact_erf_gelu():
    C = _C()
    x = torch.linspace(-12, 12, 1_000_001, device="cuda")
    y, g = C.gelu_fwd_bwd_f32(x)
    xr = x.double().requires_grad_(True)
    yr = torch.nn.functional.gelu(xr)
    yr.backward(torch.ones_like(yr))
    assert (y.double() - yr).abs().max().item() < 2e-6
    assert (g.double() - xr.grad).abs().max().item() < 2e-6


def test_peer_flag_wait_times_out_with_an_error_status():
    """A cross-GPU flag wait whose flag is never set gives up after its limit, records
    kErrPeerWait in the device error word and returns; the context stays usable."""
    import mini_megatron_b200.ops as ops
    C = ops.native()
    C.clear_error()
    flags = torch.zeros(8, dtype=torch.int32, device="cuda")     # nothing will ever raise these
    slots = torch.zeros(4, 256, dtype=torch.bfloat16, device="cuda")
    out = torch.full((4, 256), 7.0, device="cuda")
    t0 = time.time()
    C.tp_rs_reduce(slots.data_ptr(), slots.numel(), 1, flags.data_ptr(), 1, None, out, None, slots.numel(),
                   timeout_ms=50)
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    assert C.get_error() == 301, C.get_error()
    assert elapsed < 5.0
    assert torch.all(out == 7.0)        # the kernel returned without touching the output
    with pytest.raises(RuntimeError):
        ops.check_errors()              # the host-side check turns the status into an exception
    C.clear_error()
    # the context is still usable
    flags.fill_(1)
    C.tp_rs_reduce(slots.data_ptr(), slots.numel(), 1, flags.data_ptr(), 1, None, out, None, slots.numel(),
                   timeout_ms=50)
    torch.cuda.synchronize()
    assert C.get_error() == 0 and torch.all(out == 0.0)


@pytest.mark.parametrize("M,N,n_valid", [(512, 1024, 1000), (300, 50304, 50257), (128, 256, 256)])
def test_lm_head_gemm_with_fused_ce_statistics(M, N, n_valid):
    """gemm_ce_stats: bf16 logits identical to the plain GEMM, and (max, sumexp, target) equal to the
    standalone statistics pass over those logits (fp32 PyTorch reference on the stored bf16 values)."""
    import mini_megatron_b200.ops as ops
    C = ops.native()
    torch.manual_seed(0)
    K = 256
    A = (torch.randn(M, K, device="cuda") * 0.5).bfloat16()
    B = (torch.randn(N, K, device="cuda") * 0.5).bfloat16()
    lab = torch.randint(0, n_valid, (M,), device="cuda")
    lab[::7] = -100
    D = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    mx, se, tg = C.gemm_ce_stats(A, B, D, lab, 0, n_valid)
    D2 = torch.empty_like(D)
    C.gemm(A, False, B, False, D2, C.EPI_BF16)
    torch.cuda.synchronize()
    assert torch.equal(D, D2)
    x = D.float()[:, :n_valid]
    ref_max = x.max(dim=1).values
    ref_lse = torch.logsumexp(x, dim=1)
    assert torch.allclose(mx, ref_max)
    assert torch.allclose(mx + torch.log(se), ref_lse, atol=1e-4, rtol=1e-5)
    ok = lab >= 0
    ref_tg = torch.zeros(M, device="cuda")
    ref_tg[ok] = x[ok].gather(1, lab[ok].unsqueeze(1)).squeeze(1)
    assert torch.equal(tg, ref_tg)
