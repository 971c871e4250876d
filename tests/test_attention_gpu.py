"""tcgen05 causal flash attention (forward + backward) vs an fp32 PyTorch reference."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(qkv, B, S, nh, d):
    t = qkv.float().view(B, S, 3, nh, d)
    q, k, v = (t[:, :, i].transpose(1, 2) for i in range(3))
    s = (q @ k.transpose(-1, -2)) / math.sqrt(d)
    mask = torch.ones(S, S, device=qkv.device, dtype=torch.bool).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(s, -1)
    o = torch.softmax(s, -1) @ v
    return o.transpose(1, 2).reshape(B * S, nh * d), lse


@pytest.mark.parametrize("B,S,nh,d", [(2, 128, 2, 64), (2, 384, 3, 64), (1, 512, 2, 128), (4, 1024, 12, 64),
                                      (1, 2048, 2, 128)])
def test_flash_fwd_bwd(B, S, nh, d):
    from mini_megatron_b200 import _C
    torch.manual_seed(B * S + nh + d)
    qkv = torch.randn(B * S, 3 * nh * d, device="cuda").bfloat16()
    out, lse = _C.flash_attn_fwd(qkv, B, S, nh, d)
    torch.cuda.synchronize()
    assert _C.get_error() == 0
    x = qkv.float().requires_grad_(True)
    ro, rlse = _ref(x, B, S, nh, d)
    assert (out.float() - ro).abs().max().item() < 2e-2
    torch.testing.assert_close(lse, rlse.detach(), rtol=1e-3, atol=1e-3)
    dout = torch.randn(B * S, nh * d, device="cuda").bfloat16()
    ro.backward(dout.float())
    dqkv = _C.flash_attn_bwd(dout, qkv, out, lse, B, S, nh, d)
    torch.cuda.synchronize()
    assert _C.get_error() == 0
    ref = x.grad
    err = (dqkv.float() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err < 2e-2 * scale + 1e-2, f"dqkv max err {err} (scale {scale})"
    rel = ((dqkv.float() - ref).norm() / ref.norm()).item()
    assert rel < 1e-2, rel


@pytest.mark.parametrize("B,S,nh,d,amp", [(2, 1024, 2, 64, 3.0), (1, 1152, 2, 128, 2.0)])
def test_flash_fwd_large_scores_rescale(B, S, nh, d, amp):
    """Scores spread over tens of log2 units, so the running row maximum grows by more than the
    forward's lazy-rescale threshold on many key tiles and the in-TMEM rescale of O is exercised
    (S = 1152: nine query tiles, the last work item has a single tile)."""
    from mini_megatron_b200 import _C
    torch.manual_seed(7 + d)
    qkv = (torch.randn(B * S, 3 * nh * d, device="cuda") * amp).bfloat16()
    out, lse = _C.flash_attn_fwd(qkv, B, S, nh, d)
    torch.cuda.synchronize()
    assert _C.get_error() == 0
    ro, rlse = _ref(qkv, B, S, nh, d)
    assert (out.float() - ro).abs().max().item() < 3e-2 * ro.abs().max().item()
    torch.testing.assert_close(lse, rlse, rtol=1e-3, atol=2e-3)
