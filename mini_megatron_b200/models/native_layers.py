"""Fused native (CUDA) forward/backward for the GPT building blocks.

Each block is ONE autograd Function whose forward and backward drive the
sm_100a kernels directly, so a decoder layer costs a fixed, small set of
launches and no autograd bookkeeping per op:

layer forward   LN1 -> [SP all-gather] -> QKV GEMM -> flash attention ->
                O GEMM (+residual epilogue | TP reduce) -> LN2 -> [SP AG] ->
                fc1 GEMM (+GELU epilogue) -> fc2 GEMM (+residual | TP reduce)
layer backward  fc2 dgrad (+dGELU epilogue), fc2/fc1 wgrad (fp32 accumulate
                into main_grad, split-K), fc1 dgrad -> [TP reduce] -> LN2
                backward (+residual grad) -> O dgrad/wgrad -> attention
                backward -> QKV dgrad/wgrad -> [TP reduce] -> LN1 backward

Residual stream: fp32 ``[B, S_local, H]`` (the reference keeps it fp32 under
autocast, main.py:93 + model/transformer.py:59-62).  GEMM operands are bf16,
accumulation fp32.  Weight gradients never pass through autograd: the
wgrad GEMMs accumulate into ``param.main_grad`` (see param_buffer.py).

Tensor-parallel collectives: with a ``TPWorkspace`` attached (``tp_impl``
"fused", the default on CUDA with tp > 1; parallel/fused_tp.py) the decoder
layers, the head and the embedding run the sequence-parallel dataflow with
every collective inside the kernels (NVLink pushes and flag waits); otherwise
they go through NCCL via torch.distributed.  ``S_local = S / tp`` under
sequence parallelism, ``S`` otherwise.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..comm import sequence_parallel as spc
from ..ops import native
from ..ops.attention import flash_attn_bwd, flash_attn_fwd
from ..ops.linear import EPI_DGELU, EPI_RESID, linear_dgrad, linear_fwd, linear_gelu_fwd, linear_wgrad
from ..parallel.param_buffer import bf16_weight, grad_target

# Cross-entropy statistics from the lm_head GEMM epilogue (one fewer pass over the logits).
_CE_FUSED = os.environ.get("MMB_CE_FUSED", "1") == "1"

LN_EPS = 1e-5


def _world(group):
    return 1 if group is None else dist.get_world_size(group=group)


def _ln_fwd(x2, ln):
    C = native()
    rows, H = x2.shape
    y = torch.empty(rows, H, device=x2.device, dtype=torch.bfloat16)
    mean = torch.empty(rows, device=x2.device, dtype=torch.float32)
    rstd = torch.empty_like(mean)
    C.layernorm_fwd(x2, ln.weight.detach(), ln.bias.detach(), y, mean, rstd, ln.eps)
    return y, mean, rstd


def _ln_bwd(dy, x2, mean, rstd, ln, dres=None, want_bf16=False):
    """LayerNorm backward; with ``want_bf16`` the same kernel also writes a bf16 copy of dx."""
    dx = torch.empty_like(x2)
    dxb = torch.empty(x2.shape, device=x2.device, dtype=torch.bfloat16) if want_bf16 else None
    native().layernorm_bwd(dy.contiguous(), x2, mean, rstd, ln.weight.detach(), dres, dx, grad_target(ln.weight),
                           grad_target(ln.bias), dxb)
    if want_bf16:
        dx._mmb_bf16 = dxb  # travels with the residual-stream gradient to the next layer's backward
    return dx


def _bf16_of(t):
    b = getattr(t, "_mmb_bf16", None)
    return b if b is not None else t.to(torch.bfloat16)


def _gather_seq(t2, B, group):
    """[B*S_l, H] -> [B*S, H] (all-gather along the sequence)."""
    H = t2.shape[-1]
    return spc.sp_all_gather(t2.view(B, -1, H), group=group).reshape(-1, H)


def _reduce(t2, B, group, sp):
    """TP reduction of a [B*S, H] partial: reduce-scatter along S (SP) or all-reduce."""
    if _world(group) == 1:
        return t2
    if sp:
        H = t2.shape[-1]
        return spc.sp_reduce_scatter(t2.view(B, -1, H), group=group).reshape(-1, H)
    dist.all_reduce(t2, group=group)
    return t2


def _layer_forward(x2, layer, B, S, group, sp):
    """Forward of one DecoderLayer on [B*S_l, H] fp32; returns (out, saved tensors)."""
    attn, mlp = layer.attn, layer.mlp
    t = _world(group)
    ln1, m1, r1 = _ln_fwd(x2, layer.ln1)
    ln1_full = _gather_seq(ln1, B, group) if sp else ln1
    qkv = linear_fwd(ln1_full, bf16_weight(attn.qkv.weight))
    ctx_out, lse = flash_attn_fwd(qkv, B, S, attn.num_heads, attn.head_dim)
    if t == 1:
        x1 = linear_fwd(ctx_out, bf16_weight(attn.o.weight), out=torch.empty_like(x2), epi=EPI_RESID, resid=x2)
    else:
        part = linear_fwd(ctx_out, bf16_weight(attn.o.weight))
        x1 = x2 + _reduce(part, B, group, sp).float()
    ln2, m2, r2 = _ln_fwd(x1, layer.ln2)
    ln2_full = _gather_seq(ln2, B, group) if sp else ln2
    act, gelu_grad = linear_gelu_fwd(ln2_full, bf16_weight(mlp.fc1.weight))
    if t == 1:
        out = linear_fwd(act, bf16_weight(mlp.fc2.weight), out=torch.empty_like(x1), epi=EPI_RESID, resid=x1)
    else:
        part = linear_fwd(act, bf16_weight(mlp.fc2.weight))
        out = x1 + _reduce(part, B, group, sp).float()
    saved = (x2, m1, r1, ln1_full, qkv, ctx_out, lse, x1, m2, r2, ln2_full, gelu_grad, act)
    return out, saved


def _layer_backward(dout, saved, layer, B, S, group, sp):
    attn, mlp = layer.attn, layer.mlp
    t = _world(group)
    (x2, m1, r1, ln1_full, qkv, ctx_out, lse, x1, m2, r2, ln2_full, gelu_grad, act) = saved
    # ---- MLP
    g = _bf16_of(dout)
    g_full = _gather_seq(g, B, group) if sp else g
    w2, w1 = mlp.fc2.weight, mlp.fc1.weight
    d_pre = linear_dgrad(g_full, bf16_weight(w2), epi=EPI_DGELU, aux=gelu_grad)
    linear_wgrad(g_full, act, grad_target(w2))
    d_ln2 = linear_dgrad(d_pre, bf16_weight(w1))
    linear_wgrad(d_pre, ln2_full, grad_target(w1))
    if t > 1:
        d_ln2 = _reduce(d_ln2, B, group, sp)
    dx1 = _ln_bwd(d_ln2, x1, m2, r2, layer.ln2, dres=dout, want_bf16=True)
    # ---- attention
    g = dx1._mmb_bf16
    g_full = _gather_seq(g, B, group) if sp else g
    wo, wqkv = attn.o.weight, attn.qkv.weight
    d_ctx = linear_dgrad(g_full, bf16_weight(wo))
    linear_wgrad(g_full, ctx_out, grad_target(wo))
    dqkv = flash_attn_bwd(d_ctx, qkv, ctx_out, lse, B, S, attn.num_heads, attn.head_dim)
    d_ln1 = linear_dgrad(dqkv, bf16_weight(wqkv))
    linear_wgrad(dqkv, ln1_full, grad_target(wqkv))
    if t > 1:
        d_ln1 = _reduce(d_ln1, B, group, sp)
    return _ln_bwd(d_ln1, x2, m1, r1, layer.ln1, dres=dx1, want_bf16=True)


def _layer_forward_fused(x2, layer, B, S, ws):
    """Sequence-parallel layer forward with the TP collectives fused into the kernels (parallel/fused_tp.py)."""
    attn, mlp = layer.attn, layer.mlp
    slot = layer._mmb_tp_slot
    ln1_full, m1, r1, e1 = ws.ln_fwd_ag(x2, layer.ln1, 2 * slot)
    qkv = torch.empty(ws.rows, attn.qkv.weight.shape[0], device=x2.device, dtype=torch.bfloat16)
    ws.gemm_ag(ln1_full, e1, bf16_weight(attn.qkv.weight), False, qkv)
    ctx_out, lse = flash_attn_fwd(qkv, B, S, attn.num_heads, attn.head_dim)
    x1 = ws.rs_reduce(ws.gemm_rs(ctx_out, bf16_weight(attn.o.weight), False), resid=x2)
    ln2_full, m2, r2, e2 = ws.ln_fwd_ag(x1, layer.ln2, 2 * slot + 1)
    n_ffn = mlp.fc1.weight.shape[0]
    act = torch.empty(ws.rows, n_ffn, device=x2.device, dtype=torch.bfloat16)
    gelu_grad = torch.empty_like(act)
    ws.gemm_ag(ln2_full, e2, bf16_weight(mlp.fc1.weight), False, act, epi=3, aux=gelu_grad)
    out = ws.rs_reduce(ws.gemm_rs(act, bf16_weight(mlp.fc2.weight), False), resid=x1)
    if ws.copy_saved:  # several microbatches in flight (pipeline): keep private copies for the wgrads
        ln1_full, ln2_full = ln1_full.clone(), ln2_full.clone()
    saved = (x2, m1, r1, ln1_full, qkv, ctx_out, lse, x1, m2, r2, ln2_full, gelu_grad, act)
    return out, saved


def _layer_backward_fused(dout, saved, layer, B, S, ws):
    attn, mlp = layer.attn, layer.mlp
    (x2, m1, r1, ln1_full, qkv, ctx_out, lse, x1, m2, r2, ln2_full, gelu_grad, act) = saved
    w2, w1, wo, wqkv = mlp.fc2.weight, mlp.fc1.weight, attn.o.weight, attn.qkv.weight
    # ---- MLP: gathered output gradient (pushed by the producer of dout, or pushed here)
    g_full, eg = ws.gather_grad(dout)
    d_pre = torch.empty(ws.rows, w1.shape[0], device=dout.device, dtype=torch.bfloat16)
    ws.gemm_ag(g_full, eg, bf16_weight(w2), True, d_pre, epi=EPI_DGELU, aux=gelu_grad)
    linear_wgrad(g_full, act, grad_target(w2))
    e_rs = ws.gemm_rs(d_pre, bf16_weight(w1), True)
    linear_wgrad(d_pre, ln2_full, grad_target(w1))
    d_ln2 = ws.rs_reduce(e_rs, out_bf16=True)
    dx1 = ws.ln_bwd_ag(d_ln2, x1, m2, r2, layer.ln2, dout, grad_target)
    # ---- attention
    g_full, eg = dx1._mmb_gathered
    d_ctx = torch.empty(ws.rows, wo.shape[1], device=dout.device, dtype=torch.bfloat16)
    ws.gemm_ag(g_full, eg, bf16_weight(wo), True, d_ctx)
    linear_wgrad(g_full, ctx_out, grad_target(wo))
    dqkv = flash_attn_bwd(d_ctx, qkv, ctx_out, lse, B, S, attn.num_heads, attn.head_dim)
    e_rs = ws.gemm_rs(dqkv, bf16_weight(wqkv), True)
    linear_wgrad(dqkv, ln1_full, grad_target(wqkv))
    d_ln1 = ws.rs_reduce(e_rs, out_bf16=True)
    return ws.ln_bwd_ag(d_ln1, x2, m1, r1, layer.ln1, dx1, grad_target)


class DecoderLayerFn(torch.autograd.Function):
    """x_out = x + MLP(LN2(x1)), x1 = x + Attn(LN1(x)) on the native kernels."""

    @staticmethod
    def forward(ctx, x, layer, group, sp, recompute, *params):
        # ``params`` are passed only so autograd knows the output depends on
        # them; their gradients are accumulated into main_grad by the kernels.
        ctx.n_params = len(params)
        B, S_l, H = x.shape
        S = S_l * (_world(group) if sp else 1)
        x2 = x.reshape(-1, H).contiguous()
        ws = getattr(layer, "_mmb_tp_ws", None) if sp else None
        ctx.ws = ws
        if ws is not None:
            out, saved = _layer_forward_fused(x2, layer, B, S, ws)
        else:
            out, saved = _layer_forward(x2, layer, B, S, group, sp)
        ctx.layer, ctx.group, ctx.sp, ctx.B, ctx.S, ctx.recompute = layer, group, sp, B, S, recompute
        if recompute:
            ctx.save_for_backward(x2)
        else:
            ctx.save_for_backward(*saved)
        for hook in getattr(layer, "_mmb_fwd_hooks", ()):
            hook()
        return out.view(B, S_l, H)

    @staticmethod
    def backward(ctx, dout):
        B, S_l, H = dout.shape
        d2 = dout.reshape(-1, H).contiguous()
        ws = ctx.ws
        if ctx.recompute:
            (x2,) = ctx.saved_tensors
            if ws is not None:
                _, saved = _layer_forward_fused(x2, ctx.layer, ctx.B, ctx.S, ws)
            else:
                _, saved = _layer_forward(x2, ctx.layer, ctx.B, ctx.S, ctx.group, ctx.sp)
        else:
            saved = ctx.saved_tensors
        if getattr(dout, "_mmb_bf16", None) is not None:
            d2._mmb_bf16 = dout._mmb_bf16.view(-1, H)
        if getattr(dout, "_mmb_gathered", None) is not None:
            d2._mmb_gathered = dout._mmb_gathered
        if ws is not None:
            dx = _layer_backward_fused(d2, saved, ctx.layer, ctx.B, ctx.S, ws)
        else:
            dx = _layer_backward(d2, saved, ctx.layer, ctx.B, ctx.S, ctx.group, ctx.sp)
        for hook in getattr(ctx.layer, "_mmb_grad_ready_hooks", ()):
            hook()
        out = dx.view(B, S_l, H)
        if getattr(dx, "_mmb_bf16", None) is not None:
            out._mmb_bf16 = dx._mmb_bf16.view(B, S_l, H)
        if getattr(dx, "_mmb_gathered", None) is not None:
            out._mmb_gathered = dx._mmb_gathered
        return (out, None, None, None, None) + (None,) * ctx.n_params


def run_grad_ready_hooks(module):
    """Tell the data-parallel gradient sync that ``module``'s gradients are final (its backward was enqueued)."""
    for hook in getattr(module, "_mmb_grad_ready_hooks", ()):
        hook()


class EmbeddingFn(torch.autograd.Function):
    """x = tok_emb(ids) (vocab-parallel, TP-summed) + pos_emb; SP keeps the local sequence shard."""

    @staticmethod
    def forward(ctx, ids, emb, group, sp, *params):
        ctx.n_params = len(params)
        C = native()
        tok = emb.token_embedding
        B, S = ids.shape
        H = tok.weight.shape[1]
        ids_c = ids.contiguous()
        ws = getattr(emb, "_mmb_tp_ws", None) if sp else None
        ctx.ws = ws
        if ws is not None:
            # fused TP: each vocabulary owner writes tok + pos of its rows into their sequence owner
            out = ws.emb_fwd(ids_c.view(-1), tok.weight.detach(), emb.position_embedding.weight.detach(),
                             tok.vocab_start_index, tok.vocab_end_index)
            ctx.save_for_backward(ids_c)
            ctx.emb, ctx.group, ctx.sp = emb, group, sp
            return out.view(B, -1, H)
        full = torch.empty(B * S, H, device=ids.device, dtype=torch.float32)
        tp_rank = dist.get_rank(group=group) if _world(group) > 1 else 0
        wpe = emb.position_embedding.weight.detach() if tp_rank == 0 else None
        C.embedding_fwd(ids_c.view(-1), tok.weight.detach(), wpe, full, S, tok.vocab_start_index,
                        tok.vocab_end_index)
        out = _reduce(full, B, group, sp) if _world(group) > 1 else full
        ctx.save_for_backward(ids_c)
        ctx.emb, ctx.group, ctx.sp = emb, group, sp
        return out.view(B, -1, H)

    @staticmethod
    def backward(ctx, dout):
        (ids,) = ctx.saved_tensors
        emb, group = ctx.emb, ctx.group
        tok, pos = emb.token_embedding, emb.position_embedding
        B, S = ids.shape
        H = dout.shape[-1]
        d2 = dout.reshape(-1, H).contiguous().float()
        if ctx.ws is not None:
            ctx.ws.emb_bwd(ids.view(-1), d2, grad_target(tok.weight),
                           grad_target(pos.weight) if pos.weight.requires_grad else None,
                           tok.vocab_start_index, tok.vocab_end_index)
            run_grad_ready_hooks(emb)
            return (None, None, None, None) + (None,) * ctx.n_params
        if ctx.sp:
            d2 = _gather_seq(d2, B, group).contiguous()
        native().embedding_bwd(ids.view(-1), d2, grad_target(tok.weight),
                               grad_target(pos.weight) if pos.weight.requires_grad else None, B, S,
                               tok.vocab_start_index, tok.vocab_end_index)
        run_grad_ready_hooks(emb)
        return (None, None, None, None) + (None,) * ctx.n_params


class HeadLossFn(torch.autograd.Function):
    """loss = masked mean of vocab-parallel CE(lm_head(ln_f(x)), labels)."""

    @staticmethod
    def forward(ctx, x, ln_f, lm_head, labels, loss_mask, n_vocab, group, sp, *params):
        ctx.n_params = len(params)
        B, S_l, H = x.shape
        x2 = x.reshape(-1, H).contiguous()
        w = lm_head.weight
        V_local = w.shape[0]
        tp_rank = dist.get_rank(group=group) if _world(group) > 1 else 0
        vstart = tp_rank * V_local
        n_valid = max(0, min(V_local, n_vocab - vstart))
        lab = labels.reshape(-1).contiguous()
        ws = getattr(lm_head, "_mmb_tp_ws", None) if sp else None
        ctx.ws = ws
        if ws is not None:
            # fused TP: ln_f rows pushed to every rank, lm_head GEMM waiting per source rank, the
            # cross-entropy statistics combined over NVLink (no NCCL collective in the head)
            ln_full, m, r, e = ws.ln_fwd_ag(x2, ln_f, lm_head._mmb_tp_slot)
            logits = torch.empty(ln_full.shape[0], V_local, device=x.device, dtype=torch.bfloat16)
            mx, se, tg = ws.gemm_ce(ln_full, e, bf16_weight(w), logits, lab, vstart, n_valid)
            if ws.copy_saved:
                ln_full = ln_full.clone()
            lse, tg = ws.ce_allreduce(mx, se, tg)
            valid = (lab != -100).float()
            mask = loss_mask.reshape(-1).float()
            denom = mask.sum()
            loss = ((lse - tg) * valid * mask).sum() / denom
            ctx.save_for_backward(x2, m, r, ln_full, logits, lse, lab, valid * mask / denom)
            ctx.ln_f, ctx.lm_head, ctx.group, ctx.sp, ctx.B, ctx.vstart, ctx.n_valid = (
                ln_f, lm_head, group, sp, B, vstart, n_valid)
            ctx.x_shape = x.shape
            ctx.mark_non_differentiable(logits)
            ctx.set_materialize_grads(False)
            return loss, logits
        ln, m, r = _ln_fwd(x2, ln_f)
        ln_full = _gather_seq(ln, B, group) if sp else ln
        if _CE_FUSED:
            # the lm_head epilogue writes per-tile (max, sumexp) partials: no second pass over the logits
            logits = torch.empty(ln_full.shape[0], V_local, device=x.device, dtype=torch.bfloat16)
            mx, se, tg = native().gemm_ce_stats(ln_full, bf16_weight(w), logits, lab, vstart, n_valid)
        else:
            logits = linear_fwd(ln_full, bf16_weight(w))       # [B*S, V_local] bf16
            mx, se, tg = native().ce_fwd_stats(logits, lab, vstart, n_valid)
        if _world(group) > 1:
            gmax = mx.clone()
            dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=group)
            se = se * torch.exp(mx - gmax)
            dist.all_reduce(se, group=group)
            dist.all_reduce(tg, group=group)
            mx = gmax
        lse = mx + torch.log(se)
        valid = (lab != -100).float()
        mask = loss_mask.reshape(-1).float()
        denom = mask.sum()
        loss = ((lse - tg) * valid * mask).sum() / denom
        ctx.save_for_backward(x2, m, r, ln_full, logits, lse, lab, valid * mask / denom)
        ctx.ln_f, ctx.lm_head, ctx.group, ctx.sp, ctx.B, ctx.vstart, ctx.n_valid = (
            ln_f, lm_head, group, sp, B, vstart, n_valid)
        ctx.x_shape = x.shape
        ctx.mark_non_differentiable(logits)
        ctx.set_materialize_grads(False)  # no zero-filled [tokens, V] gradient for the logits output
        return loss, logits

    @staticmethod
    def backward(ctx, dloss, dlogits_unused):
        x2, m, r, ln_full, logits, lse, lab, wscale = ctx.saved_tensors
        if dloss is None:
            dloss = torch.zeros((), device=x2.device)
        scale = (wscale * dloss.float()).contiguous()
        native().ce_bwd(logits, lab, ctx.vstart, ctx.n_valid, lse.contiguous(), scale)   # logits -> dlogits
        w = ctx.lm_head.weight
        ws = ctx.ws
        if ws is not None:
            # lm_head input gradient: partial tiles pushed to their owners, reduced there; ln_f backward
            # pushes its bf16 rows to every rank for the last layer's gathered gradient
            e_rs = ws.gemm_rs(logits, bf16_weight(w), True)
            linear_wgrad(logits, ln_full, grad_target(w))
            d_ln = ws.rs_reduce(e_rs, out_bf16=True)
            dx = ws.ln_bwd_ag(d_ln, x2, m, r, ctx.ln_f, None, grad_target)
            run_grad_ready_hooks(ctx.lm_head)
            run_grad_ready_hooks(ctx.ln_f)
            out = dx.view(ctx.x_shape)
            out._mmb_gathered = dx._mmb_gathered
            return (out, None, None, None, None, None, None, None) + (None,) * ctx.n_params
        d_ln = linear_dgrad(logits, bf16_weight(w))
        linear_wgrad(logits, ln_full, grad_target(w))
        if _world(ctx.group) > 1:
            d_ln = _reduce(d_ln, ctx.B, ctx.group, ctx.sp)
        dx = _ln_bwd(d_ln, x2, m, r, ctx.ln_f, want_bf16=True)
        run_grad_ready_hooks(ctx.lm_head)
        run_grad_ready_hooks(ctx.ln_f)
        out = dx.view(ctx.x_shape)
        out._mmb_bf16 = dx._mmb_bf16.view(ctx.x_shape)
        return (out, None, None, None, None, None, None, None) + (None,) * ctx.n_params
