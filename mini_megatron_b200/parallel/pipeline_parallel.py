"""Non-interleaved 1F1B pipeline schedule (and the legacy serial schedule).

Schedule (same op order as the reference, parallel/pipeline_parallel.py:9-32,
i.e. Megatron's non-interleaved 1F1B): stage ``r`` of ``p`` runs
``min(p-r-1, m)`` warm-up forwards, then alternates forward(next) /
backward(oldest), then drains the remaining backwards.  Bubble fraction
(p-1)/(2m+p-1) vs (p-1)/p for lock-step.

Runtime (``PipelineEngine``):

* each stage is its own autograd graph; the received activation is a leaf
  with ``requires_grad`` and its ``.grad`` is what goes upstream;
* the receive of the NEXT op is posted right after the current op is issued
  (look-ahead), so the transfer overlaps this op's compute;
* sends are fire-and-forget with at most one outstanding send kept alive;
* peers are this rank's neighbours in its pipeline group (global ranks),
  and p2p runs on NCCL (gloo on CPU).  torch's NCCL process group orders
  its communication stream after the compute stream at issue time and
  ``wait()`` orders the compute stream after it, so no host synchronisation
  is needed between ops.

Microbatch data is produced by ``batch_fn(mb) -> (tokens, labels, loss_mask)``
on every stage that needs it (first: tokens, last: labels/mask); with a
seeded generator that is the reference's "every stage draws from its own
iterator copy" (parallel/pipeline_parallel.py:180-190) made explicit.
"""
from __future__ import annotations

import contextlib
import time

import torch
import torch.distributed as dist


def build_1f1b_schedule(pp_rank, pp_size, num_microbatches):
    """Op order for one stage: list of ('F'|'B', microbatch)."""
    warmup = min(pp_size - pp_rank - 1, num_microbatches)
    ops = [("F", i) for i in range(warmup)]
    f, b = warmup, 0
    while f < num_microbatches:
        ops.append(("F", f))
        ops.append(("B", b))
        f += 1
        b += 1
    ops.extend(("B", i) for i in range(b, num_microbatches))
    return ops


def build_serial_schedule(num_microbatches):
    """All forwards, then all backwards (GPipe-style fill/drain)."""
    return [("F", i) for i in range(num_microbatches)] + [("B", i) for i in range(num_microbatches)]


class PipelineEngine:
    """Drive one optimizer step worth of microbatches through a pipeline stage.

    ``stage(x_or_tokens, labels=None, loss_mask=None)`` must return the
    activation (non-last stages) or ``(logits, loss)`` / ``loss`` (last stage).
    """

    def __init__(self, stage, pp_rank, pp_size, prev_rank, next_rank, act_shape, device,
                 act_dtype=torch.float32, schedule="1f1b", group=None, amp_ctx=None):
        self.stage = stage
        self.pp_rank, self.pp_size = pp_rank, pp_size
        self.is_first, self.is_last = pp_rank == 0, pp_rank == pp_size - 1
        self.prev, self.next = prev_rank, next_rank
        self.act_shape, self.device, self.act_dtype = tuple(act_shape), device, act_dtype
        self.schedule, self.group = schedule, group
        self.amp_ctx = amp_ctx if amp_ctx is not None else contextlib.nullcontext()

    def _recv_op(self, src):
        buf = torch.empty(self.act_shape, dtype=self.act_dtype, device=self.device)
        return buf, dist.P2POp(dist.irecv, buf, src, group=self.group)

    def run(self, batch_fn, num_microbatches, loss_scale=1.0, on_loss=None, pre_backward=None):
        """Run forward/backward for ``num_microbatches``; returns the last stage's loss tensors.

        Every op's outgoing send is issued in ONE ``batch_isend_irecv`` group
        together with the look-ahead receive of the next op.  Issuing them as
        separate calls can deadlock on NCCL once messages exceed its p2p
        buffer: a send and a receive to the same peer share a stream, so two
        neighbouring stages that each start with a send wait on each other.
        """
        m = num_microbatches
        if self.schedule == "1f1b":
            ops = build_1f1b_schedule(self.pp_rank, self.pp_size, m)
        else:
            ops = build_serial_schedule(m)
        fwd_in, fwd_out, losses = {}, {}, {}
        sends = []
        pending = {"F": None, "B": None}  # kind -> (mb, buf, work)

        def wait_sends(keep):
            while len(sends) > keep:
                work, _ = sends.pop(0)
                work.wait()

        def recv_spec(kind, mb):
            if kind == "F" and not self.is_first:
                return self._recv_op(self.prev)
            if kind == "B" and not self.is_last:
                return self._recv_op(self.next)
            return None

        def issue(send_op, send_keep, recv_kind, recv_mb):
            p2p, recv = [], None
            if send_op is not None:
                p2p.append(send_op)
            if recv_kind is not None:
                recv = recv_spec(recv_kind, recv_mb)
                if recv is not None:
                    p2p.append(recv[1])
            if not p2p:
                return
            works = dist.batch_isend_irecv(p2p)
            if send_op is not None:
                sends.append((works[0], send_keep))
            if recv is not None:
                pending[recv_kind] = (recv_mb, recv[0], works[-1])

        def take(kind, mb):
            if pending[kind] is None or pending[kind][0] != mb:
                issue(None, None, kind, mb)
            _, buf, work = pending[kind]
            work.wait()
            pending[kind] = None
            return buf

        for i, (kind, mb) in enumerate(ops):
            send_op = keep = None
            if kind == "F":
                if not self.is_first:
                    x = take("F", mb).requires_grad_(True)
                    fwd_in[mb] = x
                else:
                    x = batch_fn(mb)[0]
                with self.amp_ctx:
                    if self.is_last:
                        _, labels, mask = batch_fn(mb)
                        out = self.stage(x, labels, mask)
                        loss = out[1] if isinstance(out, tuple) else out
                        losses[mb] = loss
                        if on_loss is not None:
                            on_loss(mb, loss)
                    else:
                        out = self.stage(x)
                if not self.is_last:
                    fwd_out[mb] = out
                    keep = out.detach().contiguous()
                    send_op = dist.P2POp(dist.isend, keep, self.next, group=self.group)
            else:
                grad = None if self.is_last else take("B", mb)
                if pre_backward is not None:
                    pre_backward(mb)
                if self.is_last:
                    (losses[mb] * loss_scale).backward()
                else:
                    fwd_out[mb].backward(grad)
                if not self.is_first:
                    keep = fwd_in[mb].grad.contiguous()
                    send_op = dist.P2POp(dist.isend, keep, self.prev, group=self.group)
                fwd_in.pop(mb, None)
                fwd_out.pop(mb, None)
            nk, nmb = ops[i + 1] if i + 1 < len(ops) else (None, None)
            if nk is not None and pending[nk] is not None:
                nk = None
            issue(send_op, keep, nk, nmb)
            if kind == "B":
                wait_sends(1)
        wait_sends(0)
        return [losses[k] for k in sorted(losses)]


class _LooseStage(torch.nn.Module):
    """Adapter for the reference's loose (embedding, decoder_layers, ln_f, lm_head, loss_fn) tuple."""

    def __init__(self, embedding, decoder_layers, ln_f, lm_head, loss_fn):
        super().__init__()
        self.embedding, self.decoder_layers, self.ln_f, self.lm_head, self.loss_fn = (
            embedding, decoder_layers, ln_f, lm_head, loss_fn)

    def forward(self, x, labels=None, loss_mask=None):
        if self.embedding is not None:
            x = self.embedding(x)
        for layer in self.decoder_layers:
            x = layer(x)
        if self.lm_head is not None:
            logits = self.lm_head(self.ln_f(x))
            return logits, self.loss_fn(logits, labels, loss_mask)
        return x


def _compat_train(schedule, embedding, decoder_layers, ln_f, lm_head, loss_fn, optimizer, scheduler, data_iter, B,
                  S, V, device, num_microbatches, pp_rank, pp_size, rank, hidden_size, tp_size=1, log_interval=10,
                  dp_group=None, amp_ctx=None):
    from .data_parallel import allreduce_grads
    stage = _LooseStage(embedding, decoder_layers, ln_f, lm_head, loss_fn)
    prev_rank = rank - tp_size if pp_rank > 0 else None
    next_rank = rank + tp_size if pp_rank < pp_size - 1 else None
    engine = PipelineEngine(stage, pp_rank, pp_size, prev_rank, next_rank, (B, S, hidden_size), device,
                            schedule=schedule, amp_ctx=amp_ctx)
    # every stage walks the same iterator in microbatch order (first uses tokens, last uses labels)
    cache = {}

    def batch_fn(mb):
        while mb not in cache:
            cache[len(cache)] = next(data_iter)
        tok, lab = cache[mb]
        return tok.to(device), lab.to(device), torch.ones(B, S, dtype=torch.float32, device=device)

    params = list(optimizer.param_groups[0]["params"])
    optimizer.zero_grad()
    if torch.cuda.is_available() and str(device).startswith("cuda"):
        torch.cuda.synchronize()
    start = time.perf_counter()

    def log(mb, loss):
        if (mb + 1) % log_interval == 0 and pp_rank == pp_size - 1 and rank == (pp_size - 1) * tp_size:
            print(f"step {mb + 1:4d} | loss {loss.item():.4f}")

    losses = engine.run(batch_fn, num_microbatches, on_loss=log)
    if dp_group is not None:
        allreduce_grads(params, dp_group)
    optimizer.step()
    scheduler.step()
    if torch.cuda.is_available() and str(device).startswith("cuda"):
        torch.cuda.synchronize()
    elapsed = time.perf_counter() - start
    if losses and pp_rank == pp_size - 1:
        tput = B * S * num_microbatches / elapsed
        peak = torch.cuda.max_memory_allocated() / 1024 ** 3 if torch.cuda.is_available() else 0.0
        print(f"\n{'=' * 60}\nMini-Megatron PP Results ({schedule.upper()})\n{'=' * 60}")
        print(f"PP={pp_size}  |  Micro-batches: {num_microbatches}")
        print(f"Throughput:      {tput:,.0f} tok/s")
        print(f"Peak memory:     {peak:.2f} GB/GPU")
        print(f"Final loss:      {losses[-1].item():.4f}\n{'=' * 60}\n")
    return elapsed


def train_pipeline_1f1b(*args, **kwargs):
    """Reference-compatible entry point (parallel/pipeline_parallel.py:132 signature)."""
    return _compat_train("1f1b", *args, **kwargs)


def train_pipeline(*args, **kwargs):
    """Reference-compatible serial schedule (all forwards, then all backwards; no skipped backwards)."""
    return _compat_train("serial", *args, **kwargs)
