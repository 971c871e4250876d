"""Fused tensor-parallel collectives (sequence-parallel dataflow over NVLink).

With sequence parallelism every activation between tensor-parallel GEMMs is
sharded along the sequence.  Instead of NCCL all-gathers / reduce-scatters,
the kernels around each collective do the communication themselves:

* **LayerNorm + all-gather** (``layernorm_fwd_push`` / ``layernorm_bwd_push``):
  the kernel that produces a sequence shard writes every bf16 row straight into
  each TP rank's gathered buffer and the last CTA raises this rank's flag;
* **all-gather -> GEMM** (``gemm_tp`` with ``ag_flags``): the Column GEMM's TMA
  producer waits, per source rank, for that rank's flag before loading its
  rows, so tiles of already-arrived shards (the local one first) start at once;
* **GEMM -> reduce-scatter** (``gemm_tp`` with ``EPI_PUSH_BF16``): the Row GEMM's
  epilogue pushes each partial output tile into the owning rank's per-source
  slot; ``tp_rs_reduce`` waits for all sources and sums the slots plus the
  residual;
* **head**: ``ln_f`` pushes its rows like the layer LayerNorms, the lm_head GEMM
  with the cross-entropy statistics epilogue waits per source rank, the
  per-row (max, sum-exp, target) triplets of each vocabulary shard are pushed
  to every rank and combined by ``tp_ce_allreduce``, and the lm_head input
  gradient goes through the same reduce-scatter push as a Row GEMM.

``TPWorkspace`` owns the symmetric buffers of one model chunk: a signal pad
(all-gather flags, reduce-scatter flags), two gathered buffers per decoder
layer for the forward (kept for the weight gradients), two alternating
gathered buffers for the backward, and the reduce-scatter slots.  Flags carry
epochs from two counters (one per collective kind) that every rank advances
in the same order; every device-side wait is bounded.

Reference: the reference's TP all-reduces (comm/all_reduce.py:5-43) and its
unwired sequence-parallel helpers (comm/sequence_parallel.py:8-53).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..comm.symmetric import SymmetricBuffer
from ..ops import native


class TPWorkspace:
    # int32 flags: [0:8] all-gather, [8:16] reduce-scatter, [16:24] cross-entropy statistics, [24:32] embedding
    # rows, [32:40] published embedding gradients, [40:48] position-table gradient, [48:56] small-vector sums
    SIG_BYTES = 4096

    def __init__(self, tp_group, B: int, S: int, H: int, num_fwd_slots: int, copy_saved: bool = False,
                 vec_elems: int = 0):
        self.group = tp_group
        self.world = dist.get_world_size(tp_group)
        self.rank = dist.get_rank(tp_group)
        if self.world > 8:
            raise ValueError("fused TP supports up to 8 ranks (one NVSwitch node)")
        if S % self.world or (S // self.world) % 128:
            raise ValueError("fused TP needs seq_len / tp to be a multiple of 128")
        self.B, self.S, self.H = B, S, H
        self.Sl = S // self.world
        self.rows, self.rows_l = B * S, B * self.Sl
        self.copy_saved = copy_saved
        slot_bytes = self.rows * H * 2
        self.off_fwd = self.SIG_BYTES
        self.off_bwd = self.off_fwd + num_fwd_slots * slot_bytes
        self.off_rs = self.off_bwd + 2 * slot_bytes
        self.off_ce = self.off_rs + self.world * self.rows_l * H * 2   # [world][rows] float4 (mx, se, tg, -)
        self.off_embo = self.off_ce + self.world * self.rows * 16      # [rows_l, H] fp32 embedding rows (pushed in)
        self.off_embd = self.off_embo + self.rows_l * H * 4            # [rows_l, H] fp32 embedding gradient (published)
        self.off_posg = self.off_embd + self.rows_l * H * 4            # [S, H] fp32 position-table gradient
        self.off_vec = self.off_posg + S * H * 4                       # [world][vec_elems] fp32
        self.vec_elems = vec_elems
        total = self.off_vec + self.world * max(vec_elems, 1) * 4
        self.num_fwd_slots = num_fwd_slots
        self.slot_bytes = slot_bytes
        self.symm = SymmetricBuffer(total, tp_group)
        dev = self.symm.device
        self.counters = torch.zeros(16, dtype=torch.int32, device=dev)
        self.ag_flag_ptrs = [self.symm.peer_ptr(r, 0) for r in range(self.world)]
        self.rs_flag_ptrs = [self.symm.peer_ptr(r, 32) for r in range(self.world)]
        self.ce_flag_ptrs = [self.symm.peer_ptr(r, 64) for r in range(self.world)]
        self.emb_flag_ptrs = [self.symm.peer_ptr(r, 96) for r in range(self.world)]
        self.pub_flag_ptrs = [self.symm.peer_ptr(r, 128) for r in range(self.world)]
        self.pos_flag_ptrs = [self.symm.peer_ptr(r, 160) for r in range(self.world)]
        self.vec_flag_ptrs = [self.symm.peer_ptr(r, 192) for r in range(self.world)]
        self.ag_epoch = 0
        self.rs_epoch = 0
        self.ce_epoch = 0
        self.emb_epoch = self.pub_epoch = self.pos_epoch = self.vec_epoch = 0
        self._bwd_next = 0
        dist.barrier(group=tp_group)

    # ---------------------------------------------------------------- debugging
    def poison(self):
        """NaN-fill every data region (not the flags) of this rank's workspace.

        Run between steps with all ranks idle (the caller synchronises and
        barriers around it): any read of a gathered row or reduce-scatter slot
        that its producer has not written in the current step then shows up as
        NaN in the loss.  Enabled by ``MMB_POISON_SYMM=1``.
        """
        torch.cuda.synchronize(self.symm.device)
        dist.barrier(group=self.group)
        self.symm.poison(self.SIG_BYTES)
        torch.cuda.synchronize(self.symm.device)
        dist.barrier(group=self.group)

    # ---------------------------------------------------------------- buffers
    def fwd_ptrs(self, i):
        return [self.symm.peer_ptr(r, self.off_fwd + i * self.slot_bytes) for r in range(self.world)]

    def fwd_view(self, i):
        return self.symm.tensor(self.off_fwd + i * self.slot_bytes, self.rows * self.H, torch.bfloat16).view(
            self.rows, self.H)

    def next_bwd(self):
        k = self._bwd_next
        self._bwd_next ^= 1
        return k

    def bwd_ptrs(self, k):
        return [self.symm.peer_ptr(r, self.off_bwd + k * self.slot_bytes) for r in range(self.world)]

    def bwd_view(self, k):
        return self.symm.tensor(self.off_bwd + k * self.slot_bytes, self.rows * self.H, torch.bfloat16).view(
            self.rows, self.H)

    def rs_dst_ptrs(self):
        """For each owner rank: where THIS rank's partial rows go in the owner's slots."""
        stride = self.rows_l * self.H * 2
        return [self.symm.peer_ptr(r, self.off_rs + self.rank * stride) for r in range(self.world)]

    @property
    def rs_local_ptr(self):
        return self.symm.peer_ptr(self.rank, self.off_rs)

    # ---------------------------------------------------------------- fused ops
    def ln_fwd_ag(self, x2, ln, slot):
        """LayerNorm of the local shard; rows land in every rank's forward slot ``slot``."""
        C = native()
        self.ag_epoch += 1
        mean = torch.empty(x2.shape[0], device=x2.device, dtype=torch.float32)
        rstd = torch.empty_like(mean)
        C.layernorm_fwd_push(x2, ln.weight.detach(), ln.bias.detach(), mean, rstd, ln.eps, self.fwd_ptrs(slot),
                             self.ag_flag_ptrs, self.rank, self.ag_epoch, self.S, self.Sl, self.counters[0:1])
        return self.fwd_view(slot), mean, rstd, self.ag_epoch

    def ln_bwd_ag(self, dy_bf16, x2, mean, rstd, ln, dres, grad_target):
        """LayerNorm backward of the local shard; bf16 dx rows land in every rank's next backward slot."""
        C = native()
        k = self.next_bwd()
        self.ag_epoch += 1
        dx = torch.empty_like(x2)
        C.layernorm_bwd_push(dy_bf16, x2, mean, rstd, ln.weight.detach(), dres, dx, grad_target(ln.weight),
                             grad_target(ln.bias), self.bwd_ptrs(k), self.ag_flag_ptrs, self.rank, self.ag_epoch,
                             self.S, self.Sl, self.counters[1:2])
        dx._mmb_gathered = (self.bwd_view(k), self.ag_epoch)
        return dx

    def gather_grad(self, d_local):
        """Gathered bf16 copy of a local gradient shard: reuses the producer's push if there was one."""
        g = getattr(d_local, "_mmb_gathered", None)
        if g is not None:
            return g
        C = native()
        k = self.next_bwd()
        self.ag_epoch += 1
        src = d_local.reshape(-1, self.H).to(torch.bfloat16).contiguous()
        C.tp_ag_push(src, self.bwd_ptrs(k), self.ag_flag_ptrs, self.rank, self.ag_epoch, self.S, self.Sl,
                     self.counters[2:3])
        return self.bwd_view(k), self.ag_epoch

    def gemm_ag(self, A_full, ag_epoch, W, w_mn, out, epi=0, aux=None):
        """out = A_full (gathered, waited on per source rank) x W (Column forward / Row dgrad)."""
        native().gemm_tp(A_full, False, W, w_mn, out, epi, aux, self.ag_flag_ptrs[self.rank], ag_epoch, self.S,
                         self.Sl, [], [], self.rank, 0, None, out.shape[1])
        return out

    def gemm_rs(self, A, W, w_mn):
        """Partial A x W pushed tile by tile to the owning ranks' reduce-scatter slots."""
        C = native()
        self.rs_epoch += 1
        C.gemm_tp(A, False, W, w_mn, None, C.EPI_PUSH_BF16, None, 0, 0, self.S, self.Sl, self.rs_dst_ptrs(),
                  self.rs_flag_ptrs, self.rank, self.rs_epoch, self.counters[3:4], self.H)
        return self.rs_epoch

    def rs_reduce(self, epoch, resid=None, out_bf16=False):
        """Wait for every rank's partial rows of this shard; return resid + sum (fp32) or the sum in bf16."""
        C = native()
        n = self.rows_l * self.H
        dev = self.symm.device
        if out_bf16:
            o16 = torch.empty(self.rows_l, self.H, device=dev, dtype=torch.bfloat16)
            C.tp_rs_reduce(self.rs_local_ptr, n, self.world, self.rs_flag_ptrs[self.rank], epoch, resid, None, o16, n)
            return o16
        out = torch.empty(self.rows_l, self.H, device=dev, dtype=torch.float32)
        C.tp_rs_reduce(self.rs_local_ptr, n, self.world, self.rs_flag_ptrs[self.rank], epoch, resid, out, None, n)
        return out

    def gemm_ce(self, A_full, ag_epoch, W, logits, labels, vocab_start, n_valid):
        """lm_head GEMM on the gathered rows (waiting per source rank) with cross-entropy statistics."""
        return native().gemm_ce_stats(A_full, W, logits, labels, vocab_start, n_valid, self.ag_flag_ptrs[self.rank],
                                      ag_epoch, self.S, self.Sl, self.rank)

    def ce_allreduce(self, mx, se, tg):
        """(lse, target logit) of every row over the whole vocabulary from each rank's shard statistics."""
        self.ce_epoch += 1
        dst = [self.symm.peer_ptr(r, self.off_ce) for r in range(self.world)]
        return native().tp_ce_allreduce(mx.contiguous(), se.contiguous(), tg.contiguous(), dst, self.ce_flag_ptrs,
                                        self.rank, self.ce_epoch, self.counters[4:5],
                                        self.symm.peer_ptr(self.rank, self.off_ce), self.ce_flag_ptrs[self.rank])

    def _ptrs(self, off):
        return [self.symm.peer_ptr(r, off) for r in range(self.world)]

    def emb_fwd(self, ids, tok_w, pos_w, vstart, vend):
        """Embedding of this rank's sequence shard: every vocabulary owner writes tok + pos of the
        rows whose token it holds into the rows' sequence owner (no reduction: one writer per row)."""
        C = native()
        self.emb_epoch += 1
        C.tp_emb_fwd_push(ids, tok_w, pos_w, self._ptrs(self.off_embo), self.emb_flag_ptrs, self.rank,
                          self.emb_epoch, self.S, self.Sl, self.counters[5:6], vstart, vend)
        out = torch.empty(self.rows_l, self.H, device=self.symm.device, dtype=torch.float32)
        C.tp_wait_copy(self.symm.peer_ptr(self.rank, self.off_embo), out, 0, self.emb_flag_ptrs[self.rank],
                       self.world, self.emb_epoch)
        return out

    def emb_bwd(self, ids, d_local, tok_grad, pos_grad, vstart, vend):
        """Token-table gradient from every rank's gradient rows (read over NVLink by the row owner),
        and the full position-table gradient on every rank (each rank pushes its shard's rows)."""
        C = native()
        self.pub_epoch += 1
        C.tp_publish(d_local, self._ptrs(self.off_embd), self.pub_flag_ptrs, self.rank, self.pub_epoch,
                     self.counters[6:7])
        C.embedding_bwd_peers(ids, self._ptrs(self.off_embd), self.pub_flag_ptrs[self.rank], self.pub_epoch, self.S,
                              self.Sl, tok_grad, vstart, vend)
        if pos_grad is not None:
            self.pos_epoch += 1
            C.tp_pos_grad_push(d_local, self.B, self._ptrs(self.off_posg), self.pos_flag_ptrs, self.rank,
                               self.pos_epoch, self.S, self.Sl, self.counters[7:8])
            C.tp_wait_copy(self.symm.peer_ptr(self.rank, self.off_posg), pos_grad[:self.S], 1,
                           self.pos_flag_ptrs[self.rank], self.world, self.pos_epoch)

    def vec_allreduce(self, grads):
        """In-place sum over the TP group of a few small fp32 tensors (sequence-parallel LayerNorm grads)."""
        flat = torch.cat([g.reshape(-1) for g in grads])
        if flat.numel() > self.vec_elems:
            raise ValueError("TP workspace sized for fewer vector elements")
        self.vec_epoch += 1
        out = torch.empty_like(flat)
        native().tp_vec_allreduce(flat, out, self._ptrs(self.off_vec), self.vec_flag_ptrs, self.rank, self.vec_epoch,
                                  self.counters[8:9], self.symm.peer_ptr(self.rank, self.off_vec),
                                  self.vec_flag_ptrs[self.rank])
        off = 0
        for g in grads:
            n = g.numel()
            g.copy_(out[off:off + n].view_as(g))
            off += n

    def close(self):
        if self.symm is not None:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            self.symm.close()
            self.symm = None
