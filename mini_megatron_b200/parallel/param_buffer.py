"""Flat parameter / gradient / bf16-shadow buffers.

Every parameter of a model chunk becomes a view into ONE contiguous fp32
buffer (``param.data``), with a matching fp32 gradient buffer
(``param.main_grad`` and ``param.grad``) and a bf16 shadow buffer
(``param.bf16``) that the GEMM kernels read.  Consequences:

* the optimizer step is one kernel over the flat buffers (AdamW writes the
  fp32 master and the bf16 shadow in the same pass; no per-GEMM casts);
* weight-gradient GEMMs accumulate straight into ``main_grad`` in fp32;
* data-parallel buckets and ZeRO-1 shards are contiguous slices, so
  reduce-scatter / all-gather need no packing.

Parameters are laid out in REVERSE registration order: backward produces
gradients from the last layer to the first, so the first bucket to become
ready is the first slice of the buffer.  Each buffer is padded to a multiple
of ``align`` elements (and every parameter starts 16-byte aligned) so that
shards split evenly across data-parallel ranks.

The reference keeps separate per-parameter fp32 tensors and casts them to
bf16 at every F.linear under autocast (main.py:93; C13 in its profile).
"""
from __future__ import annotations

from typing import Iterable, List

import torch

_ALIGN_ELEMS = 64  # 256 B for fp32, 128 B for bf16


def _round_up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


class ParamBuffer:
    """Flat fp32 params + fp32 grads + bf16 shadow, split into DP buckets.

    ``bucket_elems`` (0 = one bucket) groups consecutive parameters into
    buckets of at least that many elements; every bucket is padded to a
    multiple of ``64 * align`` elements so it splits into ``align`` (= DP size)
    equal, 256-byte-aligned shards for reduce-scatter / ZeRO-1.
    """

    def __init__(self, params: Iterable[torch.nn.Parameter], device=None, align: int = 1,
                 bf16_shadow: bool = True, bucket_elems: int = 0, allocator=None):
        params = [p for p in params if p.requires_grad]
        # de-duplicate shared parameters
        seen, uniq = set(), []
        for p in params:
            if id(p) not in seen:
                seen.add(id(p))
                uniq.append(p)
        self.params: List[torch.nn.Parameter] = list(reversed(uniq))
        self.align = max(1, align)
        device = device or (self.params[0].device if self.params else torch.device("cpu"))
        bucket_quant = _ALIGN_ELEMS * self.align
        self.offsets = []
        self.buckets = []  # (start, end, [params])
        off, b_start, b_params = 0, 0, []
        for i, p in enumerate(self.params):
            self.offsets.append(off)
            b_params.append(p)
            off = _round_up(off + p.numel(), _ALIGN_ELEMS)
            last = i == len(self.params) - 1
            if last or (bucket_elems > 0 and off - b_start >= bucket_elems):
                off = _round_up(max(off, b_start + 1), bucket_quant)
                self.buckets.append((b_start, off, b_params))
                b_start, b_params = off, []
        self.numel = max(off, bucket_quant)
        if not self.buckets:
            self.buckets.append((0, self.numel, []))
        if allocator is not None:
            # caller-provided storage (e.g. one symmetric allocation shared with NVLink peers)
            self.data, self.grad, self.bf16 = allocator(self.numel)
        else:
            self.data = torch.zeros(self.numel, dtype=torch.float32, device=device)
            self.grad = torch.zeros(self.numel, dtype=torch.float32, device=device)
            self.bf16 = torch.zeros(self.numel, dtype=torch.bfloat16, device=device) if bf16_shadow else None
        for p, o in zip(self.params, self.offsets):
            n = p.numel()
            view = self.data[o:o + n].view_as(p)
            view.copy_(p.detach().to(torch.float32))
            p.data = view
            p.main_grad = self.grad[o:o + n].view_as(p)
            p.grad = p.main_grad
            if self.bf16 is not None:
                p.bf16 = self.bf16[o:o + n].view_as(p)
            p._mmb_managed = True
            p._mmb_buffer = self
        self.refresh_bf16()

    def shard_range(self, bucket_index: int, rank: int):
        """[start, end) of ``rank``'s shard of one bucket (flat-buffer coordinates)."""
        s, e, _ = self.buckets[bucket_index]
        n = (e - s) // self.align
        return s + rank * n, s + (rank + 1) * n

    def refresh_bf16(self):
        """Re-derive the bf16 shadow from the fp32 master (after a load or external edit)."""
        if self.bf16 is not None:
            self.bf16.copy_(self.data)

    def zero_grad(self):
        self.grad.zero_()

    def param_range(self, p):
        i = self.params.index(p)
        return self.offsets[i], self.offsets[i] + p.numel()


def bf16_weight(p: torch.nn.Parameter) -> torch.Tensor:
    """bf16 copy of a weight for the GEMM kernels (shadow if managed, else a cast)."""
    if getattr(p, "_mmb_managed", False) and getattr(p, "bf16", None) is not None:
        return p.bf16
    return p.detach().to(torch.bfloat16)


def grad_target(p: torch.nn.Parameter) -> torch.Tensor:
    """fp32 tensor that a kernel accumulates this parameter's gradient into."""
    g = getattr(p, "main_grad", None)
    if g is not None:
        return g
    if p.grad is None:
        p.grad = torch.zeros_like(p, dtype=torch.float32)
    return p.grad
