"""AdamW over flat parameter buffers.

``FusedAdamW`` is a ``torch.optim.Optimizer`` (so ``LambdaLR`` and friends work
and ``state_dict()`` has torch AdamW's layout: per-parameter ``step``,
``exp_avg``, ``exp_avg_sq`` plus ``param_groups``), but on CUDA the whole
step is one kernel per flat buffer (see csrc/adamw.cu): fp32 master, both
moments and the bf16 GEMM shadow are updated in a single pass.  On CPU it
performs torch's single-tensor AdamW arithmetic per parameter, which is what
the CPU parity tests compare against ``torch.optim.AdamW``.

Reference: ``AdamW(model.parameters(), lr=6e-4, weight_decay=0.1, fused=...)``
(main.py:144,177) -- weight decay applies to every parameter, as there.
"""
from __future__ import annotations

import math

import torch

from .parallel.param_buffer import ParamBuffer


class FusedAdamW(torch.optim.Optimizer):
    def __init__(self, params, lr=6e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01, grad_scale=1.0):
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        super().__init__(params, defaults)
        self.grad_scale = grad_scale
        self._step = 0
        self._buffers = []          # [(ParamBuffer, exp_avg, exp_avg_sq)]
        self._loose = []            # params not in a managed buffer
        buffers = {}
        for group in self.param_groups:
            for p in group["params"]:
                buf = getattr(p, "_mmb_buffer", None)
                if buf is not None and p.is_cuda:
                    buffers.setdefault(id(buf), buf)
                else:
                    self._loose.append(p)
        for buf in buffers.values():
            m = torch.zeros_like(buf.data)
            v = torch.zeros_like(buf.data)
            self._buffers.append((buf, m, v))
            for p, o in zip(buf.params, buf.offsets):
                n = p.numel()
                self.state[p] = {"exp_avg": m[o:o + n].view_as(p), "exp_avg_sq": v[o:o + n].view_as(p)}

    def enable_device_schedule(self, lr_table: torch.Tensor):
        """Read lr and the step count from device memory, so a captured step replays correctly.

        ``lr_table[i]`` is the learning rate of optimizer step ``i + 1`` (the
        LR schedule evaluated ahead of time); a device int32 step counter,
        advanced by a one-thread kernel inside the step, indexes it and the
        bias corrections are derived from it on the device.  Only the flat
        CUDA buffers are supported (no loose parameters).
        """
        if self._loose:
            raise ValueError("device-side schedule needs every parameter in a flat CUDA buffer")
        dev = self._buffers[0][0].data.device
        self._dev_step = torch.tensor([self._step], dtype=torch.int32, device=dev)
        self._dev_hyper = torch.zeros(4, dtype=torch.float32, device=dev)
        self._lr_table = lr_table.to(device=dev, dtype=torch.float32).contiguous()

    def advance_host_counters(self):
        """Host-side bookkeeping of one replayed step (the replay itself advances the device counter)."""
        self._step += 1

    @torch.no_grad()
    def step(self, closure=None):
        loss = closure() if closure is not None else None
        self._step += 1
        g0 = self.param_groups[0]
        lr, (b1, b2), eps, wd = g0["lr"], g0["betas"], g0["eps"], g0["weight_decay"]
        if self._buffers:
            from .ops import native
            C = native()
            if getattr(self, "_lr_table", None) is not None:
                C.adamw_hyper_step(self._dev_step, self._lr_table, b1, b2, self._dev_hyper)
                for buf, m, v in self._buffers:
                    C.adamw_flat_dev(buf.data, buf.grad, m, v, buf.bf16, self._dev_hyper, b1, b2, eps, wd,
                                     self.grad_scale)
            else:
                for buf, m, v in self._buffers:
                    C.adamw_flat(buf.data, buf.grad, m, v, buf.bf16, lr, b1, b2, eps, wd, self._step,
                                 self.grad_scale)
        bc1 = 1 - b1 ** self._step
        bc2_sqrt = math.sqrt(1 - b2 ** self._step)
        for group in self.param_groups:
            lr, (b1, b2), eps, wd = group["lr"], group["betas"], group["eps"], group["weight_decay"]
            for p in group["params"]:
                if getattr(p, "_mmb_buffer", None) is not None and p.is_cuda:
                    continue
                if p.grad is None:
                    continue
                st = self.state[p]
                if "exp_avg" not in st:
                    st["exp_avg"] = torch.zeros_like(p)
                    st["exp_avg_sq"] = torch.zeros_like(p)
                g = p.grad if self.grad_scale == 1.0 else p.grad * self.grad_scale
                p.mul_(1 - lr * wd)
                st["exp_avg"].lerp_(g, 1 - b1)
                st["exp_avg_sq"].mul_(b2).addcmul_(g, g, value=1 - b2)
                denom = (st["exp_avg_sq"].sqrt() / bc2_sqrt).add_(eps)
                p.addcdiv_(st["exp_avg"], denom, value=-lr / bc1)
        return loss

    def zero_grad(self, set_to_none: bool = False):
        for buf, _, _ in self._buffers:
            buf.zero_grad()
        for p in self._loose:
            if p.grad is not None:
                if set_to_none:
                    p.grad = None
                else:
                    p.grad.zero_()

    def state_dict(self):
        for group in self.param_groups:
            for p in group["params"]:
                self.state.setdefault(p, {})
                if "exp_avg" in self.state[p]:
                    self.state[p]["step"] = torch.tensor(float(self._step))
        return super().state_dict()

    def load_state_dict(self, state_dict):
        views = {p: dict(st) for p, st in self.state.items()}
        super().load_state_dict(state_dict)
        steps = []
        for p, st in self.state.items():
            if "step" in st:
                steps.append(int(float(st["step"])))
            if p in views and "exp_avg" in views[p]:
                # copy loaded moments into the flat buffers and keep the views
                for k in ("exp_avg", "exp_avg_sq"):
                    if k in st:
                        views[p][k].copy_(st[k])
                        st[k] = views[p][k]
        self._step = max(steps) if steps else 0
        if getattr(self, "_dev_step", None) is not None:
            self._dev_step.fill_(self._step)
        for buf, _, _ in self._buffers:
            buf.refresh_bf16()


def make_param_buffer(module: torch.nn.Module, align: int = 1, bucket_elems: int = 0) -> ParamBuffer:
    """Flatten ``module``'s parameters into one managed buffer (training path)."""
    return ParamBuffer(module.parameters(), align=align, bucket_elems=bucket_elems)
