"""Numerical parity gates between two implementations of the same model.

The gate compares, for identical initial weights and one fixed next-token
batch: the logits, the loss, every parameter gradient, and every parameter
after one AdamW step; initial weights must match exactly.  Two views are
always reported side by side:

* **per-tensor** -- the worst relative L2 over all parameters (the original
  gate of the reference's campaign);
* **global** -- one relative L2 over all parameters together plus the
  largest absolute difference (the calibrated view, robust to near-zero
  LayerNorm biases whose per-tensor relative error is unstable).

Gate sets (``GATES``): ``fp32`` and ``fp32-tp`` are the reference's fp32
thresholds (experiments/validate_mcore_equivalence.py:130-134; the amended
TP parameter bound from its TP calibration); ``pp-calibrated`` is its global
PP calibration (experiments/summarize_fair_pp_gate.py:26-33).  ``bf16`` is
this framework's gate for its bf16 tensor-core path against an fp32 or bf16
autocast reference: thresholds sized to bf16 operand rounding (8 mantissa
bits), evaluated on the global view.

    python -m mini_megatron_b200.harness.parity --impl-a reference --impl-b ours [--device cuda] [--amp]

``reference`` builds the reference's modules from ``baseline/_ref`` (its own
code, unmodified); ``ours`` builds this framework's GPT (native kernels on
CUDA, eager PyTorch modules on CPU).
"""
from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import sys
from pathlib import Path

import torch

from .contract import CONTRACT, from_reference_state, full_parameter_names, tensor_digest, to_reference_state

REPO = Path(__file__).resolve().parents[2]

GATES = {
    "fp32": {"view": "per_tensor", "loss_abs": 3e-4, "logits_relative_l2": 5e-4, "gradient_relative_l2": 5e-4,
             "parameter_relative_l2": 1e-4},
    "fp32-tp": {"view": "per_tensor", "loss_abs": 3e-4, "logits_relative_l2": 5e-4, "gradient_relative_l2": 5e-4,
                "parameter_relative_l2": 1.25e-4},
    "pp-calibrated": {"view": "global", "loss_abs": 3e-4, "logits_relative_l2": 5e-4,
                      "gradient_relative_l2": 6.5e-4, "parameter_relative_l2": 1.25e-4,
                      "parameter_max_abs": 1.25e-3},
    "bf16": {"view": "global", "loss_abs": 2e-2, "logits_relative_l2": 2e-2, "gradient_relative_l2": 5e-2,
             "parameter_relative_l2": 2e-3, "parameter_max_abs": 2.5e-3},
}


def relative_l2(a, b) -> float:
    a, b = a.detach().float(), b.detach().float()
    return float((a - b).norm() / a.norm().clamp_min(1e-12))


def max_abs(a, b) -> float:
    return float((a.detach().float() - b.detach().float()).abs().max()) if a.numel() else 0.0


def compare_tensors(left: dict, right: dict, names) -> dict:
    """Per-tensor and global comparison of two name -> tensor maps (left is the yardstick)."""
    rows, dsq, rsq, worst_abs = [], 0.0, 0.0, 0.0
    for n in names:
        a, b = left[n].detach().float().cpu(), right[n].detach().float().cpu()
        if a.shape != b.shape:
            raise ValueError(f"shape mismatch for {n}: {tuple(a.shape)} vs {tuple(b.shape)}")
        d = a - b
        m = float(d.abs().max()) if d.numel() else 0.0
        rows.append({"parameter": n, "max_abs": m, "relative_l2": relative_l2(a, b)})
        dsq += float(d.square().sum())
        rsq += float(a.square().sum())
        worst_abs = max(worst_abs, m)
    return {"count": len(rows), "global_relative_l2": math.sqrt(dsq) / max(math.sqrt(rsq), 1e-12),
            "global_max_abs": worst_abs, "worst_relative_l2": max(rows, key=lambda r: r["relative_l2"]),
            "worst_max_abs": max(rows, key=lambda r: r["max_abs"])}


def evaluate(report: dict, gate: dict) -> dict:
    """Apply one gate set to a parity report; returns {check: bool} plus 'passed'."""
    view = gate["view"]
    g, p = report["gradients"], report["parameters_after_one_step"]
    if view == "per_tensor":
        grad_v, par_v = g["worst_relative_l2"]["relative_l2"], p["worst_relative_l2"]["relative_l2"]
    else:
        grad_v, par_v = g["global_relative_l2"], p["global_relative_l2"]
    checks = {"initial_weights_exact": report["initial_parameters"]["global_max_abs"] == 0.0,
              "loss_abs": report["loss_abs"] <= gate["loss_abs"],
              "logits_relative_l2": report["logits_relative_l2"] <= gate["logits_relative_l2"],
              "gradient_relative_l2": grad_v <= gate["gradient_relative_l2"],
              "parameter_relative_l2": par_v <= gate["parameter_relative_l2"]}
    if "parameter_max_abs" in gate:
        checks["parameter_max_abs"] = p["global_max_abs"] <= gate["parameter_max_abs"]
    checks["passed"] = all(checks.values())
    return checks


# ----------------------------------------------------------------------------- implementations
class _Impl:
    """One implementation under test: params(), forward(tokens, labels, mask) -> (logits, loss), step()."""

    def params(self) -> dict: ...
    def grads(self) -> dict: ...


def _ref_modules():
    ref = REPO / "baseline" / "_ref"
    if not (ref / "model" / "transformer.py").exists():
        raise RuntimeError("reference sources not present under baseline/_ref")
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    import config as rcfg
    from model.embedding import Embedding
    from model.loss import CrossEntropyLoss
    from model.transformer import GPT, Decoder
    from parallel.process_groups import set_model_parallel
    from parallel.tensor_parallel import ColumnParallelLinear
    return rcfg, Embedding, CrossEntropyLoss, GPT, Decoder, set_model_parallel, ColumnParallelLinear


class ReferenceImpl(_Impl):
    """The reference's own modules and torch AdamW (its main.py training step)."""

    def __init__(self, mc, device, amp, lr=6e-4, weight_decay=0.1):
        rcfg, Embedding, CE, GPT, Decoder, set_mp, Column = _ref_modules()
        set_mp(None)
        V, H = mc["vocab_size"], mc["hidden_size"]
        self.model = GPT(Embedding(V, H, mc["max_seq_len"]), Decoder(H, mc["num_attention_heads"],
                                                                     mc["ffn_hidden_size"], mc["num_layers"]),
                         torch.nn.LayerNorm(H), Column(H, V, bias=False, gather_output=True), CE()).to(device)
        self.opt = torch.optim.AdamW(self.model.parameters(), lr=lr, weight_decay=weight_decay, betas=(0.9, 0.999),
                                     fused=False)
        self.amp = amp
        self.device = device

    def params(self):
        return {n: p.detach().clone() for n, p in self.model.named_parameters()}

    def grads(self):
        return {n: p.grad.detach().clone() for n, p in self.model.named_parameters()}

    def load(self, state):
        self.model.load_state_dict(state, strict=True)

    def forward_backward(self, tokens, labels, mask):
        ctx = torch.autocast(self.device.type, dtype=torch.bfloat16) if self.amp else contextlib.nullcontext()
        self.opt.zero_grad(set_to_none=True)
        with ctx:
            logits, loss = self.model(tokens, labels, mask)
        loss.backward()
        return logits.detach().float().clone(), float(loss.detach())

    def step(self):
        self.opt.step()


class OursImpl(_Impl):
    """This framework's GPT (native kernels on CUDA) with its AdamW over the flat buffer."""

    def __init__(self, mc, device, lr=6e-4, weight_decay=0.1):
        from ..config import GPTConfig
        from ..models.gpt import build_gpt
        from ..optim import FusedAdamW, make_param_buffer
        from ..parallel import process_groups as pg
        pg.set_model_parallel(None)
        self.cfg = GPTConfig(**{k: mc[k] for k in ("num_layers", "hidden_size", "num_attention_heads",
                                                   "ffn_hidden_size", "max_seq_len", "vocab_size")})
        self.model = build_gpt(self.cfg).to(device)
        self.device = device
        if device.type == "cuda":
            make_param_buffer(self.model)
        self.opt = FusedAdamW(self.model.parameters(), lr=lr, weight_decay=weight_decay, betas=(0.9, 0.999))

    def params(self):
        return to_reference_state({n: p.detach().clone() for n, p in self.model.named_parameters()},
                                  self.cfg.vocab_size)

    def grads(self):
        out = {}
        for n, p in self.model.named_parameters():
            g = getattr(p, "main_grad", None)
            out[n] = (g if g is not None else p.grad).detach().clone()
        return to_reference_state(out, self.cfg.vocab_size)

    def load(self, state):
        with torch.no_grad():
            padded = from_reference_state(state, self.model.embedding.token_embedding.weight.size(0))
            for n, p in self.model.named_parameters():
                p.copy_(padded[n])
            buf = getattr(next(self.model.parameters()), "_mmb_buffer", None)
            if buf is not None:
                buf.refresh_bf16()

    def forward_backward(self, tokens, labels, mask):
        self.opt.zero_grad()
        logits, loss = self.model(tokens, labels, mask)
        logits = logits[..., :self.cfg.vocab_size].detach().float().clone()  # overwritten by its grad in backward
        loss.backward()
        return logits, float(loss.detach())

    def step(self):
        self.opt.step()


def build_impl(kind, mc, device, amp):
    if kind == "reference":
        return ReferenceImpl(mc, device, amp)
    if kind == "ours":
        return OursImpl(mc, device)
    raise ValueError(kind)


def fixed_batch(batch_size, seq_len, vocab, seed):
    """Uniform tokens from an explicit CPU generator; labels = next token, last = -100."""
    g = torch.Generator().manual_seed(seed)
    tokens = torch.randint(0, vocab, (batch_size, seq_len), generator=g, dtype=torch.long)
    labels = torch.roll(tokens, -1, dims=1)
    labels[:, -1] = -100
    return tokens, labels, (labels != -100).float()


def run_parity(a, b, mc, tokens, labels, mask, device) -> dict:
    """Copy a's initial weights into b, run one step on both, compare (a is the yardstick)."""
    b.load(a.params())
    names = full_parameter_names(mc)
    init = compare_tensors(a.params(), b.params(), names)
    t, l, m = tokens.to(device), labels.to(device), mask.to(device)
    la, lossa = a.forward_backward(t, l, m)
    lb, lossb = b.forward_backward(t, l, m)
    keep = m.bool()
    grads = compare_tensors(a.grads(), b.grads(), names)
    a.step()
    b.step()
    params = compare_tensors(a.params(), b.params(), names)
    return {"schema_version": 1, "contract": CONTRACT, "batch_shape": list(tokens.shape),
            "input_sha256": tensor_digest(tokens), "mapped_parameters": len(names),
            "initial_parameters": init, "loss_a": lossa, "loss_b": lossb, "loss_abs": abs(lossa - lossb),
            "logits_relative_l2": relative_l2(la[keep], lb[keep]), "logits_max_abs": max_abs(la[keep], lb[keep]),
            "gradients": grads, "parameters_after_one_step": params}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--impl-a", default="reference", choices=("reference", "ours"))
    ap.add_argument("--impl-b", default="ours", choices=("reference", "ours"))
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--amp", action="store_true", help="bf16 autocast for the reference implementation")
    ap.add_argument("--amp-b", action="store_true",
                    help="bf16 autocast for impl b only (e.g. the reference in fp32 against itself under autocast)")
    ap.add_argument("--no-tf32", action="store_true", help="full fp32 matmuls for the fp32 reference (no TF32)")
    ap.add_argument("--preset", default="gpt-125m")
    ap.add_argument("--seq-len", type=int, default=None)
    ap.add_argument("--batch-size", type=int, default=2)
    ap.add_argument("--seed", type=int, default=20260818)
    ap.add_argument("--gate", default=None, choices=sorted(GATES))
    ap.add_argument("--output")
    args = ap.parse_args(argv)
    from ..config import PRESETS
    c = PRESETS[args.preset]
    mc = dict(num_layers=c.num_layers, hidden_size=c.hidden_size, num_attention_heads=c.num_attention_heads,
              ffn_hidden_size=c.ffn_hidden_size, max_seq_len=args.seq_len or c.max_seq_len, vocab_size=c.vocab_size)
    device = torch.device(args.device)
    if device.type == "cuda":
        torch.cuda.set_device(device.index or 0)
    import torch.distributed as dist
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29400 + os.getpid() % 500))
        dist.init_process_group("gloo", rank=0, world_size=1)
    torch.manual_seed(args.seed)
    if args.no_tf32:
        torch.backends.cuda.matmul.allow_tf32 = False
        torch.backends.cudnn.allow_tf32 = False
    a = build_impl(args.impl_a, mc, device, args.amp)
    b = build_impl(args.impl_b, mc, device, args.amp or args.amp_b)
    tokens, labels, mask = fixed_batch(args.batch_size, mc["max_seq_len"], mc["vocab_size"], args.seed + 1)
    rep = run_parity(a, b, mc, tokens, labels, mask, device)
    native = any(k == "ours" for k in (args.impl_a, args.impl_b)) and device.type == "cuda"
    gate_name = args.gate or ("bf16" if (native or args.amp or args.amp_b) else "fp32")
    rep.update({"impl_a": args.impl_a, "impl_b": args.impl_b, "device": str(device), "amp": args.amp,
                "amp_b": args.amp_b, "tf32": not args.no_tf32,
                "model": mc, "gate_name": gate_name, "gate": GATES[gate_name],
                "checks": evaluate(rep, GATES[gate_name])})
    rep["passed"] = rep["checks"]["passed"]
    text = json.dumps(rep, indent=2, sort_keys=True)
    print(text)
    if args.output:
        Path(args.output).parent.mkdir(parents=True, exist_ok=True)
        Path(args.output).write_text(text + "\n", encoding="utf-8")
    return 0 if rep["passed"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
