"""Training engine: one object that owns topology, model chunk, optimizer, schedule.

``Trainer(cfg).train_step(tokens, labels)`` runs ONE optimizer step:
``num_microbatches`` forward/backward passes (through the 1F1B pipeline when
pp > 1), the data-parallel gradient reduction (bucketed and overlapped with
the last microbatch's backward), the sequence-parallel LayerNorm gradient
reduction, then AdamW (flat, fused; or ZeRO-1 sharded) and the LR schedule.

It is the framework's public training API; ``main.py`` (reference-compatible
CLI) and ``bench.py`` are thin drivers around it.  The pieces it composes are
usable on their own (see the package ``__init__``).

Data: ``tokens``/``labels`` are ``[num_microbatches, B, S]`` int64 tensors (host
or device; host tensors should be pinned and are copied asynchronously).
Every rank passes the same batch for its data-parallel replica; stages that
do not need tokens or labels ignore them.
"""
from __future__ import annotations

import dataclasses
import math
import os

import torch
import torch.distributed as dist

from .config import GPTConfig
from .models.gpt import GPTStage, build_gpt
from .optim import FusedAdamW, make_param_buffer
from .parallel import process_groups as pg
from .parallel.data_parallel import GradSync, allreduce_sequence_parallel_grads
from .parallel.distributed_optimizer import DistributedOptimizer
from .parallel.pipeline_parallel import PipelineEngine


class _nvtx:
    """NVTX range around a phase when enabled (for Nsight timelines); a no-op otherwise."""

    def __init__(self, enabled, name):
        self.enabled, self.name = enabled and torch.cuda.is_available(), name

    def __enter__(self):
        if self.enabled:
            torch.cuda.nvtx.range_push(self.name)
        return self

    def __exit__(self, *exc):
        if self.enabled:
            torch.cuda.nvtx.range_pop()
        return False


def make_lr_lambda(warmup_steps, num_steps):
    """Linear warm-up then cosine decay to 0 over ``num_steps`` total (reference main.py:36-43)."""
    def get_lr(step):
        if step < warmup_steps:
            return step / max(warmup_steps, 1)
        progress = (step - warmup_steps) / max(num_steps - warmup_steps, 1)
        return 0.5 * (1.0 + math.cos(progress * math.pi))
    return get_lr


def compute_mfu(model, seq_len, micro_batch_size, tp, pp, elapsed, num_steps, peak_flops=None):
    """Reference MFU formula (main.py:46-66) with the peak as a parameter (B200 dense bf16 by default)."""
    L, h, V = model["num_layers"], model["hidden_size"], model["vocab_size"]
    B, s = micro_batch_size, seq_len
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    dp_w = max(1, ws // (tp * pp))
    gpu_world = tp * pp * dp_w
    token_linear = (24 * h * h + 48 * h * h) * L + 6 * h * V
    core_attn = 6 * h * L * B
    flops_per_step = token_linear * B * s + core_attn * s * s
    peak = peak_flops if peak_flops is not None else 2.25e15
    return min(flops_per_step * num_steps * dp_w / (elapsed * peak * gpu_world), 1.0)


@dataclasses.dataclass
class TrainConfig:
    model: GPTConfig = dataclasses.field(default_factory=GPTConfig)
    micro_batch_size: int = 4
    seq_len: int | None = None          # default: model.max_seq_len
    num_microbatches: int = 1
    tp: int = 1
    pp: int = 1
    sequence_parallel: bool = False
    zero1: bool = False
    schedule: str = "1f1b"
    lr: float = 6e-4
    weight_decay: float = 0.1
    betas: tuple = (0.9, 0.999)
    eps: float = 1e-8
    warmup_steps: int = 10
    num_steps: int = 100
    dp_overlap: bool = True
    dp_impl: str = "auto"               # "fused" (NVLink kernel), "nccl", or "auto" (fused on CUDA when dp > 1)
    tp_impl: str = "auto"               # "fused" (collectives inside LN/GEMM kernels; implies sequence
                                        # parallelism), "nccl", or "auto" (fused on CUDA when tp > 1)
    bucket_mb: float = 64.0
    recompute: bool = False
    average_microbatches: bool = True   # False = reference PP semantics (sum of microbatch losses)
    seed: int = 42
    nvtx: bool = False                  # NVTX ranges per phase (also MMB_NVTX=1)
    dp_early_buckets: bool = True       # launch DP buckets during backward (MMB_DP_EARLY_BUCKETS=0 turns it off)
    cuda_graph: str = "auto"            # "on", "off", or "auto": replay each whole step as one CUDA graph
                                        # where supported (CUDA, tp = pp = dp = 1, flat fused AdamW)
    error_check_interval: int = 20      # read the native kernels' device error word every N steps (0 = never;
                                        # ``Trainer.check_device_errors`` checks on demand)


class Trainer:
    def __init__(self, cfg: TrainConfig, device=None, mpu=None):
        self.cfg = cfg
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else \
                torch.device("cpu")
        self.device = torch.device(device)
        if not dist.is_initialized():
            raise RuntimeError("torch.distributed must be initialised (world size 1 is fine)")
        seq_len = cfg.seq_len or cfg.model.max_seq_len
        fused_tp = (self.device.type == "cuda" and cfg.tp > 1 and cfg.tp_impl in ("auto", "fused")
                    and seq_len % cfg.tp == 0 and (seq_len // cfg.tp) % 128 == 0)
        if cfg.tp_impl == "fused" and not fused_tp and cfg.tp > 1:
            raise ValueError("fused TP needs CUDA and seq_len / tp divisible by 128")
        self.tp_impl = "fused" if fused_tp else "nccl"
        self.mpu = mpu or pg.init_model_parallel(cfg.tp, cfg.pp, cfg.sequence_parallel or fused_tp)
        pg.set_model_parallel(self.mpu)
        mpu = self.mpu
        self.seq_len = cfg.seq_len or cfg.model.max_seq_len
        if self.seq_len > cfg.model.max_seq_len:
            raise ValueError("seq_len exceeds the position table")
        sp = self.mpu["sequence_parallel"]
        if sp and self.seq_len % cfg.tp:
            raise ValueError("sequence parallelism needs seq_len % tp == 0")
        # identical init on every rank of a TP group and every DP replica (same seed),
        # distinct per pipeline stage only through construction order
        torch.manual_seed(cfg.seed)
        if cfg.pp > 1:
            self.model = GPTStage(cfg.model, mpu["pp_rank"], cfg.pp, recompute=cfg.recompute)
        else:
            self.model = build_gpt(cfg.model, recompute=cfg.recompute)
        self.model.to(self.device)
        dp = mpu["dp_size"]
        bucket_elems = int(cfg.bucket_mb * (1 << 20) / 4)
        grad_scale = 1.0 / dp
        impl = cfg.dp_impl
        if impl == "auto":
            impl = "fused" if (self.device.type == "cuda" and dp > 1) else "nccl"
        self.dp_impl = impl
        self.dp_early = cfg.dp_early_buckets and os.environ.get("MMB_DP_EARLY_BUCKETS", "1") != "0"
        if impl == "fused" and sp:
            # The fused kernel applies AdamW as soon as a bucket's gradients are final across the DP
            # group, but sequence-parallel LayerNorm gradients are only complete after their TP
            # all-reduce at the end of backward: every bucket then starts after that reduction.
            self.dp_early = False
        if impl == "fused":
            from .parallel.fused_dp import FusedDPOptimizer
            early = self.dp_early
            self.optimizer = FusedDPOptimizer(self.model, mpu["dp_group"], lr=cfg.lr, betas=cfg.betas, eps=cfg.eps,
                                              weight_decay=cfg.weight_decay, bucket_elems=bucket_elems,
                                              overlap=cfg.dp_overlap, defer_done=early)
            self.buf = self.optimizer.buf
            self.grad_sync = self.optimizer
        elif cfg.zero1:
            self.buf = make_param_buffer(self.model, align=dp, bucket_elems=bucket_elems)
            self.optimizer = DistributedOptimizer(self.buf, mpu["dp_group"], lr=cfg.lr, betas=cfg.betas,
                                                  eps=cfg.eps, weight_decay=cfg.weight_decay,
                                                  overlap=cfg.dp_overlap)
            self.grad_sync = self.optimizer.grad_sync
        else:
            self.buf = make_param_buffer(self.model, align=dp, bucket_elems=bucket_elems)
            self.optimizer = FusedAdamW(self.model.parameters(), lr=cfg.lr, betas=cfg.betas, eps=cfg.eps,
                                        weight_decay=cfg.weight_decay, grad_scale=grad_scale)
            self.grad_sync = GradSync(self.buf, mpu["dp_group"], mode="allreduce", overlap=cfg.dp_overlap)
        layers = self.model.decoder_layers if cfg.pp > 1 else self.model.decoder.layers
        self.tp_ws = None
        if self.tp_impl == "fused":
            from .parallel.fused_tp import TPWorkspace
            sp_elems = sum(p.numel() for p in self.model.parameters() if getattr(p, "sequence_parallel_grad", False))
            self.tp_ws = TPWorkspace(mpu["tp_group"], cfg.micro_batch_size, self.seq_len, cfg.model.hidden_size,
                                     num_fwd_slots=2 * len(layers) + 1, copy_saved=cfg.pp > 1, vec_elems=sp_elems)
            for i, layer in enumerate(layers):
                layer._mmb_tp_ws = self.tp_ws
                layer._mmb_tp_slot = i
            head = getattr(self.model, "lm_head", None)
            if head is not None:  # the last pipeline stage: ln_f / lm_head / cross-entropy collectives fused too
                head._mmb_tp_ws = self.tp_ws
                head._mmb_tp_slot = 2 * len(layers)
            emb = getattr(self.model, "embedding", None)
            if emb is not None:  # the first pipeline stage: the embedding's TP exchange over NVLink too
                emb._mmb_tp_ws = self.tp_ws
        # Modules whose native backward announces "gradients final".  DP buckets launch strictly in
        # order, head first, so the head and the embedding are attached as well: buckets then start
        # during backward (with MMB_DP_EARLY_BUCKETS=0 every bucket starts after backward).
        ready = [] if (self.dp_impl == "fused" and sp) else list(layers)
        if self.dp_early:
            for name in ("embedding", "ln_f", "lm_head"):
                mod = getattr(self.model, name, None)
                if mod is not None:
                    ready.append(mod)
        self.grad_sync.attach(ready)
        self.scheduler = torch.optim.lr_scheduler.LambdaLR(self.optimizer,
                                                           make_lr_lambda(cfg.warmup_steps, cfg.num_steps))
        self.sp_params = [p for p in self.model.parameters() if getattr(p, "sequence_parallel_grad", False)]
        S_local = self.seq_len // cfg.tp if sp else self.seq_len
        self.engine = None
        if cfg.pp > 1:
            prev, nxt = pg.pp_peers()
            self.engine = PipelineEngine(self.model, mpu["pp_rank"], cfg.pp, prev, nxt,
                                         (cfg.micro_batch_size, S_local, cfg.model.hidden_size), self.device,
                                         schedule=cfg.schedule)
        self.step_count = 0
        self.nvtx = cfg.nvtx or os.environ.get("MMB_NVTX") == "1"
        self.poison_symm = os.environ.get("MMB_POISON_SYMM") == "1"
        self._setup_cuda_graph()
        # a collective on the default group before the first (batched) p2p
        if dist.get_world_size() > 1:
            t = torch.zeros(1, device=self.device)
            dist.all_reduce(t)

    # ------------------------------------------------------------------ step
    def _loss_mask(self):
        return torch.ones(self.cfg.micro_batch_size, self.seq_len, dtype=torch.float32, device=self.device)

    def train_step(self, tokens, labels, loss_mask=None):
        """One optimizer step over ``tokens/labels [m, B, S]``; returns the mean loss tensor (last stage) or None."""
        if self.tp_ws is not None and self.poison_symm:
            self.tp_ws.poison()
        with _nvtx(self.nvtx, "train_step"):
            if self.graph_mode:
                out = self._graph_step(tokens, labels, loss_mask)
            else:
                out = self._train_step(tokens, labels, loss_mask)
        n = self.cfg.error_check_interval
        if n and self.step_count % n == 0:
            self.check_device_errors()
        return out

    def check_device_errors(self):
        """Raise if a native kernel recorded an error since the last check.

        The fused TP/DP kernels bound every wait on a peer or an mbarrier; a
        wait that runs out records an error code in a device word and the
        kernel returns early, leaving that step's results incomplete (for the
        fused DP kernel: parameters stale or partly updated on some ranks).
        Reading the word synchronises the device, so it is read every
        ``error_check_interval`` steps rather than after each one.
        """
        if self.device.type != "cuda":
            return
        from .ops import check_errors
        check_errors()

    # ------------------------------------------------------------------ CUDA graphs
    GRAPH_WARMUP = 1

    def _setup_cuda_graph(self):
        """Decide whether whole steps are replayed from one captured CUDA graph.

        A captured step launches its ~300 kernels with one call and no host
        gaps between them.  Everything step-dependent must then live on the
        device: the optimizer reads lr and its step count from device memory
        (``FusedAdamW.enable_device_schedule``, lr precomputed from the
        schedule), and the batch is copied into static input buffers before
        each replay.  Supported for single-GPU chunks (tp = pp = dp = 1) with
        the flat fused AdamW; other layouts run eagerly.
        """
        cfg = self.cfg
        single = (self.mpu["dp_size"] == 1 and isinstance(self.optimizer, FusedAdamW) and not self.optimizer._loose)
        # the fused-DP step (no NCCL inside) with device-side epochs; gated with the early-bucket mode
        fused_dp = (self.dp_impl == "fused" and self.mpu["dp_size"] > 1 and not self.mpu["sequence_parallel"]
                    and self.dp_early)
        supported = self.device.type == "cuda" and cfg.tp == 1 and cfg.pp == 1 and (single or fused_dp)
        if cfg.cuda_graph == "on" and not supported:
            raise ValueError("cuda_graph='on' needs CUDA, tp = pp = 1 and either dp = 1 with the flat fused AdamW "
                             "or the fused-DP optimizer in early-bucket mode")
        self.graph_mode = supported and cfg.cuda_graph in ("on", "auto") and os.environ.get("MMB_CUDA_GRAPH") != "0"
        self._graph = None
        self._graph_calls = 0
        if self.graph_mode:
            lam = self.scheduler.lr_lambdas[0]
            base = self.scheduler.base_lrs[0]
            n = 2 * cfg.num_steps + 1024
            table = torch.tensor([base * lam(i) for i in range(n)], dtype=torch.float32)
            self.optimizer.enable_device_schedule(table)

    def eager(self):
        """Context manager: run the enclosed steps eagerly even in graph mode (e.g. under a profiler)."""
        trainer = self

        class _Eager:
            def __enter__(self):
                self.prev = trainer.graph_mode
                trainer.graph_mode = False

            def __exit__(self, *exc):
                trainer.graph_mode = self.prev
                return False
        return _Eager()

    def _graph_step(self, tokens, labels, loss_mask):
        if tokens.dim() == 2:
            tokens, labels = tokens.unsqueeze(0), labels.unsqueeze(0)
        if self._graph is None and self._graph_calls < self.GRAPH_WARMUP:
            # eager warm-up on a side stream (allocator and lazy initialisation settle before capture)
            self._graph_calls += 1
            side = torch.cuda.Stream(device=self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                out = self._train_step(tokens, labels, loss_mask)
            torch.cuda.current_stream(self.device).wait_stream(side)
            return out
        first = self._graph is None
        if first:
            self._static_tokens = torch.empty(tokens.shape, dtype=tokens.dtype, device=self.device)
            self._static_labels = torch.empty(labels.shape, dtype=labels.dtype, device=self.device)
            self._static_mask = (self._loss_mask() if loss_mask is None else
                                 torch.empty(loss_mask.shape, dtype=torch.float32, device=self.device))
        if tokens.shape != self._static_tokens.shape:
            raise ValueError("a captured step needs the same batch shape every step")
        self._static_tokens.copy_(tokens, non_blocking=True)
        self._static_labels.copy_(labels, non_blocking=True)
        if loss_mask is not None:
            self._static_mask.copy_(loss_mask, non_blocking=True)
        if first:
            torch.cuda.synchronize(self.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                self._static_loss = self._train_step(self._static_tokens, self._static_labels, self._static_mask)
            self._graph = g
            # capturing ran this step's host-side bookkeeping (scheduler, step counters) once; now run its kernels
        else:
            self.optimizer.advance_host_counters()
            self.scheduler.step()
            self.step_count += 1
        self._graph.replay()
        return None if self._static_loss is None else self._static_loss.clone()

    def _train_step(self, tokens, labels, loss_mask):
        cfg = self.cfg
        m = cfg.num_microbatches
        if tokens.dim() == 2:
            tokens, labels = tokens.unsqueeze(0), labels.unsqueeze(0)
        tokens = tokens.to(self.device, non_blocking=True)
        labels = labels.to(self.device, non_blocking=True)
        mask = self._loss_mask() if loss_mask is None else loss_mask.to(self.device, non_blocking=True)
        scale = 1.0 / m if cfg.average_microbatches else 1.0
        self.optimizer.zero_grad()
        self.grad_sync.reset()
        if self.engine is None:
            total = None
            for mb in range(m):
                if mb == m - 1:
                    self.grad_sync.overlap = cfg.dp_overlap
                else:
                    self.grad_sync.overlap = False
                with _nvtx(self.nvtx, f"forward mb{mb}"):
                    _, loss = self.model(tokens[mb], labels[mb], mask if mask.dim() == 2 else mask[mb])
                with _nvtx(self.nvtx, f"backward mb{mb}"):
                    (loss * scale).backward()
                total = loss.detach() if total is None else total + loss.detach()
            result = total / m
        else:
            def batch_fn(mb):
                return tokens[mb], labels[mb], (mask if mask.dim() == 2 else mask[mb])

            def pre_backward(mb):
                # only the last microbatch's backward may launch DP buckets
                self.grad_sync.overlap = cfg.dp_overlap if mb == m - 1 else False

            with _nvtx(self.nvtx, "pipeline 1f1b"):
                losses = self.engine.run(batch_fn, m, loss_scale=scale, pre_backward=pre_backward)
            result = torch.stack([l.detach() for l in losses]).mean() if losses else None
        self.grad_sync.overlap = cfg.dp_overlap
        with _nvtx(self.nvtx, "grad sync + optimizer"):
            if not cfg.zero1 and self.dp_impl != "fused":
                self.grad_sync.finish()
            if self.sp_params:
                if self.tp_ws is not None:   # fused TP: summed over NVLink
                    self.tp_ws.vec_allreduce([grad_of(p) for p in self.sp_params])
                else:
                    allreduce_sequence_parallel_grads(self.sp_params, self.mpu["tp_group"])
            self.optimizer.step()
            self.scheduler.step()
        self.step_count += 1
        return result

    # ------------------------------------------------------------------ utils
    def state_for_checkpoint(self):
        return self.model, self.optimizer, self.scheduler

    def destroy(self):
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
            self.check_device_errors()
        self._graph = None
        if self.tp_ws is not None:
            self.tp_ws.close()
            self.tp_ws = None
        if hasattr(self.optimizer, "close"):
            self.optimizer.close()
        pg.set_model_parallel(None)


def grad_of(p):
    """The gradient a native kernel accumulated for ``p`` (main_grad when managed, else .grad)."""
    g = getattr(p, "main_grad", None)
    return g if g is not None else p.grad


def synthetic_batch(num_microbatches, B, S, vocab, seed=0, pin=False, shift=True):
    """Uniform-random tokens with next-token-shift labels (last label = -100)."""
    g = torch.Generator().manual_seed(seed)
    toks = torch.randint(0, vocab, (num_microbatches, B, S + (1 if shift else 0)), generator=g)
    if shift:
        tokens, labels = toks[..., :-1].contiguous(), toks[..., 1:].contiguous()
    else:
        tokens, labels = toks, toks.clone()
    if pin and torch.cuda.is_available():
        tokens, labels = tokens.pin_memory(), labels.pin_memory()
    return tokens, labels
