"""Model contracts between this framework, the reference and Megatron-Core.

The shared logical model: bias-free GPT with learned absolute positions,
pre-LN (LayerNorm with bias), exact-erf GELU, no dropout, untied lm_head,
causal next-token cross-entropy.

* **Names.** This framework keeps the reference's state_dict names
  (``embedding.token_embedding.weight``, ``decoder.layers.{i}.attn.qkv.weight``,
  ...; pipeline stages use ``decoder_layers.{local_i}``).  ``mcore_name_pairs``
  maps them to Megatron-Core's ``GPTModel`` names.
* **QKV layout.** Here (and in the reference) the fused QKV weight's rows are
  ``[all Q | all K | all V]``; Megatron-Core interleaves per head
  ``[Q_h K_h V_h]``.  ``qkv_to_mcore`` / ``qkv_from_mcore`` convert.
* **Vocabulary padding.** Embedding / lm_head rows are padded here to a
  multiple of 128 * tp; ``to_reference_state`` drops the padding and
  ``from_reference_state`` adds zero rows.
* **TP shards.** ``tp_shard`` cuts an unsharded tensor into this framework's
  (= the reference's) shard: stride-3 rows for QKV (every rank gets a
  matching set of Q, K and V heads), contiguous rows for the other
  Column-parallel weights and the vocabulary tables, contiguous columns for
  Row-parallel weights.  ``mcore_tp_shard`` gives Megatron-Core's shard
  (per-head interleave, then contiguous rows).
* **Pipeline stages.** ``stage_parameter_plan`` lists, for one stage, the
  (full name, stage-local name) pairs.

Reference: experiments/fair_tp1_contract.py:44-103, experiments/fair_tp_parallel_contract.py:14-47,
experiments/create_fair_pp_artifacts.py:60-77 (stage names).
"""
from __future__ import annotations

import hashlib

import torch

CONTRACT = ("bias-free GPT, learned absolute positions, pre-LN with LayerNorm bias, exact-erf GELU, no dropout, "
            "untied lm_head, causal next-token cross entropy")

_LAYER_KEYS = ("ln1.weight", "ln1.bias", "attn.qkv.weight", "attn.o.weight", "ln2.weight", "ln2.bias",
               "mlp.fc1.weight", "mlp.fc2.weight")
_MCORE_LAYER_KEYS = ("input_layernorm.weight", "input_layernorm.bias", "self_attention.linear_qkv.weight",
                     "self_attention.linear_proj.weight", "pre_mlp_layernorm.weight", "pre_mlp_layernorm.bias",
                     "mlp.linear_fc1.weight", "mlp.linear_fc2.weight")


def _cfg(model_config, key):
    if isinstance(model_config, dict):
        return model_config[key]
    return getattr(model_config, key)


def full_parameter_names(model_config) -> list:
    L = _cfg(model_config, "num_layers")
    names = ["embedding.token_embedding.weight", "embedding.position_embedding.weight"]
    for i in range(L):
        names += [f"decoder.layers.{i}.{k}" for k in _LAYER_KEYS]
    return names + ["ln_f.weight", "ln_f.bias", "lm_head.weight"]


def mcore_name_pairs(model_config) -> list:
    """[(name here / in the reference, Megatron-Core GPTModel name)]."""
    pairs = [("embedding.token_embedding.weight", "embedding.word_embeddings.weight"),
             ("embedding.position_embedding.weight", "embedding.position_embeddings.weight"),
             ("ln_f.weight", "decoder.final_layernorm.weight"),
             ("ln_f.bias", "decoder.final_layernorm.bias"),
             ("lm_head.weight", "output_layer.weight")]
    for i in range(_cfg(model_config, "num_layers")):
        pairs += [(f"decoder.layers.{i}.{a}", f"decoder.layers.{i}.{b}") for a, b in zip(_LAYER_KEYS,
                                                                                           _MCORE_LAYER_KEYS)]
    return pairs


def is_qkv(name: str) -> bool:
    return name.endswith("attn.qkv.weight") or name.endswith("self_attention.linear_qkv.weight")


def qkv_to_mcore(w: torch.Tensor, num_heads: int) -> torch.Tensor:
    """Rows ``[all Q | all K | all V]`` -> Megatron-Core's per-head ``[Q_h K_h V_h]``."""
    if w.dim() != 2 or w.size(0) % (3 * num_heads):
        raise ValueError("QKV weight must be 2-D with 3 * heads * head_dim rows")
    d = w.size(0) // (3 * num_heads)
    return w.reshape(3, num_heads, d, w.size(1)).transpose(0, 1).reshape(w.shape).contiguous()


def qkv_from_mcore(w: torch.Tensor, num_heads: int) -> torch.Tensor:
    """Inverse of :func:`qkv_to_mcore`."""
    if w.dim() != 2 or w.size(0) % (3 * num_heads):
        raise ValueError("QKV weight must be 2-D with 3 * heads * head_dim rows")
    d = w.size(0) // (3 * num_heads)
    return w.reshape(num_heads, 3, d, w.size(1)).transpose(0, 1).reshape(w.shape).contiguous()


def to_mcore_state(state: dict, model_config) -> dict:
    heads = _cfg(model_config, "num_attention_heads")
    out = {}
    for ours, mc in mcore_name_pairs(model_config):
        t = state[ours]
        out[mc] = qkv_to_mcore(t, heads) if is_qkv(ours) else t
    return out


def from_mcore_state(state: dict, model_config) -> dict:
    heads = _cfg(model_config, "num_attention_heads")
    out = {}
    for ours, mc in mcore_name_pairs(model_config):
        t = state[mc]
        out[ours] = qkv_from_mcore(t, heads) if is_qkv(ours) else t
    return out


# ----------------------------------------------------------------------------- vocabulary padding
_VOCAB_TABLES = ("embedding.token_embedding.weight", "lm_head.weight")


def to_reference_state(state: dict, vocab_size: int) -> dict:
    """Drop the vocabulary padding rows so the tables have exactly ``vocab_size`` rows."""
    out = dict(state)
    for k in _VOCAB_TABLES:
        if k in out and out[k].size(0) > vocab_size:
            out[k] = out[k][:vocab_size].contiguous()
    return out


def from_reference_state(state: dict, padded_vocab: int) -> dict:
    """Add zero padding rows to the vocabulary tables (padded rows start at zero here)."""
    out = dict(state)
    for k in _VOCAB_TABLES:
        if k in out and out[k].size(0) < padded_vocab:
            t = out[k]
            out[k] = torch.cat([t, t.new_zeros(padded_vocab - t.size(0), *t.shape[1:])])
    return out


# ----------------------------------------------------------------------------- TP shards
def is_column_parallel(name: str) -> bool:
    return (name.endswith("token_embedding.weight") or name.endswith("attn.qkv.weight")
            or name.endswith("mlp.fc1.weight") or name.endswith("lm_head.weight"))


def is_row_parallel(name: str) -> bool:
    return name.endswith("attn.o.weight") or name.endswith("mlp.fc2.weight")


def _strided_rows(t, tp, rank, stride):
    if t.size(0) % (tp * stride):
        raise ValueError("rows must divide evenly by tp * stride")
    chunk = t.size(0) // (tp * stride)
    return torch.cat([t.narrow(0, (s * tp + rank) * chunk, chunk) for s in range(stride)]).contiguous()


def tp_shard(full: torch.Tensor, name: str, tp: int, rank: int) -> torch.Tensor:
    """This framework's (and the reference's) TP shard of an unsharded tensor."""
    if tp == 1:
        return full
    if name.endswith("attn.qkv.weight"):
        return _strided_rows(full, tp, rank, 3)
    if is_column_parallel(name):
        return _strided_rows(full, tp, rank, 1)
    if is_row_parallel(name):
        w = full.size(1) // tp
        return full.narrow(1, rank * w, w).contiguous()
    return full


def tp_unshard(shards: list, name: str) -> torch.Tensor:
    """Inverse of :func:`tp_shard` given every rank's shard in rank order."""
    tp = len(shards)
    if tp == 1:
        return shards[0]
    if name.endswith("attn.qkv.weight"):
        c = shards[0].size(0) // 3
        return torch.cat([sh.narrow(0, s * c, c) for s in range(3) for sh in shards])
    if is_column_parallel(name):
        return torch.cat(shards, 0)
    if is_row_parallel(name):
        return torch.cat(shards, 1)
    return shards[0]


def mcore_tp_shard(full_ours: torch.Tensor, name: str, num_heads: int, tp: int, rank: int) -> torch.Tensor:
    """Megatron-Core's TP shard of an unsharded tensor given in this framework's layout."""
    if is_qkv(name):
        mc = qkv_to_mcore(full_ours, num_heads)
        rows = mc.size(0) // tp
        return mc.narrow(0, rank * rows, rows).contiguous()
    return tp_shard(full_ours, name, tp, rank)


# ----------------------------------------------------------------------------- pipeline stages
def stage_layer_range(num_layers: int, pp_rank: int, pp: int):
    """Layers of one stage: ``num_layers // pp`` each, the last stage takes the remainder."""
    per = num_layers // pp
    start = pp_rank * per
    return start, (start + per if pp_rank < pp - 1 else num_layers)


def stage_parameter_plan(model_config, pp_rank: int, pp: int) -> list:
    """[(full name, stage-local name)] for the parameters stage ``pp_rank`` owns."""
    L = _cfg(model_config, "num_layers")
    start, end = stage_layer_range(L, pp_rank, pp)
    plan = []
    if pp_rank == 0:
        plan += [(n, n) for n in ("embedding.token_embedding.weight", "embedding.position_embedding.weight")]
    for i in range(start, end):
        plan += [(f"decoder.layers.{i}.{k}", f"decoder_layers.{i - start}.{k}") for k in _LAYER_KEYS]
    if pp_rank == pp - 1:
        plan += [(n, n) for n in ("ln_f.weight", "ln_f.bias", "lm_head.weight")]
    return plan


def shard_state(full_state: dict, model_config, tp: int, tp_rank: int, pp: int = 1, pp_rank: int = 0) -> dict:
    """The state_dict of one (tp_rank, pp_rank) model chunk, cut from an unsharded state_dict."""
    if pp == 1:
        return {n: tp_shard(full_state[n], n, tp, tp_rank) for n in full_parameter_names(model_config)}
    return {local: tp_shard(full_state[n], n, tp, tp_rank) for n, local in
            stage_parameter_plan(model_config, pp_rank, pp)}


def tensor_digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()
