"""External baseline arms.

* **The reference mini-megatron** (``baseline/_ref``, its unmodified
  sources): ``bench.py --impl reference``, ``harness.parity --impl-a
  reference`` and ``harness.fair_bench --implementation reference`` drive its
  own modules and training-loop functions.
* **Megatron-Core** (``megatron.core``), when installed: ``build_mcore_gpt``
  builds the matching ``GPTModel`` (local layer spec, learned absolute
  positions, no bias, LayerNorm, exact GELU, no dropout, untied output
  layer) and ``mcore_train_step`` runs one optimizer step with it, so the
  same harness (artifacts in the Megatron-Core layout from
  ``harness.contract.to_mcore_state``, parity, fair_bench-style timing) can
  compare against it.  This image ships no Megatron-Core, so
  ``mcore_available()`` is False here and the builders raise a clear error.

Reference: eval/run_megatron_baseline.py:20-219 (matching custom loop around
MCore's GPTModel).
"""
from __future__ import annotations

import importlib.util
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]


def reference_available() -> bool:
    return (REPO / "baseline" / "_ref" / "model" / "transformer.py").exists()


def mcore_available() -> bool:
    try:
        return importlib.util.find_spec("megatron.core") is not None
    except ModuleNotFoundError:
        return False


def build_mcore_gpt(model_config: dict, tp: int = 1, pp: int = 1, bf16: bool = True):
    """Megatron-Core GPTModel matching the shared contract (requires megatron.core and its parallel state)."""
    if not mcore_available():
        raise RuntimeError("Megatron-Core (megatron.core) is not installed in this environment")
    import torch
    from megatron.core.models.gpt import GPTModel
    from megatron.core.models.gpt.gpt_layer_specs import get_gpt_layer_local_spec
    from megatron.core.transformer.transformer_config import TransformerConfig
    cfg = TransformerConfig(
        num_layers=model_config["num_layers"], hidden_size=model_config["hidden_size"],
        num_attention_heads=model_config["num_attention_heads"], ffn_hidden_size=model_config["ffn_hidden_size"],
        tensor_model_parallel_size=tp, pipeline_model_parallel_size=pp, hidden_dropout=0.0, attention_dropout=0.0,
        add_bias_linear=False, gated_linear_unit=False, normalization="LayerNorm",
        activation_func=torch.nn.functional.gelu, bf16=bf16, params_dtype=torch.float32,
        init_method_std=0.02, apply_residual_connection_post_layernorm=False)
    return GPTModel(config=cfg, transformer_layer_spec=get_gpt_layer_local_spec(), vocab_size=model_config["vocab_size"],
                    max_sequence_length=model_config["max_seq_len"], position_embedding_type="learned_absolute",
                    share_embeddings_and_output_weights=False, parallel_output=False)


def mcore_train_step(model, optimizer, tokens, labels):
    """One step of the matching custom loop: causal forward, next-token CE, backward, AdamW."""
    import torch
    B, S = tokens.shape
    pos = torch.arange(S, device=tokens.device).unsqueeze(0).expand(B, -1)
    mask = torch.triu(torch.ones(S, S, dtype=torch.bool, device=tokens.device), diagonal=1)[None, None]
    optimizer.zero_grad(set_to_none=True)
    logits = model(tokens, position_ids=pos, attention_mask=mask)
    loss = torch.nn.functional.cross_entropy(logits.reshape(-1, logits.size(-1)).float(), labels.reshape(-1),
                                             ignore_index=-100)
    loss.backward()
    optimizer.step()
    return loss.detach()
