"""mini_megatron_b200: a Megatron-style GPT training framework built for NVIDIA B200 (sm_100a).

Layers (bottom-up):
  csrc/        sm_100a CUDA kernels (tcgen05/TMEM/TMA GEMM with fused epilogues,
               LayerNorm, vocab-parallel cross-entropy, embedding, flat AdamW, ...)
  ops/         Python access to the kernels (fails loudly if the extension is missing)
  comm/        autograd collectives (TP f/g, sequence parallel), P2P, overlap helpers
  parallel/    (dp, pp, tp) topology, TP layers, 1F1B pipeline, DP sync, ZeRO-1, flat buffers
  models/      GPT (embedding, decoder, vocab-parallel loss) + native fused layer functions
  training.py  Trainer: one optimizer step across all of the above
  utils/       checkpointing, kernel micro-benchmarks
"""
__version__ = "0.1.0"
