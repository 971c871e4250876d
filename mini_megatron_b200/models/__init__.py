"""GPT model family (embedding, decoder, vocab-parallel loss, builders)."""
from .embedding import Embedding  # noqa: F401
from .gpt import GPTStage, build_gpt, padded_vocab, stage_layer_range  # noqa: F401
from .loss import CrossEntropyLoss, vocab_parallel_cross_entropy  # noqa: F401
from .transformer import GPT, MLP, Attention, Decoder, DecoderLayer  # noqa: F401
