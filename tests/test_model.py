"""CPU unit tests of the model components (reference tests/test_model.py in spirit)."""
import torch

from mini_megatron_b200.models import GPT, MLP, Attention, CrossEntropyLoss, Decoder, DecoderLayer, Embedding
from mini_megatron_b200.parallel.tensor_parallel import ColumnParallelLinear


def test_embedding_forward_shape():
    embed = Embedding(vocab_size=100, hidden_size=16, max_seq_len=8)
    assert embed(torch.randint(0, 100, (2, 8))).shape == (2, 8, 16)


def test_embedding_position_dependency():
    embed = Embedding(vocab_size=10, hidden_size=4, max_seq_len=4)
    out = embed(torch.tensor([[0, 0, 0, 0]]))
    assert not torch.allclose(out[0, 0], out[0, 1])


def test_attention_mlp_layer_shapes():
    torch.manual_seed(0)
    x = torch.randn(2, 8, 16)
    assert Attention(16, 4)(x).shape == (2, 8, 16)
    assert MLP(16, 64)(x).shape == (2, 8, 16)
    assert DecoderLayer(16, 4, 64)(x).shape == (2, 8, 16)
    dec = Decoder(16, 4, 64, num_layers=6)
    assert len(dec.layers) == 6 and dec(x).shape == (2, 8, 16)


def test_attention_is_causal():
    torch.manual_seed(0)
    attn = Attention(16, 4)
    x = torch.randn(1, 8, 16)
    y = attn(x)
    x2 = x.clone()
    x2[0, 5:] += 10.0
    y2 = attn(x2)
    torch.testing.assert_close(y[0, :5], y2[0, :5])
    assert not torch.allclose(y[0, 5:], y2[0, 5:])


def test_gpt_forward_with_and_without_loss():
    torch.manual_seed(0)
    HS, NH, FFN, NL, V = 16, 4, 64, 2, 32
    model = GPT(Embedding(V, HS, 8), Decoder(HS, NH, FFN, NL), torch.nn.LayerNorm(HS),
                ColumnParallelLinear(HS, V, bias=False, gather_output=True), CrossEntropyLoss())
    x = torch.randint(0, V, (2, 8))
    assert model(x).shape == (2, 8, V)
    logits, loss = model(x, labels=x, loss_mask=torch.ones(2, 8))
    assert logits.shape == (2, 8, V) and loss.ndim == 0 and loss.item() > 0


def test_cross_entropy_uniform_and_perfect():
    loss_fn = CrossEntropyLoss()
    V = 100
    loss = loss_fn(torch.zeros(8, V), torch.randint(0, V, (8,)), torch.ones(8))
    assert abs(loss.item() - torch.log(torch.tensor(float(V))).item()) < 0.01
    logits = torch.full((1, 5), -10.0)
    logits[0, 2] = 10.0
    assert loss_fn(logits, torch.tensor([2]), torch.ones(1)).item() < 0.01


def test_cross_entropy_padded_vocab_matches_unpadded():
    torch.manual_seed(0)
    V, Vp = 50, 64
    logits = torch.randn(10, Vp, requires_grad=True)
    labels = torch.randint(0, V, (10,))
    mask = torch.ones(10)
    loss = CrossEntropyLoss(vocab_size=V)(logits, labels, mask)
    ref_logits = logits.detach()[:, :V].clone().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(ref_logits, labels)
    torch.testing.assert_close(loss, ref)
    loss.backward()
    ref.backward()
    torch.testing.assert_close(logits.grad[:, :V], ref_logits.grad)
    assert logits.grad[:, V:].abs().max() == 0


def test_cross_entropy_ignore_index_stays_in_denominator():
    torch.manual_seed(0)
    logits = torch.randn(4, 10)
    labels = torch.tensor([1, -100, 3, 4])
    loss = CrossEntropyLoss(vocab_size=10)(logits, labels, torch.ones(4))
    per = torch.nn.functional.cross_entropy(logits, labels, reduction="none")
    torch.testing.assert_close(loss, per.sum() / 4)


def test_build_gpt_state_dict_names_match_reference_layout():
    from mini_megatron_b200.config import PRESETS
    from mini_megatron_b200.models import build_gpt
    names = set(build_gpt(PRESETS["tiny"]).state_dict())
    for n in ("embedding.token_embedding.weight", "embedding.position_embedding.weight",
              "decoder.layers.0.ln1.weight", "decoder.layers.0.ln1.bias", "decoder.layers.0.attn.qkv.weight",
              "decoder.layers.0.attn.o.weight", "decoder.layers.0.ln2.weight", "decoder.layers.0.ln2.bias",
              "decoder.layers.0.mlp.fc1.weight", "decoder.layers.0.mlp.fc2.weight", "ln_f.weight", "ln_f.bias",
              "lm_head.weight"):
        assert n in names, n


def test_stage_names_match_reference_pp_layout():
    from mini_megatron_b200.config import PRESETS
    from mini_megatron_b200.models import GPTStage
    first = set(GPTStage(PRESETS["tiny"], 0, 2).state_dict())
    last = set(GPTStage(PRESETS["tiny"], 1, 2).state_dict())
    assert "embedding.token_embedding.weight" in first and "decoder_layers.0.attn.qkv.weight" in first
    assert "lm_head.weight" in last and "ln_f.weight" in last and "embedding.token_embedding.weight" not in last
