"""Prompt encoders from a diffusers-layout directory (tiny random transformers models and a
word-level tokenizer written here): shapes, padding semantics, layer / template handling."""

import dataclasses

import pytest
import torch

pytest.importorskip("transformers")
pytest.importorskip("tokenizers")

from difflet_b200.models import text_encoders as TE  # noqa: E402

WORDS = ["a", "cat", "dog", "on", "the", "mat", "runs", "red", "blue", "sky", "system", "user", "describe"]


def _tokenizer(path, eos="</s>"):
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    vocab = {"<pad>": 0, "<unk>": 1, eos: 2}
    for w in WORDS:
        vocab[w] = len(vocab)
    tk = Tokenizer(models.WordLevel(vocab=vocab, unk_token="<unk>"))
    tk.pre_tokenizer = pre_tokenizers.Whitespace()
    PreTrainedTokenizerFast(tokenizer_object=tk, pad_token="<pad>", unk_token="<unk>", eos_token=eos).save_pretrained(
        str(path))


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    import transformers as T

    root = tmp_path_factory.mktemp("ckpt")
    torch.manual_seed(0)
    _tokenizer(root / "tokenizer")
    _tokenizer(root / "tokenizer_2")
    T.CLIPTextModel(T.CLIPTextConfig(vocab_size=32, hidden_size=32, intermediate_size=64, num_hidden_layers=2,
                                     num_attention_heads=2, max_position_embeddings=77, eos_token_id=2,
                                     pad_token_id=0)).save_pretrained(root / "text_encoder")
    T.T5EncoderModel(T.T5Config(vocab_size=32, d_model=32, d_kv=8, d_ff=64, num_layers=2, num_heads=4,
                                pad_token_id=0)).save_pretrained(root / "text_encoder_2")
    umt5 = root / "umt5"
    _tokenizer(umt5 / "tokenizer")
    T.UMT5EncoderModel(T.UMT5Config(vocab_size=32, d_model=32, d_kv=8, d_ff=64, num_layers=2, num_heads=4,
                                    pad_token_id=0)).save_pretrained(umt5 / "text_encoder")
    lm = root / "lm"
    _tokenizer(lm / "tokenizer")
    T.LlamaModel(T.LlamaConfig(vocab_size=32, hidden_size=32, intermediate_size=64, num_hidden_layers=3,
                               num_attention_heads=4, num_key_value_heads=2, pad_token_id=0)).save_pretrained(
        lm / "text_encoder")
    return root


def test_flux_clip_t5(ckpt):
    enc = TE.load_text_encoder("flux", ckpt, "cpu", torch.float32, max_sequence_length=16)
    emb, pooled = enc(["a red cat", "the dog runs on the mat"])
    assert emb.shape == (2, 16, 32) and pooled.shape == (2, 32)
    assert torch.isfinite(emb).all() and torch.isfinite(pooled).all()
    e1, p1 = enc(["a red cat"])
    torch.testing.assert_close(e1[0], emb[0], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(p1[0], pooled[0], atol=1e-5, rtol=1e-5)


def test_umt5_trimmed_run_equals_full_padded_run(ckpt):
    enc = TE.load_text_encoder("wan", ckpt / "umt5", "cpu", torch.float32, text_len=12)
    prompts = ["a cat", "the red dog runs on the mat"]
    emb, pooled = enc(prompts)
    assert pooled is None and emb.shape == (2, 12, 32)
    t = enc.tok(prompts, padding="max_length", max_length=12, truncation=True, return_tensors="pt")
    n = t.attention_mask.sum(-1)
    full = enc.model(t.input_ids, t.attention_mask).last_hidden_state
    for i in range(2):
        torch.testing.assert_close(emb[i, : n[i]], full[i, : n[i]], atol=1e-5, rtol=1e-5)
        assert emb[i, n[i]:].abs().max() == 0


def test_decoder_lm_template_drop_and_layer(ckpt):
    spec = dataclasses.replace(TE.QWEN_IMAGE_TEMPLATE, template="system describe {} user", drop_tokens=2,
                               max_len=8, skip_layers=1)
    enc = TE.DecoderLMTextEncoder(ckpt / "lm", "cpu", torch.float32, spec=spec)
    emb, pooled = enc(["a blue sky", "cat"])
    assert pooled is None and emb.shape == (2, 8, 32)
    t = enc.tok(["system describe a blue sky user"], padding="max_length", max_length=10, return_tensors="pt")
    hs = enc.lm(input_ids=t.input_ids, attention_mask=t.attention_mask, output_hidden_states=True).hidden_states
    ref = hs[-2][0, 2:]
    valid = int(t.attention_mask.sum()) - 2
    torch.testing.assert_close(emb[0, :valid], ref[:valid], atol=1e-5, rtol=1e-5)
    assert emb[0, valid:].abs().max() == 0


def test_missing_folders_return_none(tmp_path):
    assert TE.load_text_encoder("flux", tmp_path, "cpu") is None
    assert TE.load_text_encoder("wan", None, "cpu") is None
    with pytest.raises(ValueError):
        TE.load_text_encoder("nope", tmp_path, "cpu")


def _tiny_qwen3vl_checkpoint(root):
    """A random tiny Qwen3-VL checkpoint folder (text_encoder/ + tokenizer/) built offline."""
    import json
    import os

    from safetensors.torch import save_file
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextModel

    words = ["[PAD]", "[EOS]"] + [f"w{i}" for i in range(60)]
    tk = Tokenizer(models.WordLevel({w: i for i, w in enumerate(words)}, unk_token="[PAD]"))
    tk.pre_tokenizer = pre_tokenizers.Whitespace()
    fast = PreTrainedTokenizerFast(tokenizer_object=tk, pad_token="[PAD]", eos_token="[EOS]")
    fast.save_pretrained(os.path.join(root, "tokenizer"))
    conf = Qwen3VLConfig(text_config=dict(vocab_size=64, hidden_size=64, intermediate_size=128, num_hidden_layers=6,
                                          num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                                          rope_theta=5e6, max_position_embeddings=256, pad_token_id=0))
    enc = os.path.join(root, "text_encoder")
    os.makedirs(enc, exist_ok=True)
    conf.save_pretrained(enc)
    torch.manual_seed(0)
    full = Qwen3VLTextModel(conf.text_config).eval()
    save_file({"model.language_model." + k: v.contiguous() for k, v in full.state_dict().items()
               if not k.endswith("inv_freq")}, os.path.join(enc, "model.safetensors"))
    return full, fast


def test_layer_state_encoder_reads_the_inner_hidden_state(tmp_path):
    """Loading only the first `layer` layers and hooking the last one equals the full model's
    hidden_states[layer] (pre-norm), with the padding rows zeroed and the valid counts reported."""
    from difflet_b200.models.text_encoders import LayerStateEncoder

    full, tok = _tiny_qwen3vl_checkpoint(str(tmp_path))
    enc = LayerStateEncoder(tmp_path, "cpu", torch.float32, layer=4, seq_len=12)
    emb, pooled = enc(["w1 w2 w3", "w5 w6 w7 w8 w9"])
    assert pooled is None and emb.shape == (2, 12, 64) and enc.last_valid.tolist() == [3, 5]
    t = tok(["w1 w2 w3", "w5 w6 w7 w8 w9"], add_special_tokens=False, padding="max_length", max_length=12,
            return_tensors="pt")
    with torch.no_grad():
        hs = full(input_ids=t.input_ids, attention_mask=t.attention_mask, output_hidden_states=True).hidden_states
    ref = hs[4] * t.attention_mask[..., None]
    assert torch.allclose(emb, ref, atol=1e-5, rtol=1e-4)
    assert emb[0, 3:].abs().sum() == 0
