"""Prompt encoders loaded from a diffusers checkpoint directory with ``transformers``.

Text encoding runs once per request, off the denoising hot path, so it uses the released
encoder implementations (the reference does the same: UMT5 on the device for Wan,
difflet/backends/cuda/wan/application.py:52-89; CLIP-L + T5-XXL inside diffusers'
``FluxPipeline`` for FLUX, difflet/backends/cuda/flux/application.py).  Every encoder has the
call signature of the synthetic stand-in (``SyntheticTextEncoder``): ``enc(prompts) ->
(sequence embeddings [B, L, D], pooled [B, P] or None)``.

* ``FluxTextEncoders``: CLIP-L (``text_encoder`` / ``tokenizer``, 77 tokens, pooled output)
  and T5 (``text_encoder_2`` / ``tokenizer_2``, ``max_sequence_length`` tokens padded to that
  length, last hidden state).
* ``UMT5TextEncoder``: Wan's UMT5 (``text_encoder`` / ``tokenizer``), padded to ``text_len``;
  the model runs on the longest prompt's valid prefix only (its attention is masked, so real
  tokens never see padding) and positions past each prompt's own length are zero.
* ``DecoderLMTextEncoder``: a decoder-only LM used as a text encoder (Qwen-Image's
  Qwen2.5-VL, HunyuanVideo's Llama): the prompt is wrapped in the model's template, the
  hidden state of layer ``-1 - skip_layers`` is taken, the template's first ``drop_tokens``
  positions are removed and the rest is padded / cut to ``max_len``; optional CLIP pooled
  vector (HunyuanVideo).

* ``LayerStateEncoder``: a decoder LM read at one inner hidden state (MiniMax-H3: Qwen3-VL-32B's
  language model, ``hidden_states[50]`` = the raw output of decoder layer 49, before any later
  layer and without the final norm).  Only the layers up to that one are built and loaded; the
  prompt is tokenised without special tokens, right-padded (causal attention: valid rows never
  see the padding) and the padding rows are zeroed; the valid token count comes back as
  ``last_valid``.

``load_text_encoder(family, model_path, ...)`` returns the family's encoder, or None when the
checkpoint has no encoder folders (the caller keeps the synthetic stand-in).
"""

from __future__ import annotations

import dataclasses
import os
from dataclasses import dataclass

import torch


def _has(model_path, *subs) -> bool:
    return model_path is not None and all(os.path.isdir(os.path.join(str(model_path), s)) for s in subs)


def _tokenizer(path):
    from transformers import AutoTokenizer

    return AutoTokenizer.from_pretrained(path)


def _model(cls_name: str, path, device, dtype):
    import transformers

    cls = getattr(transformers, cls_name)
    m = cls.from_pretrained(path, dtype=dtype)
    m = m.to(device).eval()
    m.requires_grad_(False)
    return m


class FluxTextEncoders:
    def __init__(self, model_path, device, dtype=torch.bfloat16, max_sequence_length: int = 512,
                 clip_len: int = 77):
        root = str(model_path)
        self.device, self.dtype = torch.device(device), dtype
        self.t5_len, self.clip_len = int(max_sequence_length), int(clip_len)
        self.clip_tok = _tokenizer(os.path.join(root, "tokenizer"))
        self.clip = _model("CLIPTextModel", os.path.join(root, "text_encoder"), self.device, dtype)
        self.t5_tok = _tokenizer(os.path.join(root, "tokenizer_2"))
        self.t5 = _model("T5EncoderModel", os.path.join(root, "text_encoder_2"), self.device, dtype)

    @torch.no_grad()
    def __call__(self, prompts: list[str]):
        c = self.clip_tok(prompts, padding="max_length", max_length=self.clip_len, truncation=True,
                          return_tensors="pt")
        pooled = self.clip(c.input_ids.to(self.device), output_hidden_states=False).pooler_output
        t = self.t5_tok(prompts, padding="max_length", max_length=self.t5_len, truncation=True, return_tensors="pt")
        emb = self.t5(t.input_ids.to(self.device), output_hidden_states=False)[0]
        return emb.to(self.dtype), pooled.to(self.dtype)


class UMT5TextEncoder:
    def __init__(self, model_path, device, dtype=torch.bfloat16, text_len: int = 512):
        root = str(model_path)
        self.device, self.dtype, self.text_len = torch.device(device), dtype, int(text_len)
        self.tok = _tokenizer(os.path.join(root, "tokenizer"))
        self.model = _model("UMT5EncoderModel", os.path.join(root, "text_encoder"), self.device, dtype)

    @torch.no_grad()
    def __call__(self, prompts: list[str]):
        t = self.tok(prompts, padding="max_length", max_length=self.text_len, truncation=True,
                     add_special_tokens=True, return_attention_mask=True, return_tensors="pt")
        mask = t.attention_mask
        valid = max(int(mask.sum(-1).max()), 1)
        m = mask[:, :valid].to(self.device)
        hidden = self.model(t.input_ids[:, :valid].to(self.device), m).last_hidden_state
        hidden = hidden * m.unsqueeze(-1).to(hidden.dtype)  # zero past each prompt's own length
        out = torch.zeros(len(prompts), self.text_len, hidden.shape[-1], device=self.device, dtype=self.dtype)
        out[:, :valid] = hidden.to(self.dtype)
        return out, None


@dataclass
class LMTemplate:
    template: str            # str.format template with one "{}" for the prompt
    drop_tokens: int         # template positions removed from the front of the hidden states
    max_len: int             # sequence length after the drop (padded with zeros / cut)
    skip_layers: int = 0     # hidden state of layer -1 - skip_layers
    model_cls: str = "AutoModel"
    clip_pooled: bool = False


QWEN_IMAGE_TEMPLATE = LMTemplate(
    "<|im_start|>system\nDescribe the image by detailing the color, shape, size, texture, quantity, text, spatial "
    "relationships of the objects and background:<|im_end|>\n<|im_start|>user\n{}<|im_end|>\n<|im_start|>assistant\n",
    drop_tokens=34, max_len=512)
HUNYUAN_VIDEO_TEMPLATE = LMTemplate(
    "<|start_header_id|>system<|end_header_id|>\n\nDescribe the video by detailing the following aspects: "
    "1. The main content and theme of the video.2. The color, shape, size, texture, quantity, text, and spatial "
    "relationships of the objects.3. Actions, events, behaviors temporal relationships, physical movement changes "
    "of the objects.4. background environment, light, style and atmosphere.5. camera angles, movements, and "
    "transitions used in the video:<|eot_id|><|start_header_id|>user<|end_header_id|>\n\n{}<|eot_id|>",
    drop_tokens=95, max_len=256, skip_layers=2, clip_pooled=True)


class DecoderLMTextEncoder:
    def __init__(self, model_path, device, dtype=torch.bfloat16, spec: LMTemplate = QWEN_IMAGE_TEMPLATE,
                 lm_subdir: str = "text_encoder", tok_subdir: str = "tokenizer"):
        root = str(model_path)
        self.device, self.dtype, self.spec = torch.device(device), dtype, spec
        self.tok = _tokenizer(os.path.join(root, tok_subdir))
        self.lm = _model(spec.model_cls, os.path.join(root, lm_subdir), self.device, dtype)
        self.clip = self.clip_tok = None
        if spec.clip_pooled and _has(root, "text_encoder_2", "tokenizer_2"):
            self.clip_tok = _tokenizer(os.path.join(root, "tokenizer_2"))
            self.clip = _model("CLIPTextModel", os.path.join(root, "text_encoder_2"), self.device, dtype)

    @torch.no_grad()
    def __call__(self, prompts: list[str]):
        s = self.spec
        texts = [s.template.format(p) for p in prompts]
        t = self.tok(texts, padding="max_length", max_length=s.max_len + s.drop_tokens, truncation=True,
                     return_attention_mask=True, return_tensors="pt")
        ids, mask = t.input_ids.to(self.device), t.attention_mask.to(self.device)
        hs = self.lm(input_ids=ids, attention_mask=mask, output_hidden_states=True).hidden_states
        h = hs[-1 - s.skip_layers][:, s.drop_tokens:]
        h = h * mask[:, s.drop_tokens:].unsqueeze(-1).to(h.dtype)
        out = torch.zeros(len(prompts), s.max_len, h.shape[-1], device=self.device, dtype=self.dtype)
        n = min(s.max_len, h.shape[1])
        out[:, :n] = h[:, :n].to(self.dtype)
        pooled = None
        if self.clip is not None:
            c = self.clip_tok(prompts, padding="max_length", max_length=77, truncation=True, return_tensors="pt")
            pooled = self.clip(c.input_ids.to(self.device)).pooler_output.to(self.dtype)
        return out, pooled


class LayerStateEncoder:
    """``enc(prompts) -> ([B, seq_len, hidden] with zero padding rows, None)``; ``last_valid`` holds
    the per-prompt valid token counts of the last call."""

    def __init__(self, model_path, device, dtype=torch.bfloat16, *, layer: int = 50, seq_len: int = 512,
                 lm_subdir: str = "text_encoder", tok_subdir: str = "tokenizer", weight_prefix: str | None = None):
        import json

        from safetensors import safe_open
        from transformers import AutoConfig

        root = str(model_path)
        enc_dir = os.path.join(root, lm_subdir)
        conf = AutoConfig.from_pretrained(enc_dir)
        text_conf = getattr(conf, "text_config", conf)
        if int(text_conf.num_hidden_layers) < layer:
            raise ValueError(f"the encoder has {text_conf.num_hidden_layers} layers; hidden_states[{layer}] needed")
        text_conf.num_hidden_layers = layer  # hidden_states[layer] is the output of layer index layer - 1
        if getattr(text_conf, "pad_token_id", None) is None:
            text_conf.pad_token_id = 0
        text_conf._attn_implementation = "sdpa"
        model_cls = _text_model_class(text_conf)
        with torch.device("meta"):
            model = model_cls(text_conf)
        files = sorted(f for f in os.listdir(enc_dir) if f.endswith(".safetensors"))
        idx = os.path.join(enc_dir, "model.safetensors.index.json")
        if os.path.exists(idx):
            files = sorted(set(json.load(open(idx))["weight_map"].values()))
        state = {}
        for f in files:
            with safe_open(os.path.join(enc_dir, f), framework="pt") as fh:
                for key in fh.keys():
                    name = _strip_lm_prefix(key, weight_prefix)
                    if name is None:
                        continue
                    if name.startswith("layers.") and int(name.split(".")[1]) >= layer:
                        continue
                    state[name] = fh.get_tensor(key).to(dtype)
        missing, unexpected = model.load_state_dict(state, strict=False, assign=True)
        missing = [m for m in missing if not m.endswith("inv_freq")]
        if missing or unexpected:
            raise RuntimeError(f"text encoder load: missing {missing[:4]}, unexpected {unexpected[:4]}")
        for name, buf in list(model.named_buffers()):
            if buf.is_meta:  # rotary tables: rebuilt for real from the config
                model.rotary_emb = type(model.rotary_emb)(config=text_conf)
                break
        self.model = model.to(device).eval().requires_grad_(False)
        self.tok = _tokenizer(os.path.join(root, tok_subdir))
        if self.tok.pad_token_id is None:
            self.tok.pad_token = self.tok.eos_token
        self.device, self.dtype, self.layer, self.seq_len = torch.device(device), dtype, layer, seq_len
        self.last_valid = None

    @torch.no_grad()
    def __call__(self, prompts: list[str]):
        t = self.tok(list(prompts), add_special_tokens=False, padding="max_length", max_length=self.seq_len,
                     truncation=True, return_attention_mask=True, return_tensors="pt")
        ids, mask = t.input_ids.to(self.device), t.attention_mask.to(self.device)
        captured = []
        hook = self.model.layers[self.layer - 1].register_forward_hook(
            lambda mod, args, out: captured.append(out[0] if isinstance(out, tuple) else out))
        try:
            pos = torch.arange(ids.shape[1], device=self.device)[None].expand(ids.shape[0], -1)
            self.model(input_ids=ids, attention_mask=mask, position_ids=pos, use_cache=False)
        finally:
            hook.remove()
        h = captured[-1] * mask.unsqueeze(-1).to(captured[-1].dtype)
        self.last_valid = mask.sum(1).cpu()
        return h.to(self.dtype), None


def _strip_lm_prefix(key: str, prefix: str | None):
    """The language model's own parameter name of a checkpoint key (None: not a language-model
    weight, e.g. the vision tower or lm_head)."""
    for p in ([prefix] if prefix else ["model.language_model.", "language_model.model.", "model.", ""]):
        if key.startswith(p):
            rest = key[len(p):]
            if rest.startswith(("layers.", "embed_tokens.", "norm.")):
                return rest
    return None


def _text_model_class(text_conf):
    mt = getattr(text_conf, "model_type", "")
    if mt.startswith("qwen3_vl"):
        from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLTextModel

        return Qwen3VLTextModel
    from transformers import AutoModel

    return type(AutoModel.from_config(text_conf))


def load_text_encoder(family: str, model_path, device, dtype=torch.bfloat16, **kw):
    """The family's encoder from ``model_path`` (diffusers layout), or None without encoder folders."""
    if family == "flux":
        if not _has(model_path, "text_encoder", "tokenizer", "text_encoder_2", "tokenizer_2"):
            return None
        return FluxTextEncoders(model_path, device, dtype, max_sequence_length=kw.get("max_sequence_length", 512))
    if family == "wan":
        if not _has(model_path, "text_encoder", "tokenizer"):
            return None
        return UMT5TextEncoder(model_path, device, dtype, text_len=kw.get("text_len", 512))
    if family in ("qwen_image", "hunyuan_video"):
        if not _has(model_path, "text_encoder", "tokenizer"):
            return None
        spec = kw.get("template") or (QWEN_IMAGE_TEMPLATE if family == "qwen_image" else HUNYUAN_VIDEO_TEMPLATE)
        if kw.get("max_len"):  # the pipeline's text length
            spec = dataclasses.replace(spec, max_len=int(kw["max_len"]))
        return DecoderLMTextEncoder(model_path, device, dtype, spec=spec)
    if family == "minimax_h3":
        if not _has(model_path, "text_encoder", "tokenizer"):
            return None
        return LayerStateEncoder(model_path, device, dtype, layer=int(kw.get("layer", 50)),
                                 seq_len=int(kw.get("text_len", 512)))
    raise ValueError(f"no text encoder recipe for family {family!r}")


__all__ = ["DecoderLMTextEncoder", "FluxTextEncoders", "HUNYUAN_VIDEO_TEMPLATE", "LMTemplate", "LayerStateEncoder",
           "QWEN_IMAGE_TEMPLATE", "UMT5TextEncoder", "load_text_encoder"]
