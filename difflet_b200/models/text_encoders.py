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
    raise ValueError(f"no text encoder recipe for family {family!r}")


__all__ = ["DecoderLMTextEncoder", "FluxTextEncoders", "HUNYUAN_VIDEO_TEMPLATE", "LMTemplate", "QWEN_IMAGE_TEMPLATE",
           "UMT5TextEncoder", "load_text_encoder"]
