"""MiniMax-H3 checkpoint names (diffusers' ``MiniMaxH3Transformer3DModel`` module names,
difflet/models/minimax_h3/modeling_minimax_h3.py:419-585) <-> the fused layout: q|k|v
fused, SwiGLU ``ff.net.0.proj`` ([value ; gate] halves) interleaved in 32-row groups
for the GEMM epilogue."""

from __future__ import annotations

import torch

from difflet_b200.ops.fused import swiglu_interleave


def _deinterleave(w_up: torch.Tensor):
    F2 = w_up.shape[0]
    g = w_up.reshape(F2 // 64, 2, 32, *w_up.shape[1:])
    return g[:, 0].reshape(F2 // 2, *w_up.shape[1:]), g[:, 1].reshape(F2 // 2, *w_up.shape[1:])


def _block_names(prefix):
    return {"n1": prefix + "norm1.weight", "n2": prefix + "norm2.weight", "qn": prefix + "attn.norm_q.weight",
            "kn": prefix + "attn.norm_k.weight", "o.w": prefix + "attn.to_out.0.weight",
            "down.w": prefix + "ff.net.2.weight"}


def from_diffusers(cfg, sd: dict) -> dict:
    w = {"proj_in.w": sd["proj_in.weight"], "proj_in.b": sd["proj_in.bias"],
         "audio_proj_in.w": sd["audio_proj_in.weight"], "audio_proj_in.b": sd["audio_proj_in.bias"],
         "ctx.w": sd["context_embedder.weight"], "ctx.b": sd["context_embedder.bias"],
         "t.w1": sd["time_embedder.linear_1.weight"], "t.b1": sd["time_embedder.linear_1.bias"],
         "t.w2": sd["time_embedder.linear_2.weight"], "t.b2": sd["time_embedder.linear_2.bias"],
         "ref.final": sd["token_refiner.final_norm.weight"], "out.norm": sd["norm_out.norm.weight"],
         "out.w": sd["norm_out.linear.weight"], "out.b": sd["norm_out.linear.bias"],
         "proj_out.w": sd["proj_out.weight"], "proj_out.b": sd["proj_out.bias"],
         "audio_proj_out.w": sd["audio_proj_out.weight"], "audio_proj_out.b": sd["audio_proj_out.bias"]}
    blocks = [(f"ref.{j}.", f"token_refiner.refiner_blocks.{j}.") for j in range(cfg.refiner_layers)]
    blocks += [(f"blk.{i}.", f"transformer_blocks.{i}.") for i in range(cfg.layers)]
    for q, p in blocks:
        for k, n in _block_names(p).items():
            w[q + k] = sd[n]
        w[q + "qkv.w"] = torch.cat([sd[p + f"attn.to_{c}.weight"] for c in "qkv"], 0)
        up = sd[p + "ff.net.0.proj.weight"]
        h, g = up.chunk(2, 0)
        w[q + "up.w"] = swiglu_interleave(h, g)
        if q.startswith("blk."):
            w[q + "ada.w"], w[q + "ada.b"] = sd[p + "adaln_proj.linear.weight"], sd[p + "adaln_proj.linear.bias"]
    return w


def to_diffusers(cfg, w: dict) -> dict:
    sd = {"proj_in.weight": w["proj_in.w"], "proj_in.bias": w["proj_in.b"],
          "audio_proj_in.weight": w["audio_proj_in.w"], "audio_proj_in.bias": w["audio_proj_in.b"],
          "context_embedder.weight": w["ctx.w"], "context_embedder.bias": w["ctx.b"],
          "time_embedder.linear_1.weight": w["t.w1"], "time_embedder.linear_1.bias": w["t.b1"],
          "time_embedder.linear_2.weight": w["t.w2"], "time_embedder.linear_2.bias": w["t.b2"],
          "token_refiner.final_norm.weight": w["ref.final"], "norm_out.norm.weight": w["out.norm"],
          "norm_out.linear.weight": w["out.w"], "norm_out.linear.bias": w["out.b"],
          "proj_out.weight": w["proj_out.w"], "proj_out.bias": w["proj_out.b"],
          "audio_proj_out.weight": w["audio_proj_out.w"], "audio_proj_out.bias": w["audio_proj_out.b"]}
    blocks = [(f"ref.{j}.", f"token_refiner.refiner_blocks.{j}.") for j in range(cfg.refiner_layers)]
    blocks += [(f"blk.{i}.", f"transformer_blocks.{i}.") for i in range(cfg.layers)]
    I = cfg.inner
    for q, p in blocks:
        for k, n in _block_names(p).items():
            sd[n] = w[q + k]
        for j, c in enumerate("qkv"):
            sd[p + f"attn.to_{c}.weight"] = w[q + "qkv.w"][j * I:(j + 1) * I]
        h, g = _deinterleave(w[q + "up.w"])
        sd[p + "ff.net.0.proj.weight"] = torch.cat([h, g], 0)
        if q.startswith("blk."):
            sd[p + "adaln_proj.linear.weight"], sd[p + "adaln_proj.linear.bias"] = w[q + "ada.w"], w[q + "ada.b"]
    return sd
