"""Checkpoint conversion for the MMDiT families: diffusers names <-> fused layout.

Diffusers modules and their fused targets (FLUX ``FluxTransformer2DModel``,
HunyuanVideo ``HunyuanVideoTransformer3DModel``, Qwen-Image
``QwenImageTransformer2DModel``; the reference converts the same checkpoints for
its own module tree in ``difflet/models/flux/modeling_flux.py:1475-1519`` and
``difflet/models/qwen_image/modeling_qwen_image.py``):

  q/k/v (per stream)                       -> one [3D, D] matrix
  single block to_q | proj_mlp | to_k | to_v -> one [7D, D] matrix ([q|mlp|k|v])
  every adaLN linear (per block + norm_out) -> row ranges of one modulation matrix
  HunyuanVideo patch Conv3d (kernel = stride) -> a [D, C*pt*ph*pw] linear
  HunyuanVideo token-refiner attention q/k/v -> one [3D, D] matrix per layer
"""

from __future__ import annotations

import torch

from difflet_b200.models.mmdit.config import MMDiTConfig


def _names(cfg: MMDiTConfig):
    """Per-family diffusers name table for the shared pieces."""
    if cfg.family == "qwen_image":
        return {
            "x_embed": "img_in", "ctx_embed": "txt_in", "t_embed": "time_text_embed.timestep_embedder",
            "img_mod": "img_mod.1", "txt_mod": "txt_mod.1",
            "img_up": "img_mlp.net.0.proj", "img_down": "img_mlp.net.2",
            "txt_up": "txt_mlp.net.0.proj", "txt_down": "txt_mlp.net.2",
        }
    return {
        "x_embed": "x_embedder", "ctx_embed": "context_embedder", "t_embed": "time_text_embed.timestep_embedder",
        "g_embed": "time_text_embed.guidance_embedder", "p_embed": "time_text_embed.text_embedder",
        "img_mod": "norm1.linear", "txt_mod": "norm1_context.linear",
        "img_up": "ff.net.0.proj", "img_down": "ff.net.2", "txt_up": "ff_context.net.0.proj",
        "txt_down": "ff_context.net.2",
    }


def _lin(sd, name):
    return sd[name + ".weight"], sd[name + ".bias"]


def convert_diffusers(cfg: MMDiTConfig, sd: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    D, F_ = cfg.hidden, cfg.mlp_hidden
    nm = _names(cfg)
    w: dict[str, torch.Tensor] = {}
    if cfg.family == "hunyuan_video":
        w["x_embed.w"] = sd["x_embedder.proj.weight"].reshape(D, -1)
        w["x_embed.b"] = sd["x_embedder.proj.bias"]
    else:
        w["x_embed.w"], w["x_embed.b"] = _lin(sd, nm["x_embed"])
    if cfg.refiner_layers == 0:
        w["ctx_embed.w"], w["ctx_embed.b"] = _lin(sd, nm["ctx_embed"])
    if cfg.txt_norm:
        w["txt_norm"] = sd["txt_norm.weight"]
    for key in ("t_embed", "g_embed", "p_embed"):
        if key == "g_embed" and not cfg.guidance_embed or key == "p_embed" and not cfg.pooled_dim:
            continue
        w[key + ".w1"], w[key + ".b1"] = _lin(sd, nm[key] + ".linear_1")
        w[key + ".w2"], w[key + ".b2"] = _lin(sd, nm[key] + ".linear_2")
    if cfg.refiner_layers:
        ce = "context_embedder."
        for dst, src in (("ref.t", "time_text_embed.timestep_embedder"), ("ref.p", "time_text_embed.text_embedder")):
            w[dst + ".w1"], w[dst + ".b1"] = _lin(sd, ce + src + ".linear_1")
            w[dst + ".w2"], w[dst + ".b2"] = _lin(sd, ce + src + ".linear_2")
        w["ref.proj.w"], w["ref.proj.b"] = _lin(sd, ce + "proj_in")
        for i in range(cfg.refiner_layers):
            p, s = f"ref.{i}.", f"{ce}token_refiner.refiner_blocks.{i}."
            w[p + "n1.w"], w[p + "n1.b"] = _lin(sd, s + "norm1")
            w[p + "qkv.w"] = torch.cat([sd[s + f"attn.to_{c}.weight"] for c in "qkv"], 0)
            w[p + "qkv.b"] = torch.cat([sd[s + f"attn.to_{c}.bias"] for c in "qkv"], 0)
            w[p + "out.w"], w[p + "out.b"] = _lin(sd, s + "attn.to_out.0")
            w[p + "n2.w"], w[p + "n2.b"] = _lin(sd, s + "norm2")
            w[p + "up.w"], w[p + "up.b"] = _lin(sd, s + "ff.net.0.proj")
            w[p + "down.w"], w[p + "down.b"] = _lin(sd, s + "ff.net.2")
            w[p + "ada.w"], w[p + "ada.b"] = _lin(sd, s + "norm_out.linear")
    mods_w, mods_b = [], []
    for i in range(cfg.double_blocks):
        p, q = f"transformer_blocks.{i}.", f"double.{i}."
        for st in ("img", "txt"):
            mw, mb = _lin(sd, p + nm[st + "_mod"])
            mods_w.append(mw)
            mods_b.append(mb)
        a = p + "attn."
        for st, names in (("img", ("to_q", "to_k", "to_v")), ("txt", ("add_q_proj", "add_k_proj", "add_v_proj"))):
            w[q + st + "_qkv.w"] = torch.cat([sd[a + n + ".weight"] for n in names], 0)
            w[q + st + "_qkv.b"] = torch.cat([sd[a + n + ".bias"] for n in names], 0)
        w[q + "img_qnorm"], w[q + "img_knorm"] = sd[a + "norm_q.weight"], sd[a + "norm_k.weight"]
        w[q + "txt_qnorm"], w[q + "txt_knorm"] = sd[a + "norm_added_q.weight"], sd[a + "norm_added_k.weight"]
        w[q + "img_out.w"], w[q + "img_out.b"] = _lin(sd, a + "to_out.0")
        w[q + "txt_out.w"], w[q + "txt_out.b"] = _lin(sd, a + "to_add_out")
        for st in ("img", "txt"):
            w[q + st + "_up.w"], w[q + st + "_up.b"] = _lin(sd, p + nm[st + "_up"])
            w[q + st + "_down.w"], w[q + st + "_down.b"] = _lin(sd, p + nm[st + "_down"])
    for j in range(cfg.single_blocks):
        p, q = f"single_transformer_blocks.{j}.", f"single.{j}."
        mw, mb = _lin(sd, p + "norm.linear")
        mods_w.append(mw)
        mods_b.append(mb)
        a = p + "attn."
        w[q + "fused.w"] = torch.cat([sd[a + "to_q.weight"], sd[p + "proj_mlp.weight"], sd[a + "to_k.weight"],
                                     sd[a + "to_v.weight"]], 0)
        w[q + "fused.b"] = torch.cat([sd[a + "to_q.bias"], sd[p + "proj_mlp.bias"], sd[a + "to_k.bias"],
                                     sd[a + "to_v.bias"]], 0)
        w[q + "qnorm"], w[q + "knorm"] = sd[a + "norm_q.weight"], sd[a + "norm_k.weight"]
        w[q + "proj.w"], w[q + "proj.b"] = _lin(sd, p + "proj_out")
    mw, mb = _lin(sd, "norm_out.linear")
    mods_w.append(mw)
    mods_b.append(mb)
    w["mod.w"] = torch.cat(mods_w, 0)
    w["mod.b"] = torch.cat(mods_b, 0)
    w["final.w"], w["final.b"] = _lin(sd, "proj_out")
    assert w["mod.w"].shape[0] == cfg.mod_rows, (w["mod.w"].shape, cfg.mod_rows)
    return {k: v.contiguous() for k, v in w.items()}


def to_diffusers(cfg: MMDiTConfig, w: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """Inverse of ``convert_diffusers`` (tests; writing random checkpoints in the standard layout)."""
    D, F_ = cfg.hidden, cfg.mlp_hidden
    nm = _names(cfg)
    sd: dict[str, torch.Tensor] = {}

    def put(name, wt, b):
        sd[name + ".weight"], sd[name + ".bias"] = wt, b

    if cfg.family == "hunyuan_video":
        sd["x_embedder.proj.weight"] = w["x_embed.w"].reshape(D, cfg.latent_channels, cfg.patch_t, cfg.patch, cfg.patch)
        sd["x_embedder.proj.bias"] = w["x_embed.b"]
    else:
        put(nm["x_embed"], w["x_embed.w"], w["x_embed.b"])
    if cfg.refiner_layers == 0:
        put(nm["ctx_embed"], w["ctx_embed.w"], w["ctx_embed.b"])
    if cfg.txt_norm:
        sd["txt_norm.weight"] = w["txt_norm"]
    for key in ("t_embed", "g_embed", "p_embed"):
        if key + ".w1" not in w:
            continue
        put(nm[key] + ".linear_1", w[key + ".w1"], w[key + ".b1"])
        put(nm[key] + ".linear_2", w[key + ".w2"], w[key + ".b2"])
    if cfg.refiner_layers:
        ce = "context_embedder."
        for src, dst in (("ref.t", "time_text_embed.timestep_embedder"), ("ref.p", "time_text_embed.text_embedder")):
            put(ce + dst + ".linear_1", w[src + ".w1"], w[src + ".b1"])
            put(ce + dst + ".linear_2", w[src + ".w2"], w[src + ".b2"])
        put(ce + "proj_in", w["ref.proj.w"], w["ref.proj.b"])
        for i in range(cfg.refiner_layers):
            p, s = f"ref.{i}.", f"{ce}token_refiner.refiner_blocks.{i}."
            put(s + "norm1", w[p + "n1.w"], w[p + "n1.b"])
            for n, c in enumerate("qkv"):
                put(s + f"attn.to_{c}", w[p + "qkv.w"][n * D:(n + 1) * D], w[p + "qkv.b"][n * D:(n + 1) * D])
            put(s + "attn.to_out.0", w[p + "out.w"], w[p + "out.b"])
            put(s + "norm2", w[p + "n2.w"], w[p + "n2.b"])
            put(s + "ff.net.0.proj", w[p + "up.w"], w[p + "up.b"])
            put(s + "ff.net.2", w[p + "down.w"], w[p + "down.b"])
            put(s + "norm_out.linear", w[p + "ada.w"], w[p + "ada.b"])
    mw, mb = w["mod.w"], w["mod.b"]
    for i in range(cfg.double_blocks):
        p, q = f"transformer_blocks.{i}.", f"double.{i}."
        for st in ("img", "txt"):
            o = cfg.double_mod_offset(i, st)
            put(p + nm[st + "_mod"], mw[o:o + 6 * D], mb[o:o + 6 * D])
        a = p + "attn."
        for st, names in (("img", ("to_q", "to_k", "to_v")), ("txt", ("add_q_proj", "add_k_proj", "add_v_proj"))):
            W, Bv = w[q + st + "_qkv.w"], w[q + st + "_qkv.b"]
            for n, name in enumerate(names):
                put(a + name, W[n * D:(n + 1) * D], Bv[n * D:(n + 1) * D])
        sd[a + "norm_q.weight"], sd[a + "norm_k.weight"] = w[q + "img_qnorm"], w[q + "img_knorm"]
        sd[a + "norm_added_q.weight"], sd[a + "norm_added_k.weight"] = w[q + "txt_qnorm"], w[q + "txt_knorm"]
        put(a + "to_out.0", w[q + "img_out.w"], w[q + "img_out.b"])
        put(a + "to_add_out", w[q + "txt_out.w"], w[q + "txt_out.b"])
        for st in ("img", "txt"):
            put(p + nm[st + "_up"], w[q + st + "_up.w"], w[q + st + "_up.b"])
            put(p + nm[st + "_down"], w[q + st + "_down.w"], w[q + st + "_down.b"])
    for j in range(cfg.single_blocks):
        p, q = f"single_transformer_blocks.{j}.", f"single.{j}."
        o = cfg.single_mod_offset(j)
        put(p + "norm.linear", mw[o:o + 3 * D], mb[o:o + 3 * D])
        W, Bv = w[q + "fused.w"], w[q + "fused.b"]
        a = p + "attn."
        put(a + "to_q", W[:D], Bv[:D])
        put(p + "proj_mlp", W[D:D + F_], Bv[D:D + F_])
        put(a + "to_k", W[D + F_:2 * D + F_], Bv[D + F_:2 * D + F_])
        put(a + "to_v", W[2 * D + F_:], Bv[2 * D + F_:])
        sd[a + "norm_q.weight"], sd[a + "norm_k.weight"] = w[q + "qnorm"], w[q + "knorm"]
        put(p + "proj_out", w[q + "proj.w"], w[q + "proj.b"])
    o = cfg.final_mod_offset()
    put("norm_out.linear", mw[o:o + 2 * D], mb[o:o + 2 * D])
    put("proj_out", w["final.w"], w["final.b"])
    return {k: v.contiguous() for k, v in sd.items()}
