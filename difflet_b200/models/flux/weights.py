"""FLUX checkpoint conversion: diffusers ``FluxTransformer2DModel`` names -> fused layout.

The reference converts HF weights for its own module tree
(``difflet/models/flux/modeling_flux.py:1475-1519``, including the
``proj_out`` split of the single blocks); here the fusion goes the other way:
q/k/v are concatenated per stream, the single block's q/k/v/proj_mlp become one
``[q | mlp | k | v]`` matrix, and every adaLN linear becomes a row range of one
modulation matrix.  ``to_diffusers_state_dict`` inverts the conversion (used by
the tests and by ``difflet_b200 download --random`` to write a checkpoint in
the standard layout).
"""

from __future__ import annotations

import torch

from difflet_b200.models.flux.config import FluxConfig


def convert_diffusers_flux(cfg: FluxConfig, sd: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    D, F_ = cfg.hidden, cfg.mlp_hidden
    g = lambda k: sd[k]  # noqa: E731
    w: dict[str, torch.Tensor] = {}
    w["x_embed.w"], w["x_embed.b"] = g("x_embedder.weight"), g("x_embedder.bias")
    w["ctx_embed.w"], w["ctx_embed.b"] = g("context_embedder.weight"), g("context_embedder.bias")
    tt = "time_text_embed."
    w["t_embed.w1"], w["t_embed.b1"] = g(tt + "timestep_embedder.linear_1.weight"), g(tt + "timestep_embedder.linear_1.bias")
    w["t_embed.w2"], w["t_embed.b2"] = g(tt + "timestep_embedder.linear_2.weight"), g(tt + "timestep_embedder.linear_2.bias")
    if cfg.guidance_embed:
        w["g_embed.w1"], w["g_embed.b1"] = g(tt + "guidance_embedder.linear_1.weight"), g(tt + "guidance_embedder.linear_1.bias")
        w["g_embed.w2"], w["g_embed.b2"] = g(tt + "guidance_embedder.linear_2.weight"), g(tt + "guidance_embedder.linear_2.bias")
    w["p_embed.w1"], w["p_embed.b1"] = g(tt + "text_embedder.linear_1.weight"), g(tt + "text_embedder.linear_1.bias")
    w["p_embed.w2"], w["p_embed.b2"] = g(tt + "text_embedder.linear_2.weight"), g(tt + "text_embedder.linear_2.bias")
    mods_w, mods_b = [], []
    for i in range(cfg.double_blocks):
        p = f"transformer_blocks.{i}."
        q = f"double.{i}."
        mods_w += [g(p + "norm1.linear.weight"), g(p + "norm1_context.linear.weight")]
        mods_b += [g(p + "norm1.linear.bias"), g(p + "norm1_context.linear.bias")]
        a = p + "attn."
        w[q + "img_qkv.w"] = torch.cat([g(a + "to_q.weight"), g(a + "to_k.weight"), g(a + "to_v.weight")], 0)
        w[q + "img_qkv.b"] = torch.cat([g(a + "to_q.bias"), g(a + "to_k.bias"), g(a + "to_v.bias")], 0)
        w[q + "txt_qkv.w"] = torch.cat([g(a + "add_q_proj.weight"), g(a + "add_k_proj.weight"), g(a + "add_v_proj.weight")], 0)
        w[q + "txt_qkv.b"] = torch.cat([g(a + "add_q_proj.bias"), g(a + "add_k_proj.bias"), g(a + "add_v_proj.bias")], 0)
        w[q + "img_qnorm"], w[q + "img_knorm"] = g(a + "norm_q.weight"), g(a + "norm_k.weight")
        w[q + "txt_qnorm"], w[q + "txt_knorm"] = g(a + "norm_added_q.weight"), g(a + "norm_added_k.weight")
        w[q + "img_out.w"], w[q + "img_out.b"] = g(a + "to_out.0.weight"), g(a + "to_out.0.bias")
        w[q + "txt_out.w"], w[q + "txt_out.b"] = g(a + "to_add_out.weight"), g(a + "to_add_out.bias")
        w[q + "img_up.w"], w[q + "img_up.b"] = g(p + "ff.net.0.proj.weight"), g(p + "ff.net.0.proj.bias")
        w[q + "img_down.w"], w[q + "img_down.b"] = g(p + "ff.net.2.weight"), g(p + "ff.net.2.bias")
        w[q + "txt_up.w"], w[q + "txt_up.b"] = g(p + "ff_context.net.0.proj.weight"), g(p + "ff_context.net.0.proj.bias")
        w[q + "txt_down.w"], w[q + "txt_down.b"] = g(p + "ff_context.net.2.weight"), g(p + "ff_context.net.2.bias")
    for j in range(cfg.single_blocks):
        p = f"single_transformer_blocks.{j}."
        q = f"single.{j}."
        mods_w.append(g(p + "norm.linear.weight"))
        mods_b.append(g(p + "norm.linear.bias"))
        a = p + "attn."
        w[q + "fused.w"] = torch.cat([g(a + "to_q.weight"), g(p + "proj_mlp.weight"), g(a + "to_k.weight"), g(a + "to_v.weight")], 0)
        w[q + "fused.b"] = torch.cat([g(a + "to_q.bias"), g(p + "proj_mlp.bias"), g(a + "to_k.bias"), g(a + "to_v.bias")], 0)
        w[q + "qnorm"], w[q + "knorm"] = g(a + "norm_q.weight"), g(a + "norm_k.weight")
        w[q + "proj.w"], w[q + "proj.b"] = g(p + "proj_out.weight"), g(p + "proj_out.bias")
    mods_w.append(g("norm_out.linear.weight"))
    mods_b.append(g("norm_out.linear.bias"))
    w["mod.w"] = torch.cat(mods_w, 0)
    w["mod.b"] = torch.cat(mods_b, 0)
    w["final.w"], w["final.b"] = g("proj_out.weight"), g("proj_out.bias")
    assert w["mod.w"].shape[0] == cfg.mod_rows, (w["mod.w"].shape, cfg.mod_rows)
    return {k: v.contiguous() for k, v in w.items()}


def to_diffusers_state_dict(cfg: FluxConfig, w: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    D, F_ = cfg.hidden, cfg.mlp_hidden
    sd: dict[str, torch.Tensor] = {}
    sd["x_embedder.weight"], sd["x_embedder.bias"] = w["x_embed.w"], w["x_embed.b"]
    sd["context_embedder.weight"], sd["context_embedder.bias"] = w["ctx_embed.w"], w["ctx_embed.b"]
    tt = "time_text_embed."
    for src, dst in (("t_embed", "timestep_embedder"), ("g_embed", "guidance_embedder"), ("p_embed", "text_embedder")):
        if src + ".w1" not in w:
            continue
        sd[f"{tt}{dst}.linear_1.weight"], sd[f"{tt}{dst}.linear_1.bias"] = w[src + ".w1"], w[src + ".b1"]
        sd[f"{tt}{dst}.linear_2.weight"], sd[f"{tt}{dst}.linear_2.bias"] = w[src + ".w2"], w[src + ".b2"]
    mw, mb = w["mod.w"], w["mod.b"]
    for i in range(cfg.double_blocks):
        p, q = f"transformer_blocks.{i}.", f"double.{i}."
        o = cfg.double_mod_offset(i, "img")
        sd[p + "norm1.linear.weight"], sd[p + "norm1.linear.bias"] = mw[o:o + 6 * D], mb[o:o + 6 * D]
        o = cfg.double_mod_offset(i, "txt")
        sd[p + "norm1_context.linear.weight"], sd[p + "norm1_context.linear.bias"] = mw[o:o + 6 * D], mb[o:o + 6 * D]
        a = p + "attn."
        for st, names in (("img", ("to_q", "to_k", "to_v")), ("txt", ("add_q_proj", "add_k_proj", "add_v_proj"))):
            W, Bv = w[q + st + "_qkv.w"], w[q + st + "_qkv.b"]
            for n, name in enumerate(names):
                sd[a + name + ".weight"], sd[a + name + ".bias"] = W[n * D:(n + 1) * D], Bv[n * D:(n + 1) * D]
        sd[a + "norm_q.weight"], sd[a + "norm_k.weight"] = w[q + "img_qnorm"], w[q + "img_knorm"]
        sd[a + "norm_added_q.weight"], sd[a + "norm_added_k.weight"] = w[q + "txt_qnorm"], w[q + "txt_knorm"]
        sd[a + "to_out.0.weight"], sd[a + "to_out.0.bias"] = w[q + "img_out.w"], w[q + "img_out.b"]
        sd[a + "to_add_out.weight"], sd[a + "to_add_out.bias"] = w[q + "txt_out.w"], w[q + "txt_out.b"]
        sd[p + "ff.net.0.proj.weight"], sd[p + "ff.net.0.proj.bias"] = w[q + "img_up.w"], w[q + "img_up.b"]
        sd[p + "ff.net.2.weight"], sd[p + "ff.net.2.bias"] = w[q + "img_down.w"], w[q + "img_down.b"]
        sd[p + "ff_context.net.0.proj.weight"], sd[p + "ff_context.net.0.proj.bias"] = w[q + "txt_up.w"], w[q + "txt_up.b"]
        sd[p + "ff_context.net.2.weight"], sd[p + "ff_context.net.2.bias"] = w[q + "txt_down.w"], w[q + "txt_down.b"]
    for j in range(cfg.single_blocks):
        p, q = f"single_transformer_blocks.{j}.", f"single.{j}."
        o = cfg.single_mod_offset(j)
        sd[p + "norm.linear.weight"], sd[p + "norm.linear.bias"] = mw[o:o + 3 * D], mb[o:o + 3 * D]
        W, Bv = w[q + "fused.w"], w[q + "fused.b"]
        a = p + "attn."
        sd[a + "to_q.weight"], sd[a + "to_q.bias"] = W[:D], Bv[:D]
        sd[p + "proj_mlp.weight"], sd[p + "proj_mlp.bias"] = W[D:D + F_], Bv[D:D + F_]
        sd[a + "to_k.weight"], sd[a + "to_k.bias"] = W[D + F_:2 * D + F_], Bv[D + F_:2 * D + F_]
        sd[a + "to_v.weight"], sd[a + "to_v.bias"] = W[2 * D + F_:], Bv[2 * D + F_:]
        sd[a + "norm_q.weight"], sd[a + "norm_k.weight"] = w[q + "qnorm"], w[q + "knorm"]
        sd[p + "proj_out.weight"], sd[p + "proj_out.bias"] = w[q + "proj.w"], w[q + "proj.b"]
    o = cfg.final_mod_offset()
    sd["norm_out.linear.weight"], sd["norm_out.linear.bias"] = mw[o:o + 2 * D], mb[o:o + 2 * D]
    sd["proj_out.weight"], sd["proj_out.bias"] = w["final.w"], w["final.b"]
    return {k: v.contiguous() for k, v in sd.items()}
