"""Wan checkpoint conversion: diffusers ``WanTransformer3DModel`` names <-> fused layout.

Reference: ``difflet/models/wan/checkpoint/`` (the reference keeps the diffusers
tree); here self-attention q/k/v become one [3D, D] matrix, cross-attention k/v
one [2D, D] matrix (applied once per prompt), the patch Conv3d a linear, and the
per-block ``scale_shift_table`` tensors are stacked into one [L, 6, D] f32 table.
"""

from __future__ import annotations

import torch


def _lin(sd, name):
    return sd[name + ".weight"], sd[name + ".bias"]


def convert_diffusers_wan(cfg, sd):
    D = cfg.hidden
    w = {}
    w["patch.w"] = sd["patch_embedding.weight"].reshape(D, -1)
    w["patch.b"] = sd["patch_embedding.bias"]
    ce = "condition_embedder."
    w["t.w1"], w["t.b1"] = _lin(sd, ce + "time_embedder.linear_1")
    w["t.w2"], w["t.b2"] = _lin(sd, ce + "time_embedder.linear_2")
    w["tproj.w"], w["tproj.b"] = _lin(sd, ce + "time_proj")
    w["txt.w1"], w["txt.b1"] = _lin(sd, ce + "text_embedder.linear_1")
    w["txt.w2"], w["txt.b2"] = _lin(sd, ce + "text_embedder.linear_2")
    ssts = []
    for i in range(cfg.layers):
        s, p = f"blocks.{i}.", f"blk.{i}."
        ssts.append(sd[s + "scale_shift_table"].reshape(6, D).float())
        a1, a2 = s + "attn1.", s + "attn2."
        w[p + "qkv.w"] = torch.cat([sd[a1 + f"to_{c}.weight"] for c in "qkv"], 0)
        w[p + "qkv.b"] = torch.cat([sd[a1 + f"to_{c}.bias"] for c in "qkv"], 0)
        w[p + "qn"], w[p + "kn"] = sd[a1 + "norm_q.weight"], sd[a1 + "norm_k.weight"]
        w[p + "o.w"], w[p + "o.b"] = _lin(sd, a1 + "to_out.0")
        w[p + "n2.w"], w[p + "n2.b"] = sd[s + "norm2.weight"], sd[s + "norm2.bias"]
        w[p + "cq.w"], w[p + "cq.b"] = _lin(sd, a2 + "to_q")
        w[p + "ckv.w"] = torch.cat([sd[a2 + "to_k.weight"], sd[a2 + "to_v.weight"]], 0)
        w[p + "ckv.b"] = torch.cat([sd[a2 + "to_k.bias"], sd[a2 + "to_v.bias"]], 0)
        w[p + "cqn"], w[p + "ckn"] = sd[a2 + "norm_q.weight"], sd[a2 + "norm_k.weight"]
        w[p + "co.w"], w[p + "co.b"] = _lin(sd, a2 + "to_out.0")
        w[p + "up.w"], w[p + "up.b"] = _lin(sd, s + "ffn.net.0.proj")
        w[p + "down.w"], w[p + "down.b"] = _lin(sd, s + "ffn.net.2")
    w["sst"] = torch.stack(ssts, 0)
    w["out.sst"] = sd["scale_shift_table"].reshape(2, D).float()
    w["final.w"], w["final.b"] = _lin(sd, "proj_out")
    return {k: v.contiguous() for k, v in w.items()}


def to_diffusers_wan(cfg, w):
    D = cfg.hidden
    sd = {}

    def put(n, a, b):
        sd[n + ".weight"], sd[n + ".bias"] = a, b

    pt, ph, pw = cfg.patch
    sd["patch_embedding.weight"] = w["patch.w"].reshape(D, cfg.in_channels, pt, ph, pw)
    sd["patch_embedding.bias"] = w["patch.b"]
    ce = "condition_embedder."
    put(ce + "time_embedder.linear_1", w["t.w1"], w["t.b1"])
    put(ce + "time_embedder.linear_2", w["t.w2"], w["t.b2"])
    put(ce + "time_proj", w["tproj.w"], w["tproj.b"])
    put(ce + "text_embedder.linear_1", w["txt.w1"], w["txt.b1"])
    put(ce + "text_embedder.linear_2", w["txt.w2"], w["txt.b2"])
    for i in range(cfg.layers):
        s, p = f"blocks.{i}.", f"blk.{i}."
        sd[s + "scale_shift_table"] = w["sst"][i].reshape(1, 6, D)
        a1, a2 = s + "attn1.", s + "attn2."
        for n, c in enumerate("qkv"):
            put(a1 + f"to_{c}", w[p + "qkv.w"][n * D:(n + 1) * D], w[p + "qkv.b"][n * D:(n + 1) * D])
        sd[a1 + "norm_q.weight"], sd[a1 + "norm_k.weight"] = w[p + "qn"], w[p + "kn"]
        put(a1 + "to_out.0", w[p + "o.w"], w[p + "o.b"])
        sd[s + "norm2.weight"], sd[s + "norm2.bias"] = w[p + "n2.w"], w[p + "n2.b"]
        put(a2 + "to_q", w[p + "cq.w"], w[p + "cq.b"])
        put(a2 + "to_k", w[p + "ckv.w"][:D], w[p + "ckv.b"][:D])
        put(a2 + "to_v", w[p + "ckv.w"][D:], w[p + "ckv.b"][D:])
        sd[a2 + "norm_q.weight"], sd[a2 + "norm_k.weight"] = w[p + "cqn"], w[p + "ckn"]
        put(a2 + "to_out.0", w[p + "co.w"], w[p + "co.b"])
        put(s + "ffn.net.0.proj", w[p + "up.w"], w[p + "up.b"])
        put(s + "ffn.net.2", w[p + "down.w"], w[p + "down.b"])
    sd["scale_shift_table"] = w["out.sst"].reshape(1, 2, D)
    put("proj_out", w["final.w"], w["final.b"])
    return sd
