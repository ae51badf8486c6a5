"""LTX-2 checkpoint conversion: diffusers-style module names <-> the fused layout.

Fusions: self-attention q|k|v -> one [3D, D] matrix; text cross-attention and the
cross-modal attentions' k|v -> one [2D_kv, D_in] matrix.  Names follow diffusers'
``LTX2VideoTransformer3DModel`` (the names the reference's quantization targets
use, difflet/quant/targets.py: ``transformer_blocks.N.attn1.to_q``, ``ff.net.0.proj``,
``audio_ff``, ``audio_to_video_attn``...); top-level embedder names are this
module's own where no public name is fixed.
"""

from __future__ import annotations

import torch

_ATTN = {  # fused prefix -> (diffusers attention module, q source, kv fused)
    "v": "attn1", "a": "audio_attn1",
}
_CROSS = {"v_c": "attn2", "a_c": "audio_attn2", "a2v_": "audio_to_video_attn", "v2a_": "video_to_audio_attn"}
_TOP = {
    "proj_in": "proj_in", "audio_proj_in": "audio_proj_in", "proj_out": "proj_out", "audio_proj_out": "audio_proj_out",
    "t.mod": "time_embed.linear", "at.mod": "audio_time_embed.linear",
    "av.v": "av_cross_attn_video.linear", "av.a": "av_cross_attn_audio.linear",
}


def to_diffusers(cfg, w: dict) -> dict:
    sd = {}

    def put(name, wt, b=None):
        sd[name + ".weight"] = wt
        if b is not None:
            sd[name + ".bias"] = b

    for k, n in _TOP.items():
        put(n, w[k + ".w"], w[k + ".b"])
    for src, dst in (("cap", "caption_projection"), ("acap", "audio_caption_projection")):
        put(dst + ".linear_1", w[src + ".w1"], w[src + ".b1"])
        put(dst + ".linear_2", w[src + ".w2"], w[src + ".b2"])
    for src, dst in (("t", "time_embed"), ("at", "audio_time_embed")):
        put(dst + ".emb.timestep_embedder.linear_1", w[src + ".w1"], w[src + ".b1"])
        put(dst + ".emb.timestep_embedder.linear_2", w[src + ".w2"], w[src + ".b2"])
    sd["scale_shift_table"], sd["audio_scale_shift_table"] = w["sst_out"], w["asst_out"]
    for i in range(cfg.layers):
        p, q = f"transformer_blocks.{i}.", f"blk.{i}."
        for st, mod in _ATTN.items():
            W, B = w[q + st + "_qkv.w"], w[q + st + "_qkv.b"]
            D = W.shape[0] // 3
            for j, c in enumerate("qkv"):
                put(p + mod + f".to_{c}", W[j * D:(j + 1) * D], B[j * D:(j + 1) * D])
            put(p + mod + ".to_out.0", w[q + st + "_o.w"], w[q + st + "_o.b"])
            sd[p + mod + ".norm_q.weight"], sd[p + mod + ".norm_k.weight"] = w[q + st + "_qn"], w[q + st + "_kn"]
        for pre, mod in _CROSS.items():
            put(p + mod + ".to_q", w[q + pre + "q.w"], w[q + pre + "q.b"])
            W, B = w[q + pre + "kv.w"], w[q + pre + "kv.b"]
            D = W.shape[0] // 2
            put(p + mod + ".to_k", W[:D], B[:D])
            put(p + mod + ".to_v", W[D:], B[D:])
            put(p + mod + ".to_out.0", w[q + pre + "o.w"], w[q + pre + "o.b"])
            sd[p + mod + ".norm_q.weight"] = w[q + pre + "qn"]
            sd[p + mod + ".norm_k.weight"] = w[q + pre + "kn"]
        for st, ff in (("v", "ff"), ("a", "audio_ff")):
            put(p + ff + ".net.0.proj", w[q + st + "_up.w"], w[q + st + "_up.b"])
            put(p + ff + ".net.2", w[q + st + "_down.w"], w[q + st + "_down.b"])
        sd[p + "scale_shift_table"], sd[p + "audio_scale_shift_table"] = w[q + "sst"], w[q + "asst"]
        sd[p + "av_video_scale_shift_table"], sd[p + "av_audio_scale_shift_table"] = w[q + "v_av"], w[q + "a_av"]
    return sd


def from_diffusers(cfg, sd: dict) -> dict:
    w = {}

    def get(name):
        return sd[name + ".weight"], sd.get(name + ".bias")

    for k, n in _TOP.items():
        w[k + ".w"], w[k + ".b"] = get(n)
    for src, dst in (("cap", "caption_projection"), ("acap", "audio_caption_projection")):
        w[src + ".w1"], w[src + ".b1"] = get(dst + ".linear_1")
        w[src + ".w2"], w[src + ".b2"] = get(dst + ".linear_2")
    for src, dst in (("t", "time_embed"), ("at", "audio_time_embed")):
        w[src + ".w1"], w[src + ".b1"] = get(dst + ".emb.timestep_embedder.linear_1")
        w[src + ".w2"], w[src + ".b2"] = get(dst + ".emb.timestep_embedder.linear_2")
    w["sst_out"], w["asst_out"] = sd["scale_shift_table"], sd["audio_scale_shift_table"]
    for i in range(cfg.layers):
        p, q = f"transformer_blocks.{i}.", f"blk.{i}."
        for st, mod in _ATTN.items():
            ws, bs = zip(*(get(p + mod + f".to_{c}") for c in "qkv"))
            w[q + st + "_qkv.w"], w[q + st + "_qkv.b"] = torch.cat(ws, 0), torch.cat(bs, 0)
            w[q + st + "_o.w"], w[q + st + "_o.b"] = get(p + mod + ".to_out.0")
            w[q + st + "_qn"], w[q + st + "_kn"] = sd[p + mod + ".norm_q.weight"], sd[p + mod + ".norm_k.weight"]
        for pre, mod in _CROSS.items():
            w[q + pre + "q.w"], w[q + pre + "q.b"] = get(p + mod + ".to_q")
            (wk, bk), (wv, bv) = get(p + mod + ".to_k"), get(p + mod + ".to_v")
            w[q + pre + "kv.w"], w[q + pre + "kv.b"] = torch.cat([wk, wv], 0), torch.cat([bk, bv], 0)
            w[q + pre + "o.w"], w[q + pre + "o.b"] = get(p + mod + ".to_out.0")
            w[q + pre + "qn"], w[q + pre + "kn"] = sd[p + mod + ".norm_q.weight"], sd[p + mod + ".norm_k.weight"]
        for st, ff in (("v", "ff"), ("a", "audio_ff")):
            w[q + st + "_up.w"], w[q + st + "_up.b"] = get(p + ff + ".net.0.proj")
            w[q + st + "_down.w"], w[q + st + "_down.b"] = get(p + ff + ".net.2")
        w[q + "sst"], w[q + "asst"] = sd[p + "scale_shift_table"], sd[p + "audio_scale_shift_table"]
        w[q + "v_av"], w[q + "a_av"] = sd[p + "av_video_scale_shift_table"], sd[p + "av_audio_scale_shift_table"]
    return w
