"""Straight-line PyTorch LTX-2 forward (no fused ops): the oracle the fused model is
checked against in float64.  Same weights dict and conventions as
``difflet_b200.models.ltx_2.model``."""

from __future__ import annotations

import math

import torch
import torch.nn.functional as TF

from difflet_b200.models.ltx_2.model import rope_angles


def _lin(x, w, b=None):
    y = x @ w.t()
    return y + b if b is not None else y


def _rms(x, eps, weight=None):
    y = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return y * weight if weight is not None else y


def _heads(x, H):
    B, S, D = x.shape
    return x.view(B, S, H, D // H).transpose(1, 2)


def _rope_half(x, cos, sin):
    # x [B, H, S, dh]; cos/sin [S, H * dh/2] (per-head tables)
    B, H, S, dh = x.shape
    c = cos.view(S, H, dh // 2).transpose(0, 1)
    s = sin.view(S, H, dh // 2).transpose(0, 1)
    x1, x2 = x[..., : dh // 2], x[..., dh // 2:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)


def _attn(q, k, v, mask=None):
    s = q @ k.transpose(-1, -2) / math.sqrt(q.shape[-1])
    if mask is not None:
        s = s.masked_fill(~mask, float("-inf"))
    return torch.softmax(s, -1) @ v


def _ts(t, dim):
    half = dim // 2
    f = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float64) / half)
    a = (t * 1000.0)[:, None].double() * f[None]
    return torch.cat([a.cos(), a.sin()], -1).to(t.dtype)


def ltx2_forward(cfg, w, video, audio, timestep, text, vcoords, acoords, text_valid=None, perturb_blocks=(),
                 isolate_modalities=False, audio_text=None):
    eps = cfg.eps
    B, Sv, _ = video.shape
    Sa = audio.shape[1]
    V, A = cfg.dim, cfg.audio_dim
    Hv, Ha = cfg.heads, cfg.audio_heads
    audio_text = text if audio_text is None else audio_text
    tf = _ts(timestep, cfg.timestep_dim)
    tv = _lin(TF.silu(_lin(tf, w["t.w1"], w["t.b1"])), w["t.w2"], w["t.b2"])
    ta = _lin(TF.silu(_lin(tf, w["at.w1"], w["at.b1"])), w["at.w2"], w["at.b2"])
    mv = _lin(TF.silu(tv), w["t.mod.w"], w["t.mod.b"]).view(B, 6, V)
    ma = _lin(TF.silu(ta), w["at.mod.w"], w["at.mod.b"]).view(B, 6, A)
    avv = _lin(TF.silu(tv), w["av.v.w"], w["av.v.b"]).view(B, 3, V)
    ava = _lin(TF.silu(ta), w["av.a.w"], w["av.a.b"]).view(B, 3, A)
    ang_v = rope_angles(vcoords, cfg.max_pos, V, cfg.theta)
    ang_a = rope_angles(acoords, (cfg.audio_max_pos,), A, cfg.theta)
    ang_vt = rope_angles(vcoords[:, :1], (cfg.audio_max_pos,), A, cfg.theta)
    rv, ra, rvt = [(a.cos().to(video.dtype), a.sin().to(video.dtype)) for a in (ang_v, ang_a, ang_vt)]
    mask = None
    if text_valid is not None:
        L = text.shape[1]
        mask = (torch.arange(L)[None] < text_valid[:, None])[:, None, None, :]
    ctx_v = _lin(TF.gelu(_lin(text, w["cap.w1"], w["cap.b1"]), approximate="tanh"), w["cap.w2"], w["cap.b2"])
    ctx_a = _lin(TF.gelu(_lin(audio_text, w["acap.w1"], w["acap.b1"]), approximate="tanh"), w["acap.w2"], w["acap.b2"])
    hv = _lin(video, w["proj_in.w"], w["proj_in.b"])
    ha = _lin(audio, w["audio_proj_in.w"], w["audio_proj_in.b"])

    def mod(x, shift, scale):
        return _rms(x, eps) * (1 + scale[:, None]) + shift[:, None]

    for i in range(cfg.layers):
        p = f"blk.{i}."
        sv = w[p + "sst"][None] + mv
        sa = w[p + "asst"][None] + ma
        cv = w[p + "v_av"][None] + avv
        ca = w[p + "a_av"][None] + ava
        for st, H, r, ssx in (("v", Hv, rv, sv), ("a", Ha, ra, sa)):
            x = hv if st == "v" else ha
            D = x.shape[-1]
            qkv = _lin(mod(x, ssx[:, 0], ssx[:, 1]), w[p + st + "_qkv.w"], w[p + st + "_qkv.b"])
            q, k, v = qkv.split(D, -1)
            q = _rope_half(_heads(_rms(q, eps, w[p + st + "_qn"]), H), *r)
            k = _rope_half(_heads(_rms(k, eps, w[p + st + "_kn"]), H), *r)
            v = _heads(v, H)
            o = v if i in perturb_blocks else _attn(q, k, v)
            o = o.transpose(1, 2).reshape(B, -1, D)
            x = x + ssx[:, 2][:, None] * _lin(o, w[p + st + "_o.w"], w[p + st + "_o.b"])
            if st == "v":
                hv = x
            else:
                ha = x
        for st, H, ctx in (("v", Hv, ctx_v), ("a", Ha, ctx_a)):
            x = hv if st == "v" else ha
            D = x.shape[-1]
            q = _heads(_rms(_lin(_rms(x, eps), w[p + st + "_cq.w"], w[p + st + "_cq.b"]), eps, w[p + st + "_cqn"]), H)
            kv = _lin(ctx, w[p + st + "_ckv.w"], w[p + st + "_ckv.b"])
            k, v = kv.split(D, -1)
            k = _heads(_rms(k, eps, w[p + st + "_ckn"]), H)
            v = _heads(v, H)
            o = _attn(q, k, v, mask).transpose(1, 2).reshape(B, -1, D)
            x = x + _lin(o, w[p + st + "_co.w"], w[p + st + "_co.b"])
            if st == "v":
                hv = x
            else:
                ha = x
        if not isolate_modalities:
            nv_kv, na_kv = _rms(hv, eps), _rms(ha, eps)

            def cross(xq, xkv, name, c, rq, rk):
                q = _lin(mod(xq, c[:, 0], c[:, 1]), w[p + name + "_q.w"], w[p + name + "_q.b"])
                q = _rope_half(_heads(_rms(q, eps, w[p + name + "_qn"]), Ha), *rq)
                kv = _lin(xkv, w[p + name + "_kv.w"], w[p + name + "_kv.b"])
                k, v = kv.split(A, -1)
                k = _rope_half(_heads(_rms(k, eps, w[p + name + "_kn"]), Ha), *rk)
                o = _attn(q, k, _heads(v, Ha)).transpose(1, 2).reshape(B, -1, A)
                return xq + c[:, 2][:, None] * _lin(o, w[p + name + "_o.w"], w[p + name + "_o.b"])

            hv_new = cross(hv, na_kv, "a2v", cv, rvt, ra)
            ha = cross(ha, nv_kv, "v2a", ca, ra, rvt)
            hv = hv_new
        for st, ssx in (("v", sv), ("a", sa)):
            x = hv if st == "v" else ha
            h = TF.gelu(_lin(mod(x, ssx[:, 3], ssx[:, 4]), w[p + st + "_up.w"], w[p + st + "_up.b"]),
                        approximate="tanh")
            x = x + ssx[:, 5][:, None] * _lin(h, w[p + st + "_down.w"], w[p + st + "_down.b"])
            if st == "v":
                hv = x
            else:
                ha = x
    outs = []
    for x, sst, temb, wo, bo in ((hv, "sst_out", tv, "proj_out.w", "proj_out.b"),
                                 (ha, "asst_out", ta, "audio_proj_out.w", "audio_proj_out.b")):
        fm = w[sst][None] + temb[:, None]
        n = TF.layer_norm(x, (x.shape[-1],), eps=eps) * (1 + fm[:, 1][:, None]) + fm[:, 0][:, None]
        outs.append(_lin(n, w[wo], w[bo]))
    return outs[0], outs[1]
