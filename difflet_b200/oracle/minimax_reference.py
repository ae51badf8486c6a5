"""Straight-line PyTorch MiniMax-H3 forward (no fused ops), float64 oracle of
``difflet_b200.models.minimax_h3.model`` (same weights dict; ``up.w`` rows are the
SwiGLU value / gate halves interleaved in 32-row groups)."""

from __future__ import annotations

import math

import torch
import torch.nn.functional as TF

from difflet_b200.models.minimax_h3.model import MODALITIES, rope_table


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _swiglu(x, w_up):
    y = x @ w_up.t()
    yy = y.view(*y.shape[:-1], -1, 2, 32)
    return (yy[..., 0, :] * TF.silu(yy[..., 1, :])).flatten(-2)


def _rope(x, cos, sin, R):
    # x [B, S, H, dh]; rotate-half over the first R channels
    xr, xp = x[..., :R], x[..., R:]
    x1, x2 = xr[..., : R // 2], xr[..., R // 2:]
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s, xp], -1)


def _block(cfg, w, p, h, cos, sin, mods=None, mask=None):
    B, S, D = h.shape
    H, dh, I = cfg.heads, cfg.head_dim, cfg.inner
    sh_m, sc_m, g_m, sh_f, sc_f, g_f = mods if mods is not None else (0, 0, 1, 0, 0, 1)
    n = _rms(h, w[p + "n1"], cfg.eps) * (1 + sc_m) + sh_m
    q, k, v = (n @ w[p + "qkv.w"].t()).split(I, -1)
    q = _rms(q.view(B, S, H, dh), w[p + "qn"], cfg.qk_eps)
    k = _rms(k.view(B, S, H, dh), w[p + "kn"], cfg.qk_eps)
    if cos is not None:
        R = 2 * cos.shape[-1]
        q, k = _rope(q, cos, sin, R), _rope(k, cos, sin, R)
    s = torch.einsum("bqhd,bkhd->bhqk", q, k) / math.sqrt(dh)
    if mask is not None:
        s = s.masked_fill(~mask, float("-inf"))
    o = torch.einsum("bhqk,bkhd->bqhd", torch.softmax(s, -1), v.view(B, S, H, dh)).reshape(B, S, I)
    h = h + g_m * (o @ w[p + "o.w"].t())
    n = _rms(h, w[p + "n2"], cfg.eps) * (1 + sc_f) + sh_f
    return h + g_f * (_swiglu(n, w[p + "up.w"]) @ w[p + "down.w"].t())


def _ts(t, dim):
    half = dim // 2
    f = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float64) / half)
    a = t.double()[:, None] * f[None]
    return torch.cat([a.cos(), a.sin()], -1).to(t.dtype)


def minimax_forward(cfg, w, video_rows, audio_rows, text, timestep, timestep_indices, layout, text_valid=None):
    B = video_rows.shape[0]
    D = cfg.hidden
    L = text.shape[1]
    txt = text @ w["ctx.w"].t() + w["ctx.b"]
    mask = None
    if text_valid is not None:
        mask = (torch.arange(L)[None] < text_valid[:, None])[:, None, None, :]
    for j in range(cfg.refiner_layers):
        txt = _block(cfg, w, f"ref.{j}.", txt, None, None, mask=mask)
    txt = _rms(txt, w["ref.final"], cfg.final_eps)
    S = layout.sequence_length
    h = torch.zeros(B, S, D, dtype=video_rows.dtype)
    h[:, layout.text_indices] = txt
    h[:, layout.video_indices] = video_rows @ w["proj_in.w"].t() + w["proj_in.b"]
    h[:, layout.audio_indices] = audio_rows @ w["audio_proj_in.w"].t() + w["audio_proj_in.b"]
    temb = TF.silu(_ts(timestep, cfg.freq_dim) @ w["t.w1"].t() + w["t.b1"]) @ w["t.w2"].t() + w["t.b2"]
    ang = rope_table(layout.position_ids, cfg).to(video_rows.dtype)
    cos, sin = ang.cos(), ang.sin()
    adaln = timestep_indices.long() * MODALITIES + layout.token_tags.long()
    for i in range(cfg.layers):
        p = f"blk.{i}."
        m = (TF.silu(temb) @ w[p + "ada.w"].t() + w[p + "ada.b"]).view(-1, 6, D)[adaln]  # [S, 6, D]
        h = _block(cfg, w, p, h, cos, sin, mods=tuple(m[:, j][None] for j in range(6)))
    so = TF.silu(temb) @ w["out.w"].t() + w["out.b"]
    shift, scale = so[:, :D][timestep_indices.long()], so[:, D:][timestep_indices.long()]
    n = _rms(h, w["out.norm"], cfg.final_eps) * (1 + scale[None]) + shift[None]
    vo = n[:, layout.video_indices] @ w["proj_out.w"].t() + w["proj_out.b"]
    ao = n[:, layout.audio_indices] @ w["audio_proj_out.w"].t() + w["audio_proj_out.b"]
    return vo, ao
