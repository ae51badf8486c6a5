"""Straight-line Wan DiT forward from the diffusers math (oracle for the fused model)."""

from __future__ import annotations

import math

import torch
import torch.nn.functional as Fn

from difflet_b200.layers.rope import multi_axis_angles, video_ids


def _lin(x, sd, n):
    return x @ sd[n + ".weight"].t() + sd[n + ".bias"]


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _ln(x, eps, w=None, b=None):
    return Fn.layer_norm(x, (x.shape[-1],), weight=w, bias=b, eps=eps)


def _rope(x, ang):
    # complex multiplication on interleaved pairs
    xc = torch.view_as_complex(x.reshape(*x.shape[:-1], -1, 2).contiguous())
    f = torch.polar(torch.ones_like(ang), ang)
    return torch.view_as_real(xc * f).flatten(-2)


def _tproj(t, dim):
    half = dim // 2
    ex = -math.log(10000.0) * torch.arange(half, dtype=t.dtype) / half
    arg = t[:, None] * torch.exp(ex)[None]
    return torch.cat([torch.cos(arg), torch.sin(arg)], -1)


def wan_forward(cfg, sd, x_tokens, timestep, text, grid):
    D, H, dh, eps = cfg.hidden, cfg.heads, cfg.head_dim, cfg.eps
    B, S, _ = x_tokens.shape
    ce = "condition_embedder."
    temb = _lin(Fn.silu(_lin(_tproj(timestep, cfg.timestep_dim), sd, ce + "time_embedder.linear_1")), sd,
                ce + "time_embedder.linear_2")
    tproj = _lin(Fn.silu(temb), sd, ce + "time_proj").view(B, 6, D)
    ctx = _lin(Fn.gelu(_lin(text, sd, ce + "text_embedder.linear_1"), approximate="tanh"), sd,
               ce + "text_embedder.linear_2")
    ang = multi_axis_angles(video_ids(*grid), cfg.axes_dim, cfg.theta).to(x_tokens.dtype)
    x = x_tokens @ sd["patch_embedding.weight"].reshape(D, -1).t() + sd["patch_embedding.bias"]

    def heads(t):
        return t.view(B, -1, H, dh).transpose(1, 2)

    def attn(q, k, v):
        s = torch.einsum("bhqd,bhkd->bhqk", q, k) / math.sqrt(dh)
        return torch.einsum("bhqk,bhkd->bhqd", torch.softmax(s, -1), v).transpose(1, 2).reshape(B, -1, D)

    for i in range(cfg.layers):
        s = f"blocks.{i}."
        e = sd[s + "scale_shift_table"].reshape(1, 6, D) + tproj
        sh, sc, g, csh, csc, cg = (e[:, j:j + 1] for j in range(6))
        a1, a2 = s + "attn1.", s + "attn2."
        n = _ln(x, eps) * (1 + sc) + sh
        q = heads(_rms(_lin(n, sd, a1 + "to_q"), sd[a1 + "norm_q.weight"], eps))
        k = heads(_rms(_lin(n, sd, a1 + "to_k"), sd[a1 + "norm_k.weight"], eps))
        v = heads(_lin(n, sd, a1 + "to_v"))
        x = x + g * _lin(attn(_rope(q, ang), _rope(k, ang), v), sd, a1 + "to_out.0")
        n = _ln(x, eps, sd[s + "norm2.weight"], sd[s + "norm2.bias"])
        q = heads(_rms(_lin(n, sd, a2 + "to_q"), sd[a2 + "norm_q.weight"], eps))
        k = heads(_rms(_lin(ctx, sd, a2 + "to_k"), sd[a2 + "norm_k.weight"], eps))
        v = heads(_lin(ctx, sd, a2 + "to_v"))
        x = x + _lin(attn(q, k, v), sd, a2 + "to_out.0")
        n = _ln(x, eps) * (1 + csc) + csh
        x = x + cg * _lin(Fn.gelu(_lin(n, sd, s + "ffn.net.0.proj"), approximate="tanh"), sd, s + "ffn.net.2")
    shift, scale = (sd["scale_shift_table"].reshape(1, 2, D) + temb[:, None]).chunk(2, 1)
    x = _ln(x, eps) * (1 + scale) + shift
    return _lin(x, sd, "proj_out")
