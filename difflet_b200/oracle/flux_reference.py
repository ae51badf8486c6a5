"""Straight-line FLUX forward in plain PyTorch, written from the diffusers math.

Independent of the fused model: it reads the diffusers-layout state dict,
runs separate q/k/v linears, concatenates ``[text ; image]``, applies
interleaved RoPE from ``FluxPosEmbed``-style tables and plain softmax
attention.  Used as the oracle for the fused FLUX model (and, in float64, for
the tiny-model parity check of BASELINE config 1).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as Fn

from difflet_b200.layers.rope import flux_ids, multi_axis_angles


def _lin(x, sd, name):
    return x @ sd[name + ".weight"].t() + sd[name + ".bias"]


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _ln(x, eps):
    return Fn.layer_norm(x, (x.shape[-1],), eps=eps)


def _rope(x, ang):
    # x [B, H, S, dh]; ang [S, dh/2]
    cos = torch.repeat_interleave(ang.cos(), 2, -1).to(x.dtype)
    sin = torch.repeat_interleave(ang.sin(), 2, -1).to(x.dtype)
    x_real, x_imag = x[..., 0::2], x[..., 1::2]
    rot = torch.stack([-x_imag, x_real], -1).flatten(-2)
    return x * cos + rot * sin


def _tproj(t, dim):
    half = dim // 2
    ex = -math.log(10000.0) * torch.arange(half, dtype=t.dtype) / half
    arg = t[:, None] * torch.exp(ex)[None]
    return torch.cat([torch.cos(arg), torch.sin(arg)], -1)


def _mlp_embed(x, sd, name):
    return _lin(Fn.silu(_lin(x, sd, name + ".linear_1")), sd, name + ".linear_2")


def _attn(q, k, v):
    s = torch.einsum("bhqd,bhkd->bhqk", q, k) / math.sqrt(q.shape[-1])
    return torch.einsum("bhqk,bhkd->bhqd", torch.softmax(s, -1), v)


def flux_forward(cfg, sd, x_tokens, txt, pooled, timestep, guidance=None, img_hw=None):
    D, H, dh, eps = cfg.hidden, cfg.heads, cfg.head_dim, cfg.eps
    B, S_img, _ = x_tokens.shape
    S_txt = txt.shape[1]
    if img_hw is None:
        side = int(round(math.sqrt(S_img)))
        img_hw = (side, S_img // side)
    ang = multi_axis_angles(flux_ids(S_txt, *img_hw), cfg.axes_dim, cfg.theta).to(x_tokens.dtype)
    tt = "time_text_embed."
    temb = _mlp_embed(_tproj(timestep * 1000, cfg.timestep_dim), sd, tt + "timestep_embedder")
    if cfg.guidance_embed:
        temb = temb + _mlp_embed(_tproj(guidance * 1000, cfg.timestep_dim), sd, tt + "guidance_embedder")
    temb = temb + _mlp_embed(pooled, sd, tt + "text_embedder")
    st = Fn.silu(temb)
    hs = _lin(x_tokens, sd, "x_embedder")
    es = _lin(txt, sd, "context_embedder")

    def heads(x):
        return x.view(B, -1, H, dh).transpose(1, 2)

    for i in range(cfg.double_blocks):
        p = f"transformer_blocks.{i}."
        a = p + "attn."
        m = _lin(st, sd, p + "norm1.linear")[:, None]
        mc = _lin(st, sd, p + "norm1_context.linear")[:, None]
        sh, sc, g, sh2, sc2, g2 = m.chunk(6, -1)
        csh, csc, cg, csh2, csc2, cg2 = mc.chunk(6, -1)
        n = _ln(hs, eps) * (1 + sc) + sh
        nc = _ln(es, eps) * (1 + csc) + csh
        q = _rms(heads(_lin(n, sd, a + "to_q")), sd[a + "norm_q.weight"], eps)
        k = _rms(heads(_lin(n, sd, a + "to_k")), sd[a + "norm_k.weight"], eps)
        v = heads(_lin(n, sd, a + "to_v"))
        qc = _rms(heads(_lin(nc, sd, a + "add_q_proj")), sd[a + "norm_added_q.weight"], eps)
        kc = _rms(heads(_lin(nc, sd, a + "add_k_proj")), sd[a + "norm_added_k.weight"], eps)
        vc = heads(_lin(nc, sd, a + "add_v_proj"))
        qq = _rope(torch.cat([qc, q], 2), ang)
        kk = _rope(torch.cat([kc, k], 2), ang)
        o = _attn(qq, kk, torch.cat([vc, v], 2)).transpose(1, 2).reshape(B, -1, D)
        oc, oi = o[:, :S_txt], o[:, S_txt:]
        hs = hs + g * _lin(oi, sd, a + "to_out.0")
        es = es + cg * _lin(oc, sd, a + "to_add_out")
        n = _ln(hs, eps) * (1 + sc2) + sh2
        hs = hs + g2 * _lin(Fn.gelu(_lin(n, sd, p + "ff.net.0.proj"), approximate="tanh"), sd, p + "ff.net.2")
        nc = _ln(es, eps) * (1 + csc2) + csh2
        es = es + cg2 * _lin(Fn.gelu(_lin(nc, sd, p + "ff_context.net.0.proj"), approximate="tanh"), sd, p + "ff_context.net.2")
    x = torch.cat([es, hs], 1)
    for j in range(cfg.single_blocks):
        p = f"single_transformer_blocks.{j}."
        a = p + "attn."
        sh, sc, g = _lin(st, sd, p + "norm.linear")[:, None].chunk(3, -1)
        n = _ln(x, eps) * (1 + sc) + sh
        mlp = Fn.gelu(_lin(n, sd, p + "proj_mlp"), approximate="tanh")
        q = _rope(_rms(heads(_lin(n, sd, a + "to_q")), sd[a + "norm_q.weight"], eps), ang)
        k = _rope(_rms(heads(_lin(n, sd, a + "to_k")), sd[a + "norm_k.weight"], eps), ang)
        v = heads(_lin(n, sd, a + "to_v"))
        o = _attn(q, k, v).transpose(1, 2).reshape(B, -1, D)
        x = x + g * _lin(torch.cat([o, mlp], -1), sd, p + "proj_out")
    hs = x[:, S_txt:]
    scale, shift = _lin(st, sd, "norm_out.linear")[:, None].chunk(2, -1)
    hs = _ln(hs, eps) * (1 + scale) + shift
    return _lin(hs, sd, "proj_out")
