"""Straight-line MMDiT forward (FLUX / HunyuanVideo / Qwen-Image) in plain PyTorch.

Written from the diffusers math and independent of the fused model: it reads
the diffusers-layout state dict, runs separate q/k/v linears, concatenates the
two streams in the family's order, applies interleaved RoPE from position-id
tables and plain masked softmax attention.  Used as the oracle for the fused
MMDiT (in float64 for the tiny-model parity check: 2 + 2 blocks, hidden 256, 4 Euler steps).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as Fn

from difflet_b200.layers.rope import joint_ids, multi_axis_angles


def _lin(x, sd, name):
    return x @ sd[name + ".weight"].t() + sd[name + ".bias"]


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _ln(x, eps, w=None, b=None):
    return Fn.layer_norm(x, (x.shape[-1],), weight=w, bias=b, eps=eps)


def _rope(x, ang):
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


def _attn(q, k, v, key_valid=None):
    s = torch.einsum("bhqd,bhkd->bhqk", q, k) / math.sqrt(q.shape[-1])
    if key_valid is not None:  # [B, Sk] bool
        s = s.masked_fill(~key_valid[:, None, None, :], float("-inf"))
    return torch.einsum("bhqk,bhkd->bhqd", torch.softmax(s, -1), v)


def _refiner(cfg, sd, txt, timestep, valid):
    ce = "context_embedder."
    B, S, _ = txt.shape
    H, dh = cfg.heads, cfg.head_dim
    mask = torch.arange(S)[None, :] < valid[:, None]
    pooled = (txt * mask[..., None]).sum(1) / mask.sum(1, keepdim=True)
    temb = _mlp_embed(_tproj(timestep * 1000, cfg.timestep_dim), sd, ce + "time_text_embed.timestep_embedder")
    temb = temb + _mlp_embed(pooled, sd, ce + "time_text_embed.text_embedder")
    h = _lin(txt, sd, ce + "proj_in")
    for i in range(cfg.refiner_layers):
        p = f"{ce}token_refiner.refiner_blocks.{i}."
        gm, gf = _lin(Fn.silu(temb), sd, p + "norm_out.linear")[:, None].chunk(2, -1)
        n = _ln(h, cfg.eps, sd[p + "norm1.weight"], sd[p + "norm1.bias"])
        heads = lambda x: x.view(B, S, H, dh).transpose(1, 2)  # noqa: E731
        o = _attn(heads(_lin(n, sd, p + "attn.to_q")), heads(_lin(n, sd, p + "attn.to_k")),
                  heads(_lin(n, sd, p + "attn.to_v")), mask).transpose(1, 2).reshape(B, S, -1)
        h = h + gm * _lin(o, sd, p + "attn.to_out.0")
        n = _ln(h, cfg.eps, sd[p + "norm2.weight"], sd[p + "norm2.bias"])
        h = h + gf * _lin(Fn.silu(_lin(n, sd, p + "ff.net.0.proj")), sd, p + "ff.net.2")
    return h


def mmdit_forward(cfg, sd, x_tokens, txt, pooled=None, timestep=None, guidance=None, grid=None, txt_valid=None):
    D, H, dh, eps = cfg.hidden, cfg.heads, cfg.head_dim, cfg.eps
    B, S_img, _ = x_tokens.shape
    S_txt = txt.shape[1]
    dt = x_tokens.dtype
    qwen = cfg.family == "qwen_image"
    ang = multi_axis_angles(joint_ids(cfg.family, S_txt, grid, cfg.order), cfg.axes_dim, cfg.theta).to(dt)
    if qwen:
        temb = _mlp_embed(_tproj(timestep * 1000, cfg.timestep_dim), sd, "time_text_embed.timestep_embedder")
    else:
        temb = _mlp_embed(_tproj(timestep * 1000, cfg.timestep_dim), sd, "time_text_embed.timestep_embedder")
        if cfg.guidance_embed:
            temb = temb + _mlp_embed(_tproj(guidance * 1000, cfg.timestep_dim), sd, "time_text_embed.guidance_embedder")
        if cfg.pooled_dim:
            temb = temb + _mlp_embed(pooled, sd, "time_text_embed.text_embedder")
    st = Fn.silu(temb)
    if cfg.family == "hunyuan_video":
        hs = x_tokens @ sd["x_embedder.proj.weight"].reshape(D, -1).t() + sd["x_embedder.proj.bias"]
        valid = txt_valid if txt_valid is not None else torch.full((B,), S_txt)
        es = _refiner(cfg, sd, txt, timestep, valid)
    elif qwen:
        hs = _lin(x_tokens, sd, "img_in")
        es = _lin(_rms(txt, sd["txt_norm.weight"], eps), sd, "txt_in")
    else:
        hs = _lin(x_tokens, sd, "x_embedder")
        es = _lin(txt, sd, "context_embedder")
    key_valid = None
    if txt_valid is not None and cfg.order == "img_txt":
        key_valid = torch.arange(S_img + S_txt)[None, :] < (S_img + txt_valid)[:, None]
    mod_img = "img_mod.1" if qwen else "norm1.linear"
    mod_txt = "txt_mod.1" if qwen else "norm1_context.linear"
    ff_img = ("img_mlp.net.0.proj", "img_mlp.net.2") if qwen else ("ff.net.0.proj", "ff.net.2")
    ff_txt = ("txt_mlp.net.0.proj", "txt_mlp.net.2") if qwen else ("ff_context.net.0.proj", "ff_context.net.2")

    def heads(x):
        return x.view(B, -1, H, dh).transpose(1, 2)

    def joint(img, txt_):
        return torch.cat([txt_, img], 2) if cfg.order == "txt_img" else torch.cat([img, txt_], 2)

    for i in range(cfg.double_blocks):
        p = f"transformer_blocks.{i}."
        a = p + "attn."
        sh, sc, g, sh2, sc2, g2 = _lin(st, sd, p + mod_img)[:, None].chunk(6, -1)
        csh, csc, cg, csh2, csc2, cg2 = _lin(st, sd, p + mod_txt)[:, None].chunk(6, -1)
        n = _ln(hs, eps) * (1 + sc) + sh
        nc = _ln(es, eps) * (1 + csc) + csh
        q = _rms(heads(_lin(n, sd, a + "to_q")), sd[a + "norm_q.weight"], eps)
        k = _rms(heads(_lin(n, sd, a + "to_k")), sd[a + "norm_k.weight"], eps)
        v = heads(_lin(n, sd, a + "to_v"))
        qc = _rms(heads(_lin(nc, sd, a + "add_q_proj")), sd[a + "norm_added_q.weight"], eps)
        kc = _rms(heads(_lin(nc, sd, a + "add_k_proj")), sd[a + "norm_added_k.weight"], eps)
        vc = heads(_lin(nc, sd, a + "add_v_proj"))
        o = _attn(_rope(joint(q, qc), ang), _rope(joint(k, kc), ang), joint(v, vc), key_valid)
        o = o.transpose(1, 2).reshape(B, -1, D)
        oc, oi = (o[:, :S_txt], o[:, S_txt:]) if cfg.order == "txt_img" else (o[:, S_img:], o[:, :S_img])
        hs = hs + g * _lin(oi, sd, a + "to_out.0")
        es = es + cg * _lin(oc, sd, a + "to_add_out")
        n = _ln(hs, eps) * (1 + sc2) + sh2
        hs = hs + g2 * _lin(Fn.gelu(_lin(n, sd, p + ff_img[0]), approximate="tanh"), sd, p + ff_img[1])
        nc = _ln(es, eps) * (1 + csc2) + csh2
        es = es + cg2 * _lin(Fn.gelu(_lin(nc, sd, p + ff_txt[0]), approximate="tanh"), sd, p + ff_txt[1])
    x = torch.cat([es, hs], 1) if cfg.order == "txt_img" else torch.cat([hs, es], 1)
    for j in range(cfg.single_blocks):
        p = f"single_transformer_blocks.{j}."
        a = p + "attn."
        sh, sc, g = _lin(st, sd, p + "norm.linear")[:, None].chunk(3, -1)
        n = _ln(x, eps) * (1 + sc) + sh
        mlp = Fn.gelu(_lin(n, sd, p + "proj_mlp"), approximate="tanh")
        q = _rope(_rms(heads(_lin(n, sd, a + "to_q")), sd[a + "norm_q.weight"], eps), ang)
        k = _rope(_rms(heads(_lin(n, sd, a + "to_k")), sd[a + "norm_k.weight"], eps), ang)
        v = heads(_lin(n, sd, a + "to_v"))
        o = _attn(q, k, v, key_valid).transpose(1, 2).reshape(B, -1, D)
        x = x + g * _lin(torch.cat([o, mlp], -1), sd, p + "proj_out")
    hs = x[:, S_txt:] if cfg.order == "txt_img" else x[:, :S_img]
    scale, shift = _lin(st, sd, "norm_out.linear")[:, None].chunk(2, -1)
    hs = _ln(hs, eps) * (1 + scale) + shift
    return _lin(hs, sd, "proj_out")


def flux_forward(cfg, sd, x_tokens, txt, pooled, timestep, guidance=None, img_hw=None):
    S_img = x_tokens.shape[1]
    if img_hw is None:
        side = int(round(math.sqrt(S_img)))
        img_hw = (side, S_img // side)
    return mmdit_forward(cfg, sd, x_tokens, txt, pooled, timestep, guidance, grid=(1, img_hw[0], img_hw[1]))
