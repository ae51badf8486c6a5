"""Rotary position tables.

Multi-axis RoPE as used by FLUX / HunyuanVideo / Qwen-Image (reference
``FluxPosEmbed``, ``difflet/layers/embeddings.py:148-175``, and
``get_1d_rotary_pos_embed`` ``:41-86``): for each axis ``i`` with
``axes_dim[i]`` channels, ``axes_dim[i] / 2`` frequencies
``theta ** (-2k / axes_dim[i])`` computed in float64, multiplied by that
axis' position id.  The tables are stored once per shape as float32
``cos`` / ``sin`` of shape ``[S, head_dim / 2]`` (one entry per rotated pair),
which is what the fused q/k-norm + RoPE kernel reads.
"""

from __future__ import annotations

import torch


def axis_freqs(dim: int, theta: float) -> torch.Tensor:
    return 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))


def multi_axis_angles(ids: torch.Tensor, axes_dim, theta: float = 10000.0) -> torch.Tensor:
    """ids: [S, n_axes] positions -> angles [S, sum(axes_dim)/2] (float64)."""
    parts = []
    for i, d in enumerate(axes_dim):
        f = axis_freqs(d, theta)
        parts.append(ids[:, i].to(torch.float64)[:, None] * f[None, :])
    return torch.cat(parts, dim=-1)


def rope_tables(ids: torch.Tensor, axes_dim, theta: float = 10000.0, device=None):
    ang = multi_axis_angles(ids, axes_dim, theta)
    return ang.cos().float().contiguous().to(device), ang.sin().float().contiguous().to(device)


def flux_ids(txt_len: int, h_tokens: int, w_tokens: int) -> torch.Tensor:
    """[txt ; img] position ids: text ids are zero; image ids are (0, row, col)."""
    txt = torch.zeros(txt_len, 3)
    img = torch.zeros(h_tokens, w_tokens, 3)
    img[..., 1] = torch.arange(h_tokens)[:, None]
    img[..., 2] = torch.arange(w_tokens)[None, :]
    return torch.cat([txt, img.reshape(-1, 3)], 0)


def video_ids(t_tokens: int, h_tokens: int, w_tokens: int) -> torch.Tensor:
    """(t, h, w) ids for a 3-D patch grid, row-major (t outermost)."""
    t = torch.arange(t_tokens)[:, None, None].expand(t_tokens, h_tokens, w_tokens)
    h = torch.arange(h_tokens)[None, :, None].expand(t_tokens, h_tokens, w_tokens)
    w = torch.arange(w_tokens)[None, None, :].expand(t_tokens, h_tokens, w_tokens)
    return torch.stack([t, h, w], -1).reshape(-1, 3)


def joint_ids(family: str, S_txt: int, grid, order: str = "txt_img") -> torch.Tensor:
    """Position ids of the joint sequence for an MMDiT family.

    * ``flux`` / ``hunyuan_video``: image/video tokens get (t, h, w); text gets 0
      on every axis (an identity rotation, i.e. text is not rotated).
    * ``qwen_image`` (centred "MSRoPE"): image rows / columns are centred
      (positions -(n - n//2) .. n//2 - 1); text tokens get position
      max(h//2, w//2) + i on all three axes.
    """
    t, h, w = grid
    if family == "qwen_image":
        tt = torch.arange(t)[:, None, None].expand(t, h, w)
        hh = (torch.arange(h) - (h - h // 2))[None, :, None].expand(t, h, w)
        ww = (torch.arange(w) - (w - w // 2))[None, None, :].expand(t, h, w)
        img = torch.stack([tt, hh, ww], -1).reshape(-1, 3)
        m = max(h // 2, w // 2)
        txt = torch.arange(m, m + S_txt)[:, None].expand(S_txt, 3)
    else:
        img = video_ids(t, h, w)
        txt = torch.zeros(S_txt, 3, dtype=img.dtype)
    parts = [txt, img] if order == "txt_img" else [img, txt]
    return torch.cat(parts, 0)
