"""Rotary embeddings of the public op surface (difflet/ops/embeddings.py; laws of
difflet/backends/_torch_megatron/embeddings.py:13-37).  Tables are full head-dim
``cos`` / ``sin`` with each frequency repeated for its (even, odd) pair.  The built-in
models rotate q/k inside the fused norm + RoPE + scatter kernel instead."""

from __future__ import annotations

import torch


def apply_rotary_emb(hidden_states, freqs_cos, freqs_sin):
    """Interleaved pairs (x0, x1) -> (x0 cos - x1 sin, x0 sin + x1 cos), in the input dtype."""
    dt = hidden_states.dtype
    x1, x2 = hidden_states.unflatten(-1, (-1, 2)).unbind(-1)
    cos = freqs_cos[..., 0::2]
    sin = freqs_sin[..., 1::2]
    out = torch.empty_like(hidden_states)
    out[..., 0::2] = x1 * cos - x2 * sin
    out[..., 1::2] = x1 * sin + x2 * cos
    return out.to(dt)


def apply_rotary_emb_fp32(hidden_states, freqs_cos, freqs_sin):
    """The same rotation evaluated in fp32 (x cos + rot(x) sin), cast back."""
    x = hidden_states
    re, im = x.reshape(*x.shape[:-1], -1, 2).unbind(-1)
    rot = torch.stack([-im, re], dim=-1).flatten(-2)
    return (x.float() * freqs_cos + rot.float() * freqs_sin).to(x.dtype)


def apply_rotary_emb_slices(hidden_states, freqs_cos, freqs_sin):
    """The interleaved law computed with stride-2 slices (identical to ``apply_rotary_emb``)."""
    return apply_rotary_emb(hidden_states, freqs_cos, freqs_sin)


__all__ = ["apply_rotary_emb", "apply_rotary_emb_fp32", "apply_rotary_emb_slices"]
