"""Normalization layers of the public op surface (difflet/ops/norm.py, semantics of
difflet/backends/_torch_megatron/norm.py:17-44): fp32 statistics; bf16 CUDA inputs run
the fused LayerNorm / RMSNorm kernel of ``csrc/norm.cu``, everything else plain torch."""

from __future__ import annotations

import torch
import torch.nn as nn

from difflet_b200.ops import fused as F


def _native_ok(x: torch.Tensor, d: int) -> bool:
    return x.is_cuda and x.dtype == torch.bfloat16 and d % 8 == 0 and x.stride(-1) == 1


def rms_norm_fp32(x: torch.Tensor, weight: torch.Tensor | None, eps: float) -> torch.Tensor:
    """RMSNorm over the last dim, fp32 statistics / normalisation / affine, cast back to x.dtype."""
    d = x.shape[-1]
    if _native_ok(x, d) and (weight is None or weight.dtype == torch.bfloat16):
        y = F.ln_modulate(x.reshape(-1, d), w=weight, eps=eps, rms=True)
        return y.view(x.shape)
    xn = x.float() * torch.rsqrt(x.float().pow(2).sum(-1, keepdim=True) / d + eps)
    if weight is not None:
        xn = xn * weight.float()
    return xn.to(x.dtype)


class RMSNorm(nn.Module):
    def __init__(self, hidden_size: int, eps: float = 1e-6, elementwise_affine: bool = True, **kwargs):
        super().__init__()
        del kwargs
        self.weight = nn.Parameter(torch.ones(hidden_size)) if elementwise_affine else None
        self.eps = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        d = x.shape[-1]
        w = self.weight
        if _native_ok(x, d) and (w is None or w.dtype == torch.bfloat16):
            return F.ln_modulate(x.reshape(-1, d), w=w, eps=self.eps, rms=True).view(x.shape)
        var = x.to(torch.float32).pow(2).mean(-1, keepdim=True)
        y = x * torch.rsqrt(var.to(x.dtype) + self.eps)
        return y * w if w is not None else y


CustomRMSNorm = RMSNorm


class LayerNorm(nn.LayerNorm):
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        d = x.shape[-1]
        w, b = self.weight, self.bias
        if len(self.normalized_shape) == 1 and _native_ok(x, d) and (w is None or w.dtype == torch.bfloat16):
            return F.ln_modulate(x.reshape(-1, d), w=w, b=b, eps=self.eps).view(x.shape)
        return super().forward(x)


__all__ = ["CustomRMSNorm", "LayerNorm", "RMSNorm", "rms_norm_fp32"]
