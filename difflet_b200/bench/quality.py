"""Output-quality metrics for bench comparisons (reference: difflet/bench/quality.py:27-133):
latent relative L2 and cosine, frame PSNR and SSIM (8-bit frames, Gaussian-window SSIM of
Wang et al. 2004 with sigma 1.5, 11x11 window, C1 = (0.01 L)^2, C2 = (0.03 L)^2, on luma).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rel_l2(x: torch.Tensor, ref: torch.Tensor) -> float:
    x, ref = x.double(), ref.double()
    return float((x - ref).norm() / ref.norm().clamp_min(1e-30))


def cosine(x: torch.Tensor, ref: torch.Tensor) -> float:
    return float(F.cosine_similarity(x.double().reshape(1, -1), ref.double().reshape(1, -1)).item())


def psnr(x: torch.Tensor, ref: torch.Tensor, peak: float = 255.0) -> float:
    """PSNR in dB of uint8-range frames [..., H, W, 3] (inf for identical frames)."""
    mse = float(((x.double() - ref.double()) ** 2).mean())
    return math.inf if mse == 0 else 10.0 * math.log10(peak * peak / mse)


def _luma(x: torch.Tensor) -> torch.Tensor:
    """[..., H, W, 3] -> [N, 1, H, W] (BT.601 luma)."""
    x = x.double()
    y = 0.299 * x[..., 0] + 0.587 * x[..., 1] + 0.114 * x[..., 2]
    return y.reshape(-1, 1, *y.shape[-2:])


def ssim(x: torch.Tensor, ref: torch.Tensor, peak: float = 255.0) -> float:
    """Mean SSIM over frames of [..., H, W, 3] uint8-range images."""
    a, b = _luma(x), _luma(ref)
    k = torch.arange(11, dtype=torch.float64) - 5
    g = torch.exp(-(k ** 2) / (2 * 1.5 ** 2))
    g = (g / g.sum()).to(a.device)
    win = (g[:, None] * g[None, :])[None, None]
    conv = lambda t: F.conv2d(t, win)  # noqa: E731  (valid region, as the original definition)
    mu_a, mu_b = conv(a), conv(b)
    saa = conv(a * a) - mu_a ** 2
    sbb = conv(b * b) - mu_b ** 2
    sab = conv(a * b) - mu_a * mu_b
    c1, c2 = (0.01 * peak) ** 2, (0.03 * peak) ** 2
    m = ((2 * mu_a * mu_b + c1) * (2 * sab + c2)) / ((mu_a ** 2 + mu_b ** 2 + c1) * (saa + sbb + c2))
    return float(m.mean())


def compare(out: torch.Tensor, ref: torch.Tensor, *, frames: bool = False) -> dict:
    """The metric set of one output against a reference output."""
    d = {"rel_l2": rel_l2(out, ref), "cosine": cosine(out, ref)}
    if frames:
        d["psnr_db"] = psnr(out, ref)
        d["ssim"] = ssim(out, ref)
    return d


__all__ = ["compare", "cosine", "psnr", "rel_l2", "ssim"]
