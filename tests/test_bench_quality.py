"""Bench quality metrics and provenance."""

import math

import torch

from difflet_b200.bench import provenance, quality


def test_quality_metrics():
    g = torch.Generator().manual_seed(0)
    a = torch.randint(0, 256, (2, 32, 40, 3), generator=g).float()
    assert quality.psnr(a, a) == math.inf
    assert abs(quality.ssim(a, a) - 1.0) < 1e-9
    noisy = (a + torch.randn(a.shape, generator=g) * 8).clamp(0, 255)
    p = quality.psnr(noisy, a)
    assert 25 < p < 35  # sigma 8 noise: about 30 dB
    s = quality.ssim(noisy, a)
    assert 0.3 < s < 1.0
    assert quality.ssim(torch.zeros_like(a) + 128, a) < s
    x = torch.randn(100, generator=g)
    assert quality.rel_l2(x, x) == 0 and abs(quality.cosine(2 * x, x) - 1) < 1e-12
    d = quality.compare(noisy, a, frames=True)
    assert set(d) == {"rel_l2", "cosine", "psnr_db", "ssim"}


def test_provenance_fields(monkeypatch):
    monkeypatch.setenv("DIFFLET_TEST_FLAG", "1")
    d = provenance.collect()
    assert set(d) >= {"git", "packages", "device", "env"}
    assert d["packages"]["torch"] and d["env"]["DIFFLET_TEST_FLAG"] == "1"
    assert d["git"]["sha"] is None or len(d["git"]["sha"]) == 40
