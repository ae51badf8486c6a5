"""HunyuanVideo and Qwen-Image on the shared fused MMDiT vs the straight-line oracle (float64)."""

import pytest
import torch

from difflet_b200.models.mmdit import MMDiT, get_config, pack_latents
from difflet_b200.models.mmdit.weights import convert_diffusers, to_diffusers
from difflet_b200.oracle.flux_reference import mmdit_forward


@pytest.mark.parametrize("name", ["tiny-hunyuan", "tiny-qwen", "tiny"])
def test_roundtrip(name):
    cfg = get_config(name)
    m = MMDiT.random_init(cfg, dtype=torch.float32)
    w2 = convert_diffusers(cfg, to_diffusers(cfg, m.w))
    assert set(w2) == set(m.w)
    assert all(torch.equal(w2[k], m.w[k]) for k in w2)


def test_hunyuan_video_with_padded_text():
    cfg = get_config("tiny-hunyuan")
    m = MMDiT.random_init(cfg, dtype=torch.float64, seed=2)
    sd = to_diffusers(cfg, m.w)
    g = torch.Generator().manual_seed(1)
    B, T, Hh, Ww = 2, 3, 16, 16  # latent video 3 x 16 x 16 -> 3 x 8 x 8 tokens
    x = pack_latents(torch.randn(B, 16, T, Hh, Ww, generator=g, dtype=torch.float64))
    txt = torch.randn(B, 32, cfg.text_dim, generator=g, dtype=torch.float64)
    pooled = torch.randn(B, cfg.pooled_dim, generator=g, dtype=torch.float64)
    t = torch.tensor([0.3, 0.9], dtype=torch.float64)
    gd = torch.tensor([6.0, 6.0], dtype=torch.float64)
    valid = torch.tensor([20, 32])
    grid = (T, Hh // 2, Ww // 2)
    out = m(x, txt, pooled, t, gd, grid=grid, txt_valid=valid)
    ref = mmdit_forward(cfg, sd, x, txt, pooled, t, gd, grid=grid, txt_valid=valid)
    assert (out - ref).abs().max().item() < 1e-11 * ref.abs().max().item()


def test_qwen_image():
    cfg = get_config("tiny-qwen")
    m = MMDiT.random_init(cfg, dtype=torch.float64, seed=3)
    sd = to_diffusers(cfg, m.w)
    g = torch.Generator().manual_seed(2)
    x = pack_latents(torch.randn(1, 16, 20, 24, generator=g, dtype=torch.float64))
    txt = torch.randn(1, 40, cfg.text_dim, generator=g, dtype=torch.float64)
    t = torch.tensor([0.5], dtype=torch.float64)
    grid = (1, 10, 12)
    out = m(x, txt, None, t, grid=grid)
    ref = mmdit_forward(cfg, sd, x, txt, None, t, grid=grid)
    assert (out - ref).abs().max().item() < 1e-11 * ref.abs().max().item()
