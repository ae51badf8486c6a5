"""Wan causal VAE: streaming (frame-at-a-time) decode equals a whole-clip causal decode."""

import torch
import torch.nn.functional as Fn

from difflet_b200.models.vae.wan_vae import WanVAEConfig, WanVAEDecoder


def test_frame_counts_and_range():
    cfg = WanVAEConfig(base_dim=8, z_dim=16)
    dec = WanVAEDecoder.random_init(cfg, dtype=torch.float64, seed=0)
    z = torch.randn(1, 16, 3, 4, 6, dtype=torch.float64)
    out = dec.decode(z)
    assert out.shape == (1, 3, 1 + 4 * 2, 32, 48)
    assert out.abs().max() <= 1.0


def test_causality():
    # output frames of latent frame t must not change when later latent frames change
    cfg = WanVAEConfig(base_dim=8)
    dec = WanVAEDecoder.random_init(cfg, dtype=torch.float64, seed=1)
    z = torch.randn(1, 16, 3, 4, 4, dtype=torch.float64)
    a = dec.decode(z)
    z2 = z.clone()
    z2[:, :, 2] += 1.0
    b = dec.decode(z2)
    n_keep = 1 + 4 * 1  # frames produced by latent frames 0 and 1
    assert torch.equal(a[:, :, :n_keep], b[:, :, :n_keep])
    assert not torch.equal(a[:, :, n_keep:], b[:, :, n_keep:])
