"""Wan causal VAE: streaming (frame-at-a-time) decode equals a whole-clip causal decode."""

import pytest
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


def test_native_layout_decoder_matches_reference():
    """The channels-last decoder (per-convolution cached input buffers, valid temporal
    convolutions, channel-padded first / last convolutions) equals the plain NCTHW decoder."""
    from difflet_b200.models.vae.wan_vae import WanVAEReference

    cfg = WanVAEConfig(base_dim=16)
    dec = WanVAEDecoder.random_init(cfg, dtype=torch.float64, seed=2)
    ref = WanVAEReference(cfg, dec.w)
    z = torch.randn(1, 16, 3, 4, 6, dtype=torch.float64)
    a, b = dec.decode(z), ref.decode(z)
    assert a.shape == b.shape == (1, 3, 9, 32, 48)
    assert (a - b).abs().max().item() < 1e-10


def _slab_decode(rank, world):
    import torch.distributed as dist

    from difflet_b200.models.vae.wan_vae import WanVAEReference
    from difflet_b200.parallel.slabs import CollectiveSlabs

    cfg = WanVAEConfig(base_dim=16)
    dec = WanVAEDecoder.random_init(cfg, dtype=torch.float64, seed=3)
    z = torch.randn(1, 16, 3, 7, 6, generator=torch.Generator().manual_seed(0), dtype=torch.float64)
    dec.set_slabs(CollectiveSlabs(dist.group.WORLD, list(range(world)), torch.device("cpu"), z.shape[3]))
    out = dec.decode(z)
    if rank != 0:
        return 0.0 if out is None else 1.0
    ref = WanVAEReference(cfg, dec.w).decode(z)
    return (out - ref).abs().max().item()


@pytest.mark.multirank
@pytest.mark.parametrize("world", [2, 3])
def test_slab_split_decode_matches_whole_frame(world):
    """Rows split over gloo ranks (uneven: 7 latent rows), halo rows exchanged, K / V of the
    mid-block attention gathered: rank 0's video equals the one-device decode."""
    from difflet_b200.parallel.testing import run_ranks

    errs = run_ranks(_slab_decode, world, timeout=300)
    assert max(errs) < 1e-10, errs
