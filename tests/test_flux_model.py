"""FLUX model: fused layout vs the straight-line oracle, and the tiny-MMDiT float64 parity run."""

import torch

from difflet_b200.models.flux.config import get_config
from difflet_b200.models.flux.model import FluxTransformer, pack_latents, unpack_latents
from difflet_b200.models.flux.weights import convert_diffusers_flux, to_diffusers_state_dict
from difflet_b200.oracle.flux_reference import flux_forward
from difflet_b200.schedulers import FlowMatchEulerScheduler, flux_time_shift_mu


def _inputs(cfg, B=1, S_txt=64, hw=(16, 16), dtype=torch.float64, seed=0):
    g = torch.Generator().manual_seed(seed)
    lat = torch.randn(B, cfg.latent_channels, hw[0] * 2, hw[1] * 2, generator=g, dtype=dtype)
    txt = torch.randn(B, S_txt, cfg.text_dim, generator=g, dtype=dtype)
    pooled = torch.randn(B, cfg.pooled_dim, generator=g, dtype=dtype)
    return lat, txt, pooled


def test_weight_roundtrip():
    cfg = get_config("tiny")
    m = FluxTransformer.random_init(cfg, dtype=torch.float32)
    sd = to_diffusers_state_dict(cfg, m.w)
    w2 = convert_diffusers_flux(cfg, sd)
    assert set(w2) == set(m.w)
    for k in w2:
        assert torch.equal(w2[k], m.w[k]), k


def test_fused_matches_oracle_float64():
    for name, B in (("tiny", 1), ("tiny128", 2)):
        cfg = get_config(name)
        m = FluxTransformer.random_init(cfg, dtype=torch.float64, seed=1)
        sd = to_diffusers_state_dict(cfg, m.w)
        lat, txt, pooled = _inputs(cfg, B=B)
        x = pack_latents(lat)
        t = torch.tensor([0.7] * B, dtype=torch.float64)
        g = torch.tensor([3.5] * B, dtype=torch.float64)
        out = m(x, txt, pooled, t, g, img_hw=(16, 16))
        ref = flux_forward(cfg, sd, x, txt, pooled, t, g, img_hw=(16, 16))
        err = (out - ref).abs().max().item()
        assert err < 1e-12 * max(1.0, ref.abs().max().item()), (name, err)


def test_tiny_mmdit_four_euler_steps_fp32_vs_float64():
    """The tiny MMDiT parity run: 2+2 blocks, D=256, 4x64 heads, 256 image + 64 text tokens, 4 Euler steps."""
    cfg = get_config("tiny")
    m64 = FluxTransformer.random_init(cfg, dtype=torch.float64, seed=0)
    m32 = FluxTransformer(cfg, {k: v.float() for k, v in m64.w.items()})
    lat, txt, pooled = _inputs(cfg, S_txt=64, hw=(16, 16))
    sched = FlowMatchEulerScheduler().set_timesteps(4, mu=flux_time_shift_mu(256))
    outs = {}
    for dt, m in ((torch.float64, m64), (torch.float32, m32)):
        x = pack_latents(lat.to(dt)).clone()
        for i in range(4):
            t = torch.tensor([sched.timesteps[i] / 1000.0], dtype=dt)
            v = m(x, txt.to(dt), pooled.to(dt), t, None, img_hw=(16, 16))
            x = x + sched.dt(i) * v
        outs[dt] = unpack_latents(x, 32, 32)
    diff = (outs[torch.float32].double() - outs[torch.float64]).abs().max().item()
    assert diff < 1e-4, diff
    assert torch.isfinite(outs[torch.float64]).all()


def test_pack_unpack_roundtrip():
    lat = torch.randn(2, 16, 8, 12)
    assert torch.equal(unpack_latents(pack_latents(lat), 8, 12), lat)
