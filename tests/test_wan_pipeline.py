"""Wan pipeline on CPU: two experts, CFG, UniPC, streaming VAE; DiffletPipeline entry."""

import pytest
import torch

from difflet_b200.models.vae.wan_vae import WanVAEConfig, WanVAEDecoder
from difflet_b200.models.wan.model import WanTransformer, get_wan_config
from difflet_b200.models.wan.pipeline import WanApplication


def test_wan_generate_tiny():
    cfg = get_wan_config("tiny-wan")
    experts = [WanTransformer.random_init(cfg, seed=i) for i in range(2)]
    vae = WanVAEDecoder.random_init(WanVAEConfig(base_dim=8), seed=0)
    app = WanApplication(experts, vae, flow_shift=5.0)
    vid = app.generate(prompt="a cat", height=64, width=96, num_frames=9, num_inference_steps=4,
                       guidance_scale=4.0, guidance_scale_2=3.0)
    assert vid.shape == (1, 9, 64, 96, 3) and vid.dtype == torch.uint8
    # determinism
    vid2 = app.generate(prompt="a cat", height=64, width=96, num_frames=9, num_inference_steps=4,
                        guidance_scale=4.0, guidance_scale_2=3.0)
    assert torch.equal(vid, vid2)


def test_wan_batched_cfg_equals_two_passes():
    cfg = get_wan_config("tiny-wan")
    e = WanTransformer.random_init(cfg, dtype=torch.float64, seed=7)
    app = WanApplication([e], None)
    g = torch.Generator().manual_seed(0)
    pe = torch.randn(1, cfg.text_len, cfg.text_dim, generator=g, dtype=torch.float64)
    ne = torch.randn(1, cfg.text_len, cfg.text_dim, generator=g, dtype=torch.float64)
    lat = torch.randn(1, 16, 2, 8, 8, generator=g)
    a = app.generate(prompt_embeds=pe, negative_prompt_embeds=ne, height=64, width=64, num_frames=5,
                     num_inference_steps=3, guidance_scale=5.0, latents=lat, output_type="latent")
    # guidance 1 path = cond only
    b = app.generate(prompt_embeds=pe, negative_prompt_embeds=ne, height=64, width=64, num_frames=5,
                     num_inference_steps=3, guidance_scale=1.0, latents=lat, output_type="latent")
    assert a.shape == b.shape == (1, 16, 2, 8, 8)
    assert not torch.allclose(a, b)


def _manual_loop(app, pe, ne, lat, steps, gs):
    """The unfused reference: batched CFG forward, combine in f64, UniPCScheduler.step."""
    from difflet_b200.models.wan.model import patchify, unpatchify
    from difflet_b200.schedulers.unipc import UniPCScheduler

    e = app.experts[0]
    cu, cc = e.prepare_context(ne), e.prepare_context(pe)
    ctx = [(torch.cat([ku, kc]), torch.cat([vu, vc])) for (ku, vu), (kc, vc) in zip(cu, cc)]
    x = patchify(lat.to(torch.float64))
    sched = UniPCScheduler(shift=app.flow_shift).set_timesteps(steps)
    grid = (lat.shape[2], lat.shape[3] // 2, lat.shape[4] // 2)
    for i in range(steps):
        t = float(sched.timesteps[i])
        v = e(torch.cat([x, x]).to(e.dtype), torch.full((2,), t, dtype=torch.float32), ctx, grid=grid)
        u, c = v[:1].to(torch.float64), v[1:].to(torch.float64)
        x = sched.step(u + gs * (c - u), x)
    return unpatchify(x, grid, app.cfg.patch, app.cfg.out_channels)


def test_wan_fused_sampler_matches_unfused_loop():
    """One fused kernel per step (CFG combine + UniPC corrector / predictor) against the
    plain scheduler driven step by step."""
    cfg = get_wan_config("tiny-wan")
    e = WanTransformer.random_init(cfg, dtype=torch.float64, seed=3)
    app = WanApplication([e], None, flow_shift=5.0)
    g = torch.Generator().manual_seed(2)
    pe = torch.randn(1, cfg.text_len, cfg.text_dim, generator=g, dtype=torch.float64)
    ne = torch.randn(1, cfg.text_len, cfg.text_dim, generator=g, dtype=torch.float64)
    lat = torch.randn(1, 16, 2, 8, 8, generator=g, dtype=torch.float64)
    fused = app.generate(prompt_embeds=pe, negative_prompt_embeds=ne, height=64, width=64, num_frames=5,
                         num_inference_steps=6, guidance_scale=5.0, latents=lat, output_type="latent")
    ref = _manual_loop(app, pe, ne, lat, 6, 5.0)
    assert fused.dtype == torch.float32
    assert (fused.double() - ref).abs().max().item() < 1e-4 * ref.abs().max().item()


def _cfg_ulysses(rank, world):
    """cfg2 x Ulysses(world/2) over gloo: the latents every rank ends with."""
    from difflet_b200.parallel.ulysses import make_cfg_parallel, make_sequence_parallel
    from difflet_b200.pipeline.parallel_config import DiffletParallelConfig

    cfg = get_wan_config("tiny-wan", heads=4, hidden=512, ffn=1024)
    par = DiffletParallelConfig(cfg_parallel_enabled=True, cp_degree=world // 2,
                                cp_mode="ulysses" if world > 2 else "gather_kv")
    dev = torch.device("cpu")
    e = WanTransformer.random_init(cfg, dtype=torch.float64, seed=4)
    seq = make_sequence_parallel(par, dev, transport="nccl")
    cfgp = make_cfg_parallel(par, dev, transport="nccl")
    app = WanApplication([e], None, flow_shift=5.0, cfg_par=cfgp, seq_par=seq)
    g = torch.Generator().manual_seed(5)
    pe = torch.randn(1, cfg.text_len, cfg.text_dim, generator=g, dtype=torch.float64)
    ne = torch.randn(1, cfg.text_len, cfg.text_dim, generator=g, dtype=torch.float64)
    lat = torch.randn(1, 16, 2, 8, 12, generator=g, dtype=torch.float64)
    out = app.generate(prompt_embeds=pe, negative_prompt_embeds=ne, height=64, width=96, num_frames=5,
                       num_inference_steps=4, guidance_scale=4.0, latents=lat, output_type="latent")
    ref_app = WanApplication([WanTransformer.random_init(cfg, dtype=torch.float64, seed=4)], None, flow_shift=5.0)
    ref = ref_app.generate(prompt_embeds=pe, negative_prompt_embeds=ne, height=64, width=96, num_frames=5,
                           num_inference_steps=4, guidance_scale=4.0, latents=lat, output_type="latent")
    return (out - ref).abs().max().item() / ref.abs().max().item()


@pytest.mark.multirank
@pytest.mark.parametrize("world", [2, 4])
def test_wan_cfg_parallel_times_ulysses_matches_one_process(world):
    """CFG-parallel (the exchange + combine + UniPC step) composed with Ulysses over gloo ranks
    equals the batched-CFG run in one process."""
    from difflet_b200.parallel.testing import run_ranks

    assert max(run_ranks(_cfg_ulysses, world, timeout=300)) < 1e-5
