"""Wan pipeline on CPU: two experts, CFG, UniPC, streaming VAE; DiffletPipeline entry."""

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
