"""LTX-2 audio-video DiT: the fused-op model against the straight-line oracle (float64),
guidance variants, checkpoint name round trip, decoders' shape contract, a full tiny
generation through the engine, MXFP8 application."""

import pytest
import torch

from difflet_b200.models.ltx_2.model import LTX2Transformer, audio_coords, get_ltx2_config, video_coords
from difflet_b200.oracle.ltx2_reference import ltx2_forward


def _inputs(cfg, B=2, Fr=2, H=3, W=4, Ta=5, seed=0):
    g = torch.Generator().manual_seed(seed)
    v = torch.randn(B, Fr * H * W, cfg.in_channels, generator=g, dtype=torch.float64)
    a = torch.randn(B, Ta, cfg.audio_in_channels, generator=g, dtype=torch.float64)
    text = torch.randn(B, 7, cfg.text_dim, generator=g, dtype=torch.float64)
    return v, a, text, video_coords(Fr, H, W, cfg), audio_coords(Ta)


@pytest.mark.parametrize("kw", [{}, {"perturb_blocks": (1,)}, {"isolate_modalities": True}])
def test_ltx2_matches_oracle(kw):
    cfg = get_ltx2_config("tiny-ltx2")
    m = LTX2Transformer.random_init(cfg, dtype=torch.float64, seed=1)
    v, a, text, vc, ac = _inputs(cfg)
    t = torch.tensor([0.3, 0.8], dtype=torch.float64)
    valid = torch.tensor([5, 7])
    ov, oa = m(v, a, t, m.prepare_context(text), vcoords=vc, acoords=ac, text_valid=valid, **kw)
    rv, ra = ltx2_forward(cfg, m.w, v, a, t, text, vc, ac, text_valid=valid, **kw)
    assert (ov - rv).abs().max() < 1e-12 * rv.abs().max()
    assert (oa - ra).abs().max() < 1e-12 * ra.abs().max()


def test_ltx2_weight_names_roundtrip():
    from difflet_b200.models.ltx_2.weights import from_diffusers, to_diffusers
    from difflet_b200.quant import default_spec

    cfg = get_ltx2_config("tiny-ltx2")
    m = LTX2Transformer.random_init(cfg)
    sd = to_diffusers(cfg, m.w)
    w2 = from_diffusers(cfg, sd)
    assert set(w2) == set(m.w) and all(torch.equal(w2[k], m.w[k]) for k in w2)
    spec = default_spec("ltx_2")
    assert not spec.unmatched_targets([k[:-7] for k in sd if k.endswith(".weight")])


def test_ltx2_generation_and_quant():
    from difflet_b200.models.ltx_2.pipeline import LTX2Application
    from difflet_b200.models.ltx_2.vae import TINY_DECODER, LTX2Decoders
    from difflet_b200.quant import default_spec
    from difflet_b200.quant.apply import apply_quant

    cfg = get_ltx2_config("tiny-ltx2")
    m = LTX2Transformer.random_init(cfg, seed=2)
    app = LTX2Application(m, LTX2Decoders.random_init(TINY_DECODER))
    out = app.generate("a cat playing piano", height=64, width=96, num_frames=9, num_inference_steps=2,
                       guidance_scale=3.0, stg_scale=0.5, spatio_temporal_guidance_blocks=[1], modality_scale=1.5,
                       guidance_rescale=0.3)
    assert out["frames"].shape == (9, 64, 96, 3) and out["frames"].dtype.name == "uint8"
    assert out["audio"].shape[0] == 2 and out["audio"].shape[1] == round(9 / 24 * 25) * 4 * 160
    res = apply_quant(m, default_spec("ltx_2"))
    assert "blk.0.v_qkv.w" in res["quantized"] and "blk.0.a_qkv.w" not in res["quantized"]
    lat = app.generate("a cat", height=64, width=96, num_frames=9, num_inference_steps=2, return_latents=True)
    assert torch.isfinite(lat["latents"]).all() and torch.isfinite(lat["audio_latents"]).all()


def test_ltx2_engine_via_pipeline_api(tmp_path):
    from difflet_b200.pipeline.difflet_pipeline import DiffletPipeline

    pipe = DiffletPipeline.from_pretrained("Lightricks/LTX-2", random_init=True, compile_cache_dir=str(tmp_path),
                                           height=64, width=96, num_frames=9,
                                           application_kwargs={"preset": "tiny-ltx2"})
    out = pipe(prompt="waves on a beach", num_inference_steps=2, guidance_scale=1.0)
    assert out["frames"].shape == (9, 64, 96, 3)
