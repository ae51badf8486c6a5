"""MiniMax-H3: the fused-op model against the straight-line oracle (float64), the packed
layout contract, the rectified-flow scheduler, checkpoint name round trip and a tiny
generation with and without keyframes through the engine."""

import pytest
import torch

from difflet_b200.models.minimax_h3 import layout as L
from difflet_b200.models.minimax_h3.model import MiniMaxH3Transformer, get_minimax_config
from difflet_b200.oracle.minimax_reference import minimax_forward


@pytest.mark.parametrize("anchors", [(), ("first",), ("first", "last")])
def test_minimax_matches_oracle(anchors):
    cfg = get_minimax_config("tiny-minimax-h3")
    m = MiniMaxH3Transformer.random_init(cfg, dtype=torch.float64, seed=1)
    lay = L.build_layout(num_text_tokens=6, height=64, width=96, num_frames=22, keyframe_anchors=anchors,
                         check_duration=False)
    g = torch.Generator().manual_seed(0)
    B = 2
    vr = torch.randn(B, lay.video_indices.numel(), cfg.patch_dim, generator=g, dtype=torch.float64)
    ar = torch.randn(B, lay.audio_indices.numel(), cfg.audio_in_channels, generator=g, dtype=torch.float64)
    text = torch.randn(B, 6, cfg.text_dim, generator=g, dtype=torch.float64)
    ts = torch.tensor([0.3, 0.6, 0.999], dtype=torch.float64)[: 2 + bool(anchors)]
    tidx = torch.ones(lay.sequence_length, dtype=torch.long)
    tidx[lay.audio_indices] = 0
    if anchors:
        tidx[lay.video_indices[: lay.num_condition_rows]] = 2
    valid = torch.tensor([4, 6])
    ov, oa = m(vr, ar, text, ts, tidx, lay, text_valid=valid)
    rv, ra = minimax_forward(cfg, m.w, vr, ar, text, ts, tidx, lay, text_valid=valid)
    assert (ov - rv).abs().max() < 1e-12 * rv.abs().max()
    assert (oa - ra).abs().max() < 1e-12 * ra.abs().max()


def test_layout_contract():
    lay = L.build_layout(num_text_tokens=10, height=480, width=832, num_frames=124)
    assert lay.num_latent_frames == 37 and lay.num_audio_latents == round(124 / 24 * 40)
    rows_per_frame = (480 // 32) * (832 // 32)
    assert lay.video_indices.numel() == 37 * rows_per_frame
    assert lay.sequence_length == 10 + 2 * lay.num_audio_latents + 37 * rows_per_frame
    # video time: text length then spans (1, 4, 4, 4, 4) * 5/3
    v0 = int(lay.video_indices[0])
    t = lay.position_ids[v0::rows_per_frame, 0][:6]
    assert torch.allclose(t - 10, torch.tensor([0, 1, 5, 9, 13, 17], dtype=torch.float64) * 5 / 3)
    assert L.align_num_frames(120) == 124 and L.video_latent_frames(124) == 37
    assert L.keyframe_time("first", 10, 37) == 10.0
    with pytest.raises(ValueError):
        L.build_layout(num_text_tokens=10, height=480, width=832, num_frames=60)


def test_rectified_flow_scheduler():
    from difflet_b200.schedulers.rectified_flow import RectifiedFlowScheduler

    s = RectifiedFlowScheduler(12.0).set_timesteps(5)
    assert float(s.sigmas[0]) == 1.0 and float(s.sigmas[-1]) == 0.0 and len(s) == 4
    x0 = torch.randn(3, 4)
    noise = torch.randn(3, 4)
    x = noise.clone()
    for i in range(len(s)):
        sigma = 1.0 - float(s.timesteps[i])
        v = (x0 - x) / sigma  # exact data-ward velocity
        x = s.step(v, i, x)
    assert torch.allclose(x, x0, atol=1e-5)


def test_minimax_weights_and_generation():
    from difflet_b200.models.minimax_h3.pipeline import MiniMaxH3Application
    from difflet_b200.models.minimax_h3.vae import TINY, MiniMaxDecoders
    from difflet_b200.models.minimax_h3.weights import from_diffusers, to_diffusers

    cfg = get_minimax_config("tiny-minimax-h3")
    m = MiniMaxH3Transformer.random_init(cfg, seed=3)
    w2 = from_diffusers(cfg, to_diffusers(cfg, m.w))
    assert set(w2) == set(m.w) and all(torch.equal(w2[k], m.w[k]) for k in w2)
    app = MiniMaxH3Application(m, MiniMaxDecoders.random_init(TINY))
    out = app.generate("a drum solo", height=64, width=96, num_frames=22, num_inference_steps=3, check_duration=False)
    assert out["frames"].shape == (22, 64, 96, 3) and out["audio"].shape[0] == 2
    kf = [torch.randn(1, cfg.in_channels, 1, 4, 6)]
    lat = app.generate("a drum solo", height=64, width=96, num_frames=22, num_inference_steps=3, keyframes=kf,
                       keyframe_anchors=("first",), return_latents=True, check_duration=False)
    assert lat["latents"].shape == (1, cfg.in_channels, 7, 4, 6) and torch.isfinite(lat["latents"]).all()
