"""MiniMax-H3 text(+keyframes) -> video + audio application.

Loop of the reference's ``denoise_minimax_h3_t2va`` (difflet/models/minimax_h3/
pipeline.py:291-506): guidance-distilled (one forward per step, no CFG); separate
rectified-flow schedules for video (shift 12) and audio (shift 3) over the same
number of steps; per-step timestep slots [audio, video] (+ keyframe slot
max(video, 0.999)) selected per packed row; keyframe condition rows (FL2VA) noised
once to t = 0.999 before the other draws and never stepped; draw order keyframes,
video, audio from one CPU generator.  Text embeddings come from a deterministic
stand-in for Qwen3-VL (no encoder weights offline).
"""

from __future__ import annotations

import torch

from difflet_b200.models.flux.pipeline import SyntheticTextEncoder
from difflet_b200.models.minimax_h3 import layout as L
from difflet_b200.models.minimax_h3.model import MiniMaxH3Transformer
from difflet_b200.schedulers.rectified_flow import RectifiedFlowScheduler


class MiniMaxH3Application:
    def __init__(self, transformer: MiniMaxH3Transformer, decoders=None, *, text_encoder=None, text_len: int = 128,
                 video_shift: float = 12.0, audio_shift: float = 3.0):
        self.dit = transformer
        self.cfg = transformer.cfg
        self.decoders = decoders
        self.text_len = text_len
        self.video_shift, self.audio_shift = video_shift, audio_shift
        self.text_encoder = text_encoder or SyntheticTextEncoder(text_len, self.cfg.text_dim, 1)

    @torch.no_grad()
    def generate(self, prompt: str, *, height=480, width=832, num_frames=124, num_inference_steps=30, seed=0,
                 keyframes=None, keyframe_anchors=(), output_type="np", return_latents=False,
                 check_duration=True, callback=None):
        """``keyframes``: condition latents [1, C, 1, H/16, W/16] per anchor ("first" / "last")."""
        dit, cfg = self.dit, self.cfg
        dev, dt = dit.device, dit.dtype
        num_frames = L.align_num_frames(num_frames)
        emb, _ = self.text_encoder([prompt])
        valid = getattr(self.text_encoder, "last_valid", None)
        if valid is not None:  # a real tokenizer's count of this prompt's tokens
            n_text = max(1, min(self.text_len, int(valid[0])))
        else:  # synthetic stand-in: a word-count estimate
            n_text = max(1, min(self.text_len, len(prompt.split()) * 2 + 1))
        text = emb[:, :n_text]
        keyframes = list(keyframes or [])
        anchors = tuple(keyframe_anchors)
        if len(keyframes) != len(anchors):
            raise ValueError(f"{len(keyframes)} keyframe latents for {len(anchors)} anchors")
        lay = L.build_layout(num_text_tokens=n_text, height=height, width=width, num_frames=num_frames,
                             keyframe_anchors=anchors, check_duration=check_duration)
        lh, lw = height // L.VAE_SPATIAL, width // L.VAE_SPATIAL
        g = torch.Generator().manual_seed(int(seed))
        vsched = RectifiedFlowScheduler(self.video_shift).set_timesteps(num_inference_steps)
        asched = RectifiedFlowScheduler(self.audio_shift).set_timesteps(num_inference_steps)
        if len(vsched) != len(asched):
            raise RuntimeError("video and audio schedules produced different step counts")
        cond_rows = None
        if keyframes:
            cond_rows = torch.cat([L.patchify(RectifiedFlowScheduler.scale_noise(
                k.float(), L.KEYFRAME_NOISE_AUG, torch.randn(k.shape, generator=g))) for k in keyframes], 1)
        video = torch.randn(1, cfg.in_channels, lay.num_latent_frames, lh, lw, generator=g)
        vrows = L.patchify(video).to(dev)
        arows = torch.randn(1, lay.num_audio_latents * L.AUDIO_CHANNELS, cfg.audio_in_channels, generator=g).to(dev)
        tidx = torch.ones(lay.sequence_length, dtype=torch.long)
        tidx[lay.audio_indices] = 0
        if keyframes:
            tidx[lay.video_indices[:lay.num_condition_rows]] = 2
        text_d = text.to(dev, dt)
        for i in range(len(vsched)):
            tv, ta = float(vsched.timesteps[i]), float(asched.timesteps[i])
            slots = [ta, tv] + ([max(tv, L.KEYFRAME_NOISE_AUG)] if keyframes else [])
            ts = torch.tensor(slots, device=dev, dtype=torch.float32 if dt != torch.float64 else dt)
            packed = torch.cat([cond_rows.to(dev), vrows], 1) if keyframes else vrows
            pv, pa = dit(packed.to(dt), arows.to(dt), text_d, ts, tidx, lay)
            vrows = vsched.step(pv[:, lay.num_condition_rows:], i, vrows)
            arows = asched.step(pa, i, arows)
            if callback is not None:  # per-step observer (video latent rows)
                callback(i, vrows)
        lat_v = L.unpatchify(vrows, cfg.in_channels, lay.num_latent_frames, lh, lw)
        lat_a = arows.reshape(L.AUDIO_CHANNELS, lay.num_audio_latents, cfg.audio_in_channels).permute(0, 2, 1)
        if return_latents or self.decoders is None:
            return {"latents": lat_v, "audio_latents": lat_a}
        d = self.decoders
        vid = d.decode_video(lat_v.to(dt), num_frames)[0]
        wav = d.decode_audio(lat_a.contiguous().to(dt)).float()
        frames = ((vid.float().clamp(-1, 1) + 1) * 127.5).round().to(torch.uint8).permute(1, 2, 3, 0).cpu()
        return {"frames": frames.numpy() if output_type == "np" else frames, "audio": wav.cpu().numpy(),
                "fps": L.FPS, "sample_rate": d.cfg.sample_rate}


__all__ = ["MiniMaxH3Application"]
