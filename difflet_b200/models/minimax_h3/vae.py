"""MiniMax-H3 decoders with the release's shape contract (difflet/models/minimax_h3/
pipeline.py:514-680, modeling_vae.py): video latents [1, 24, 5n + 2, H/16, W/16] decode
to 17n + 5 frames at H x W (16x spatial, four 2x depth-to-space stages; time resampled
to the requested frame count), audio latents [2, 32, T] (40 per second) to a stereo
24 kHz waveform through a BigVGAN-style stack (transposed-conv upsampling 5 x 5 x 4 x 3 x 2
= 600 samples per latent, snake activations).  Random-init weights: no decoder
checkpoint is available offline; convolutions run through cuDNN."""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as TF


@dataclass(frozen=True)
class MiniMaxDecoderConfig:
    latent_channels: int = 24
    channels: tuple = (256, 128, 64, 32)
    audio_latent_channels: int = 32
    voc_channels: int = 256
    voc_rates: tuple = (5, 5, 4, 3, 2)
    sample_rate: int = 24000


TINY = MiniMaxDecoderConfig(latent_channels=4, channels=(16, 16, 8, 8), audio_latent_channels=8, voc_channels=16)


def _shapes(cfg):
    s = {"v.in.w": (cfg.channels[0], cfg.latent_channels, 3, 3, 3), "v.in.b": (cfg.channels[0],)}
    for i, c in enumerate(cfg.channels):
        nxt = cfg.channels[i + 1] if i + 1 < len(cfg.channels) else cfg.channels[-1]
        s[f"v.c{i}.w"], s[f"v.c{i}.b"] = (c, c, 3, 3, 3), (c,)
        s[f"v.up{i}.w"], s[f"v.up{i}.b"] = (nxt * 4, c, 1, 3, 3), (nxt * 4,)
    s["v.out.w"], s["v.out.b"] = (3, cfg.channels[-1], 1, 3, 3), (3,)
    V = cfg.voc_channels
    s["a.pre.w"], s["a.pre.b"] = (V, cfg.audio_latent_channels, 7), (V,)
    c = V
    for i, r in enumerate(cfg.voc_rates):
        co = max(c // 2, 8)
        s[f"a.up{i}.w"], s[f"a.up{i}.b"] = (c, co, 2 * r), (co,)
        s[f"a.alpha{i}"] = (co,)
        s[f"a.rb{i}.w"], s[f"a.rb{i}.b"] = (co, co, 3), (co,)
        c = co
    s["a.post.w"], s["a.post.b"] = (1, c, 7), (1,)
    return s


class MiniMaxDecoders:
    def __init__(self, cfg: MiniMaxDecoderConfig, w: dict):
        self.cfg, self.w = cfg, w

    @classmethod
    def random_init(cls, cfg=MiniMaxDecoderConfig(), *, device="cpu", dtype=torch.float32, seed=0):
        g = torch.Generator().manual_seed(seed)
        w = {}
        for k, shp in _shapes(cfg).items():
            if k.endswith(".b"):
                t = torch.zeros(shp)
            elif ".alpha" in k:
                t = torch.ones(shp)
            else:
                fan = shp[1] * int(torch.tensor(shp[2:]).prod())
                t = torch.randn(shp, generator=g) / fan ** 0.5
            w[k] = t.to(device=device, dtype=dtype)
        return cls(cfg, w)

    def decode_video(self, z: torch.Tensor, num_frames: int) -> torch.Tensor:
        """[1, C, nf, h, w] -> [1, 3, num_frames, 16 h, 16 w] in [-1, 1]."""
        x = TF.conv3d(z, self.w["v.in.w"], self.w["v.in.b"], padding=1)
        for i in range(len(self.cfg.channels)):
            x = x + TF.conv3d(TF.silu(x), self.w[f"v.c{i}.w"], self.w[f"v.c{i}.b"], padding=1)
            y = TF.conv3d(TF.silu(x), self.w[f"v.up{i}.w"], self.w[f"v.up{i}.b"], padding=(0, 1, 1))
            B, C4, f, h, w = y.shape
            c = C4 // 4
            x = y.view(B, c, 2, 2, f, h, w).permute(0, 1, 4, 5, 2, 6, 3).reshape(B, c, f, 2 * h, 2 * w)
        x = TF.conv3d(TF.silu(x), self.w["v.out.w"], self.w["v.out.b"], padding=(0, 1, 1))
        x = TF.interpolate(x, size=(num_frames, x.shape[-2], x.shape[-1]), mode="trilinear", align_corners=True)
        return torch.tanh(x)

    def decode_audio(self, z: torch.Tensor) -> torch.Tensor:
        """[channels, C, T] -> waveform [channels, 600 T] in [-1, 1]."""
        x = TF.conv1d(z, self.w["a.pre.w"], self.w["a.pre.b"], padding=3)
        for i, r in enumerate(self.cfg.voc_rates):
            x = TF.conv_transpose1d(x, self.w[f"a.up{i}.w"], self.w[f"a.up{i}.b"], stride=r,
                                    padding=r // 2 + r % 2, output_padding=r % 2)
            a = self.w[f"a.alpha{i}"].view(1, -1, 1)
            snake = x + torch.sin(a * x).pow(2) / (a + 1e-9)
            x = x + TF.conv1d(snake, self.w[f"a.rb{i}.w"], self.w[f"a.rb{i}.b"], padding=1)
        return torch.tanh(TF.conv1d(x, self.w["a.post.w"], self.w["a.post.b"], padding=3))[:, 0]


__all__ = ["MiniMaxDecoderConfig", "MiniMaxDecoders", "TINY"]
