"""LTX-2 decoders: causal video VAE decoder, audio VAE decoder and vocoder.

Shape contract of the reference's LTX-2 pipeline (difflet/models/ltx_2/pipeline.py:
144-247): a video latent [B, 128, 1 + (F - 1) / 8, H / 32, W / 32] decodes to F
frames (causal first frame, temporal 8x, spatial 32x); an audio latent
[B, 8, T, 16] (25 latent frames per second) decodes to a stereo mel spectrogram
[B, 2, 4T, 64] and the vocoder turns it into a 16 kHz waveform (hop 160).

Video decoder: causal Conv3d stem, residual blocks (RMS norm + SiLU), three
depth-to-space upsamplers (2 x 2 x 2 each; the causal frame dropped after each
time doubling: f -> 2f - 1), an output convolution to 3 x 4 x 4 channels and a
final 4 x 4 unpatchify.  Audio decoder: 2-D convolutions with two 2 x 2
nearest upsamplings.  Vocoder: HiFi-GAN-style transposed-convolution upsampling
(5, 4, 2, 2, 2 = 160) with dilated residual blocks and a tanh output.
Convolutions run through cuDNN here (weights are random-init: no LTX-2 decoder
checkpoint is available offline).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as TF


@dataclass(frozen=True)
class LTX2DecoderConfig:
    latent_channels: int = 128
    channels: tuple = (512, 256, 128)   # per upsampling stage
    res_blocks: int = 2
    patch: int = 4
    audio_latent_channels: int = 8
    audio_channels: tuple = (256, 128)
    mel_bins: int = 64
    stereo: int = 2
    voc_channels: int = 256
    voc_rates: tuple = (5, 4, 2, 2, 2)
    sample_rate: int = 16000


TINY_DECODER = LTX2DecoderConfig(latent_channels=32, channels=(32, 16, 16), res_blocks=1, audio_latent_channels=2,
                                 audio_channels=(16, 16), voc_channels=16)


def _conv_shapes(cfg: LTX2DecoderConfig) -> dict:
    s = {}
    C = cfg.channels
    s["v.in.w"], s["v.in.b"] = (C[0], cfg.latent_channels, 3, 3, 3), (C[0],)
    for i, c in enumerate(C):
        for r in range(cfg.res_blocks):
            p = f"v.s{i}.r{r}."
            s[p + "n1"], s[p + "n2"] = (c,), (c,)
            s[p + "c1.w"], s[p + "c1.b"] = (c, c, 3, 3, 3), (c,)
            s[p + "c2.w"], s[p + "c2.b"] = (c, c, 3, 3, 3), (c,)
        nxt = C[i + 1] if i + 1 < len(C) else C[-1]
        s[f"v.up{i}.w"], s[f"v.up{i}.b"] = (nxt * 8, c, 3, 3, 3), (nxt * 8,)
    s["v.norm"] = (C[-1],)
    s["v.out.w"], s["v.out.b"] = (3 * cfg.patch * cfg.patch, C[-1], 3, 3, 3), (3 * cfg.patch * cfg.patch,)
    A = cfg.audio_channels
    s["a.in.w"], s["a.in.b"] = (A[0], cfg.audio_latent_channels, 3, 3), (A[0],)
    for i, c in enumerate(A):
        nxt = A[i + 1] if i + 1 < len(A) else A[-1]
        s[f"a.c{i}.w"], s[f"a.c{i}.b"] = (nxt, c, 3, 3), (nxt,)
    s["a.out.w"], s["a.out.b"] = (cfg.stereo, A[-1], 3, 3), (cfg.stereo,)
    V = cfg.voc_channels
    s["voc.pre.w"], s["voc.pre.b"] = (V, cfg.stereo * cfg.mel_bins, 7), (V,)
    c = V
    for i, r in enumerate(cfg.voc_rates):
        co = max(c // 2, 8)
        s[f"voc.up{i}.w"], s[f"voc.up{i}.b"] = (c, co, 2 * r), (co,)
        for d in range(2):
            s[f"voc.rb{i}.{d}.w"], s[f"voc.rb{i}.{d}.b"] = (co, co, 3), (co,)
        c = co
    s["voc.post.w"], s["voc.post.b"] = (cfg.stereo, c, 7), (cfg.stereo,)
    return s


class LTX2Decoders:
    def __init__(self, cfg: LTX2DecoderConfig, weights: dict):
        self.cfg, self.w = cfg, weights

    @classmethod
    def random_init(cls, cfg: LTX2DecoderConfig = LTX2DecoderConfig(), *, device="cpu", dtype=torch.float32, seed=0):
        g = torch.Generator().manual_seed(seed)
        w = {}
        for k, shp in _conv_shapes(cfg).items():
            if len(shp) == 1 and not k.endswith(".b"):
                t = torch.ones(shp)
            elif k.endswith(".b"):
                t = torch.zeros(shp)
            else:
                fan_in = shp[1] * int(torch.tensor(shp[2:]).prod())
                t = torch.randn(shp, generator=g) / fan_in ** 0.5
            w[k] = t.to(device=device, dtype=dtype)
        return cls(cfg, w)

    # ------------------------------------------------------------------ video
    def _cconv(self, x, name):
        """Causal 3x3x3 convolution: two replicated leading frames, zero spatial padding."""
        x = torch.cat([x[:, :, :1], x[:, :, :1], x], 2)
        return TF.conv3d(x, self.w[name + ".w"], self.w[name + ".b"], padding=(0, 1, 1))

    @staticmethod
    def _rms(x, g):
        return x * torch.rsqrt(x.float().pow(2).mean(1, keepdim=True) + 1e-6).to(x.dtype) * g.view(1, -1, 1, 1, 1)

    def decode_video(self, z: torch.Tensor) -> torch.Tensor:
        """[B, C, f, h, w] latent -> [B, 3, 8(f-1)+1, 32h, 32w] in [-1, 1]."""
        cfg = self.cfg
        x = self._cconv(z, "v.in")
        for i, c in enumerate(cfg.channels):
            for r in range(cfg.res_blocks):
                p = f"v.s{i}.r{r}."
                h = self._cconv(TF.silu(self._rms(x, self.w[p + "n1"])), p + "c1")
                h = self._cconv(TF.silu(self._rms(h, self.w[p + "n2"])), p + "c2")
                x = x + h
            y = self._cconv(x, f"v.up{i}")  # [B, 8c', f, h, w] -> depth to space (2, 2, 2)
            B, C8, f, hh, ww = y.shape
            c2 = C8 // 8
            y = y.view(B, c2, 2, 2, 2, f, hh, ww).permute(0, 1, 5, 2, 6, 3, 7, 4).reshape(B, c2, 2 * f, 2 * hh, 2 * ww)
            x = y[:, :, 1:]  # causal: the first frame of the doubled sequence is dropped
        x = self._cconv(TF.silu(self._rms(x, self.w["v.norm"])), "v.out")
        B, _, f, hh, ww = x.shape
        P = cfg.patch
        x = x.view(B, 3, P, P, f, hh, ww).permute(0, 1, 4, 5, 2, 6, 3).reshape(B, 3, f, hh * P, ww * P)
        return x.clamp(-1, 1)

    # ------------------------------------------------------------------ audio
    def decode_mel(self, z: torch.Tensor) -> torch.Tensor:
        """[B, 8, T, 16] audio latent -> mel [B, stereo, 4T, 64]."""
        x = TF.conv2d(z, self.w["a.in.w"], self.w["a.in.b"], padding=1)
        for i in range(len(self.cfg.audio_channels)):
            x = TF.interpolate(TF.silu(x), scale_factor=2, mode="nearest")
            x = TF.conv2d(x, self.w[f"a.c{i}.w"], self.w[f"a.c{i}.b"], padding=1)
        return TF.conv2d(TF.silu(x), self.w["a.out.w"], self.w["a.out.b"], padding=1)

    def vocode(self, mel: torch.Tensor) -> torch.Tensor:
        """mel [B, stereo, frames, 64] -> waveform [B, stereo, frames * 160] in [-1, 1]."""
        B, S, T, M = mel.shape
        x = TF.conv1d(mel.permute(0, 1, 3, 2).reshape(B, S * M, T), self.w["voc.pre.w"], self.w["voc.pre.b"],
                      padding=3)
        for i, r in enumerate(self.cfg.voc_rates):
            x = TF.conv_transpose1d(TF.leaky_relu(x, 0.1), self.w[f"voc.up{i}.w"], self.w[f"voc.up{i}.b"], stride=r,
                                    padding=r // 2 + r % 2, output_padding=r % 2)
            for d in range(2):
                h = TF.conv1d(TF.leaky_relu(x, 0.1), self.w[f"voc.rb{i}.{d}.w"], self.w[f"voc.rb{i}.{d}.b"],
                              padding=3 ** d, dilation=3 ** d)
                x = x + h
        x = TF.conv1d(TF.leaky_relu(x, 0.1), self.w["voc.post.w"], self.w["voc.post.b"], padding=3)
        return torch.tanh(x)[..., : T * 160]


__all__ = ["LTX2DecoderConfig", "LTX2Decoders", "TINY_DECODER"]
