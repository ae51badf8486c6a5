"""2-D KL autoencoder decoder (FLUX.1: 16 latent channels, 8x spatial).

Architecture of diffusers' ``AutoencoderKL`` decoder as used by the reference
FLUX pipeline (``difflet/models/flux/vae/modeling_vae.py:39-141``): conv_in ->
mid (resnet, single-head spatial attention, resnet) -> 4 up blocks of 3 resnets
(nearest x2 upsample + conv after the first three) -> GroupNorm(32) + SiLU ->
conv_out.  Weights use the diffusers names, so a real checkpoint loads
unchanged; ``random_init`` builds seeded weights for offline benchmarks.
Latents are de-normalised as ``z / scaling_factor + shift_factor``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class KLDecoderConfig:
    latent_channels: int = 16
    block_out_channels: tuple = (128, 256, 512, 512)
    layers_per_block: int = 2
    norm_groups: int = 32
    scaling_factor: float = 0.3611
    shift_factor: float = 0.1159


def _shapes(cfg: KLDecoderConfig) -> dict[str, tuple]:
    ch = list(reversed(cfg.block_out_channels))
    s = {}

    def conv(name, cin, cout, k=3):
        s[name + ".weight"] = (cout, cin, k, k)
        s[name + ".bias"] = (cout,)

    def norm(name, c):
        s[name + ".weight"] = (c,)
        s[name + ".bias"] = (c,)

    def resnet(name, cin, cout):
        norm(name + ".norm1", cin)
        conv(name + ".conv1", cin, cout)
        norm(name + ".norm2", cout)
        conv(name + ".conv2", cout, cout)
        if cin != cout:
            conv(name + ".conv_shortcut", cin, cout, 1)

    conv("decoder.conv_in", cfg.latent_channels, ch[0])
    resnet("decoder.mid_block.resnets.0", ch[0], ch[0])
    a = "decoder.mid_block.attentions.0"
    norm(a + ".group_norm", ch[0])
    for n in ("to_q", "to_k", "to_v", "to_out.0"):
        s[f"{a}.{n}.weight"] = (ch[0], ch[0])
        s[f"{a}.{n}.bias"] = (ch[0],)
    resnet("decoder.mid_block.resnets.1", ch[0], ch[0])
    prev = ch[0]
    for i, c in enumerate(ch):
        for j in range(cfg.layers_per_block + 1):
            resnet(f"decoder.up_blocks.{i}.resnets.{j}", prev if j == 0 else c, c)
        prev = c
        if i < len(ch) - 1:
            conv(f"decoder.up_blocks.{i}.upsamplers.0.conv", c, c)
    norm("decoder.conv_norm_out", ch[-1])
    conv("decoder.conv_out", ch[-1], 3)
    return s


class KLDecoder:
    def __init__(self, cfg: KLDecoderConfig, weights: dict[str, torch.Tensor]):
        self.cfg = cfg
        self.w = weights

    @classmethod
    def random_init(cls, cfg: KLDecoderConfig = KLDecoderConfig(), *, device="cpu", dtype=torch.float32, seed=0):
        g = torch.Generator(device=device).manual_seed(seed)
        w = {}
        for name, shape in _shapes(cfg).items():
            if name.endswith("bias"):
                t = torch.zeros(shape, device=device, dtype=dtype)
            elif len(shape) == 1:  # norm gain
                t = torch.ones(shape, device=device, dtype=dtype)
            else:
                fan_in = 1
                for d in shape[1:]:
                    fan_in *= d
                t = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * (1.0 / fan_in) ** 0.5
                t = t.to(dtype)
            w[name] = t
        return cls(cfg, w)

    def _gn(self, x, name, silu):
        x = F.group_norm(x, self.cfg.norm_groups, self.w[name + ".weight"], self.w[name + ".bias"], eps=1e-6)
        return F.silu(x) if silu else x

    def _native_ok(self, x, name):
        w = self.w[name + ".weight"]
        return (x.is_cuda and x.dtype == torch.bfloat16 and x.shape[1] % 32 == 0 and w.shape[0] % 32 == 0
                and w.shape[-1] in (1, 3))

    def _conv(self, x, name, pad=1, resid=None):
        """Conv2d (+ residual).  bf16 CUDA tensors with 32-multiple channel counts run the
        tcgen05 implicit-GEMM kernel on channels-last data; the rest goes to cuDNN."""
        if self._native_ok(x, name):
            from difflet_b200.ops import fused as FO

            key = name + ".cl"
            if key not in self.w:
                self.w[key] = FO.conv_weight(self.w[name + ".weight"])
            k = self.w[name + ".weight"].shape[-1]
            xc = x.permute(0, 2, 3, 1).contiguous()[:, None]  # [N, 1, H, W, C]
            rc = None if resid is None else resid.permute(0, 2, 3, 1).contiguous()[:, None]
            y = FO.conv_cl(xc, self.w[key], self.w[name + ".bias"], kt=1, kh=k, kw=k, resid=rc)
            return y[:, 0].permute(0, 3, 1, 2)  # NCHW view of channels-last data
        y = F.conv2d(x, self.w[name + ".weight"], self.w[name + ".bias"], padding=pad)
        return y if resid is None else resid + y

    def _resnet(self, x, name):
        h = self._conv(self._gn(x, name + ".norm1", True), name + ".conv1")
        if name + ".conv_shortcut.weight" in self.w:
            x = self._conv(x, name + ".conv_shortcut", pad=0)
        # the residual add is fused into the second convolution's epilogue
        return self._conv(self._gn(h, name + ".norm2", True), name + ".conv2", resid=x)

    def _attn(self, x, name):
        B, C, H, W = x.shape
        h = self._gn(x, name + ".group_norm", False).view(B, C, H * W).transpose(1, 2)
        lin = lambda t, n: F.linear(t, self.w[f"{name}.{n}.weight"], self.w[f"{name}.{n}.bias"])  # noqa: E731
        q, k, v = (lin(h, n)[:, None] for n in ("to_q", "to_k", "to_v"))
        o = F.scaled_dot_product_attention(q, k, v)[:, 0]
        o = lin(o, "to_out.0").transpose(1, 2).view(B, C, H, W)
        return x + o

    @torch.no_grad()
    def decode(self, z: torch.Tensor) -> torch.Tensor:
        """z [B, C, h, w] (normalised latents) -> image [B, 3, 8h, 8w] in [-1, 1]."""
        cfg = self.cfg
        dt = self.w["decoder.conv_in.weight"].dtype
        x = (z / cfg.scaling_factor + cfg.shift_factor).to(dt)
        x = self._conv(x, "decoder.conv_in")
        x = self._resnet(x, "decoder.mid_block.resnets.0")
        x = self._attn(x, "decoder.mid_block.attentions.0")
        x = self._resnet(x, "decoder.mid_block.resnets.1")
        n_up = len(cfg.block_out_channels)
        for i in range(n_up):
            for j in range(cfg.layers_per_block + 1):
                x = self._resnet(x, f"decoder.up_blocks.{i}.resnets.{j}")
            if i < n_up - 1:
                x = F.interpolate(x, scale_factor=2.0, mode="nearest")
                x = self._conv(x, f"decoder.up_blocks.{i}.upsamplers.0.conv")
        x = self._gn(x, "decoder.conv_norm_out", True)
        x = self._conv(x, "decoder.conv_out")
        return x.clamp(-1, 1)


def to_uint8(img: torch.Tensor) -> torch.Tensor:
    """[B, 3, H, W] in [-1, 1] -> [B, H, W, 3] uint8 (on the same device)."""
    return ((img.float() * 0.5 + 0.5).clamp(0, 1) * 255).round().to(torch.uint8).permute(0, 2, 3, 1).contiguous()
