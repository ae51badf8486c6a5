"""Causal 3-D VAE decoder of Wan 2.1 / 2.2 (16 latent channels, 4x temporal, 8x spatial).

Architecture of diffusers' ``AutoencoderKLWan`` decoder as decoded by the
reference (``difflet/models/wan/vae/modeling_vae.py:92-551``): causal Conv3d
(time padded only on the past side), channel RMS norms, residual blocks, a
per-frame single-head spatial attention in the mid block, and up blocks whose
resamplers double the spatial size (nearest + Conv2d halving the channels) and,
for ``upsample3d``, the frame count (a causal (3,1,1) conv producing two frames
per input frame; skipped for the very first latent frame, which maps to one
output frame).

Streaming decode: latent frames go through the decoder one at a time; every
causal conv keeps the last two frames of its input as state (the reference's
``CACHE_T = 2`` feature cache), so memory stays bounded at 720p x 81 frames.
Weights use the diffusers names.  Convolutions run through cuDNN here; the
denormalisation is fused into the first conv's input.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as Fn

WAN_LATENTS_MEAN = [-0.7571, -0.7089, -0.9113, 0.1075, -0.1745, 0.9653, -0.1517, 1.5508, 0.4134, -0.0715,
                    0.5517, -0.3632, -0.1922, -0.9497, 0.2503, -0.2921]
WAN_LATENTS_STD = [2.8184, 1.4541, 2.3275, 2.6558, 1.2196, 1.7708, 2.6052, 2.0743, 3.2687, 2.1526, 2.8652,
                   1.5579, 1.6382, 1.1253, 2.8251, 1.9160]


@dataclass(frozen=True)
class WanVAEConfig:
    base_dim: int = 96
    z_dim: int = 16
    dim_mult: tuple = (1, 2, 4, 4)
    num_res_blocks: int = 2
    temperal_downsample: tuple = (False, True, True)
    latents_mean: tuple = tuple(WAN_LATENTS_MEAN)
    latents_std: tuple = tuple(WAN_LATENTS_STD)

    @property
    def dims(self):
        m = list(self.dim_mult)
        return [d * self.base_dim for d in [m[-1]] + m[::-1]]

    @property
    def temperal_upsample(self):
        return list(self.temperal_downsample)[::-1]


def _block_plan(cfg: WanVAEConfig):
    """[(in_dim, out_dim, upsample_mode)] for each up block."""
    dims = cfg.dims
    plan = []
    for i, (din, dout) in enumerate(zip(dims[:-1], dims[1:])):
        if i > 0:
            din = din // 2
        up = i != len(cfg.dim_mult) - 1
        mode = ("upsample3d" if cfg.temperal_upsample[i] else "upsample2d") if up else None
        plan.append((din, dout, mode))
    return plan


def weight_shapes(cfg: WanVAEConfig) -> dict:
    s = {}

    def conv3(n, ci, co, k=(3, 3, 3)):
        s[n + ".weight"] = (co, ci) + tuple(k)
        s[n + ".bias"] = (co,)

    def res(n, ci, co):
        s[n + ".norm1.gamma"] = (ci, 1, 1, 1)
        conv3(n + ".conv1", ci, co)
        s[n + ".norm2.gamma"] = (co, 1, 1, 1)
        conv3(n + ".conv2", co, co)
        if ci != co:
            conv3(n + ".conv_shortcut", ci, co, (1, 1, 1))

    d0 = cfg.dims[0]
    conv3("post_quant_conv", cfg.z_dim, cfg.z_dim, (1, 1, 1))
    conv3("decoder.conv_in", cfg.z_dim, d0)
    res("decoder.mid_block.resnets.0", d0, d0)
    a = "decoder.mid_block.attentions.0"
    s[a + ".norm.gamma"] = (d0, 1, 1)
    s[a + ".to_qkv.weight"], s[a + ".to_qkv.bias"] = (3 * d0, d0, 1, 1), (3 * d0,)
    s[a + ".proj.weight"], s[a + ".proj.bias"] = (d0, d0, 1, 1), (d0,)
    res("decoder.mid_block.resnets.1", d0, d0)
    for i, (din, dout, mode) in enumerate(_block_plan(cfg)):
        cur = din
        for j in range(cfg.num_res_blocks + 1):
            res(f"decoder.up_blocks.{i}.resnets.{j}", cur, dout)
            cur = dout
        if mode is not None:
            u = f"decoder.up_blocks.{i}.upsamplers.0"
            s[u + ".resample.1.weight"], s[u + ".resample.1.bias"] = (dout // 2, dout, 3, 3), (dout // 2,)
            if mode == "upsample3d":
                conv3(u + ".time_conv", dout, dout * 2, (3, 1, 1))
    dl = cfg.dims[-1]
    s["decoder.norm_out.gamma"] = (dl, 1, 1, 1)
    conv3("decoder.conv_out", dl, 3)
    return s


class _CausalConv:
    """Conv3d with causal time padding and a rolling 2-frame input cache."""

    def __init__(self, w, b):
        self.w, self.b = w, b
        kt, kh, kw = w.shape[2:]
        self.pt, self.ph, self.pw = kt - 1, kh // 2, kw // 2
        self.cache = None

    def reset(self):
        self.cache = None

    def __call__(self, x):
        if self.pt == 0:
            return Fn.conv3d(x, self.w, self.b, padding=(0, self.ph, self.pw))
        prev = self.cache
        inp = x if prev is None else torch.cat([prev, x], 2)
        need = self.pt - (0 if prev is None else prev.shape[2])
        if need > 0:
            inp = Fn.pad(inp, (0, 0, 0, 0, need, 0))
        tail = torch.cat([prev, x], 2) if prev is not None else x
        self.cache = tail[:, :, -self.pt:].clone()
        return Fn.conv3d(inp, self.w, self.b, padding=(0, self.ph, self.pw))


def _rms(x, gamma):
    # channel-first RMS norm: normalize over C, scale by sqrt(C) * gamma
    return Fn.normalize(x, dim=1) * (x.shape[1] ** 0.5) * gamma


class WanVAEDecoder:
    def __init__(self, cfg: WanVAEConfig, weights: dict):
        self.cfg = cfg
        self.w = weights
        self.convs = {}

    @classmethod
    def random_init(cls, cfg: WanVAEConfig = WanVAEConfig(), *, device="cpu", dtype=torch.float32, seed=0):
        g = torch.Generator(device=device).manual_seed(seed)
        w = {}
        for n, shape in weight_shapes(cfg).items():
            if n.endswith("gamma"):
                w[n] = torch.ones(shape, device=device, dtype=dtype)
            elif n.endswith("bias"):
                w[n] = torch.zeros(shape, device=device, dtype=dtype)
            else:
                fan_in = 1
                for d in shape[1:]:
                    fan_in *= d
                w[n] = (torch.randn(shape, generator=g, device=device) * fan_in ** -0.5).to(dtype)
        return cls(cfg, w)

    def _conv(self, name):
        c = self.convs.get(name)
        if c is None:
            c = self.convs[name] = _CausalConv(self.w[name + ".weight"], self.w[name + ".bias"])
        return c

    def _res(self, x, n):
        h = self._conv(n + ".conv_shortcut")(x) if n + ".conv_shortcut.weight" in self.w else x
        y = self._conv(n + ".conv1")(Fn.silu(_rms(x, self.w[n + ".norm1.gamma"])))
        y = self._conv(n + ".conv2")(Fn.silu(_rms(y, self.w[n + ".norm2.gamma"])))
        return y + h

    def _attn(self, x, n):
        B, C, T, H, W = x.shape
        y = x.permute(0, 2, 1, 3, 4).reshape(B * T, C, H, W)
        y = Fn.normalize(y, dim=1) * (C ** 0.5) * self.w[n + ".norm.gamma"]
        qkv = Fn.conv2d(y, self.w[n + ".to_qkv.weight"], self.w[n + ".to_qkv.bias"])
        q, k, v = qkv.reshape(B * T, 3, C, H * W).permute(1, 0, 3, 2).unbind(0)  # [BT, HW, C]
        o = Fn.scaled_dot_product_attention(q[:, None], k[:, None], v[:, None])[:, 0]
        o = o.permute(0, 2, 1).reshape(B * T, C, H, W)
        o = Fn.conv2d(o, self.w[n + ".proj.weight"], self.w[n + ".proj.bias"])
        return x + o.view(B, T, C, H, W).permute(0, 2, 1, 3, 4)

    def _resample(self, x, u, mode, first):
        B, C, T, H, W = x.shape
        if mode == "upsample3d" and not first:
            y = self._conv(u + ".time_conv")(x)  # [B, 2C, T, H, W]
            x = y.view(B, 2, C, T, H, W).permute(0, 2, 3, 1, 4, 5).reshape(B, C, 2 * T, H, W)
        elif mode == "upsample3d":
            self._conv(u + ".time_conv").cache = x[:, :, -2:].clone() if x.shape[2] >= 2 else \
                torch.cat([torch.zeros_like(x), x], 2)[:, :, -2:].clone()
        T = x.shape[2]
        y = x.permute(0, 2, 1, 3, 4).reshape(B * T, C, H, W)
        y = Fn.interpolate(y, scale_factor=2.0, mode="nearest")
        y = Fn.conv2d(y, self.w[u + ".resample.1.weight"], self.w[u + ".resample.1.bias"], padding=1)
        return y.view(B, T, y.shape[1], 2 * H, 2 * W).permute(0, 2, 1, 3, 4)

    def _decode_chunk(self, z, first):
        x = self._conv("post_quant_conv")(z)
        x = self._conv("decoder.conv_in")(x)
        x = self._res(x, "decoder.mid_block.resnets.0")
        x = self._attn(x, "decoder.mid_block.attentions.0")
        x = self._res(x, "decoder.mid_block.resnets.1")
        for i, (_, _, mode) in enumerate(_block_plan(self.cfg)):
            for j in range(self.cfg.num_res_blocks + 1):
                x = self._res(x, f"decoder.up_blocks.{i}.resnets.{j}")
            if mode is not None:
                x = self._resample(x, f"decoder.up_blocks.{i}.upsamplers.0", mode, first)
        x = Fn.silu(_rms(x, self.w["decoder.norm_out.gamma"]))
        return self._conv("decoder.conv_out")(x)

    @torch.no_grad()
    def decode(self, z: torch.Tensor, frame_callback=None) -> torch.Tensor:
        """z [B, 16, T, h, w] (normalised latents) -> video [B, 3, 1 + 4 (T-1), 8h, 8w] in [-1, 1].
        ``frame_callback(frames)`` receives each decoded chunk (streaming to the host)."""
        cfg = self.cfg
        dt = self.w["decoder.conv_in.weight"].dtype
        mean = torch.tensor(cfg.latents_mean, device=z.device, dtype=torch.float32).view(1, -1, 1, 1, 1)
        std = torch.tensor(cfg.latents_std, device=z.device, dtype=torch.float32).view(1, -1, 1, 1, 1)
        z = (z.float() * std + mean).to(dt)
        for c in self.convs.values():
            c.reset()
        outs = []
        for t in range(z.shape[2]):
            y = self._decode_chunk(z[:, :, t:t + 1], first=(t == 0)).clamp_(-1, 1)
            if frame_callback is not None:
                frame_callback(y)
            else:
                outs.append(y)
        for c in self.convs.values():
            c.reset()
        return torch.cat(outs, 2) if outs else None
