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
Weights use the diffusers names.

``WanVAEDecoder`` (the engine's decoder) runs channels-last on the native kernels: every
convolution is the tcgen05 implicit GEMM (``csrc/conv.cu``) reading a per-convolution input
buffer that holds the two cached frames followed by the new ones (a valid convolution in time,
no concatenation copies), the channel RMS norm + SiLU and the nearest upsampler are
``csrc/vae.cu``.  Across GPUs each rank decodes a slab of rows (``parallel/slabs.py``): the
producer of every 3x3 convolution's input stores its boundary rows into the neighbouring ranks'
halo rows over NVLink, the mid-block attention all-gathers K / V, and rank 0 assembles the video.
``WanVAEReference`` is the plain NCTHW PyTorch decoder, kept as the oracle.
"""

from __future__ import annotations

from dataclasses import dataclass

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


def random_weights(cfg: WanVAEConfig, *, device="cpu", dtype=torch.float32, seed=0) -> dict:
    """Seeded weights: fan-in scaled normal convolutions; norm gains 1 + N(0, 0.1); biases N(0, 0.02)."""
    g = torch.Generator(device=device).manual_seed(seed)
    w = {}
    for n, shape in weight_shapes(cfg).items():
        if n.endswith("gamma"):
            w[n] = (1.0 + 0.1 * torch.randn(shape, generator=g, device=device)).to(dtype)
        elif n.endswith("bias"):
            w[n] = (0.02 * torch.randn(shape, generator=g, device=device)).to(dtype)
        else:
            fan_in = 1
            for d in shape[1:]:
                fan_in *= d
            w[n] = (torch.randn(shape, generator=g, device=device) * fan_in ** -0.5).to(dtype)
    return w


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


class WanVAEReference:
    """Plain NCTHW PyTorch decoder (the numerical oracle of ``WanVAEDecoder``)."""

    def __init__(self, cfg: WanVAEConfig, weights: dict):
        self.cfg = cfg
        self.w = weights
        self.convs = {}

    @classmethod
    def random_init(cls, cfg: WanVAEConfig = WanVAEConfig(), *, device="cpu", dtype=torch.float32, seed=0):
        return cls(cfg, random_weights(cfg, device=device, dtype=dtype, seed=seed))

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


# ------------------------------------------------------------------------------------------------
# Channels-last native decoder
# ------------------------------------------------------------------------------------------------
def _pad32(n: int) -> int:
    return -(-n // 32) * 32


class _Conv:
    """One convolution: kernel-layout weights (channels padded to multiples of 32 with zeros) and,
    for convolutions that read a spatial or temporal neighbourhood, its input buffer
    ``[2 + T_max, rows + 2 halo, W, C]``: two cached frames, then the frames of the current chunk
    (written there by the producer), halo rows above and below under a slab split."""

    def __init__(self, w, b, dt):
        Co, Ci = w.shape[:2]
        k = tuple(w.shape[2:]) if w.dim() == 5 else (1,) + tuple(w.shape[2:])
        self.kt, self.kh, self.kw = k
        self.Ci, self.Co = _pad32(Ci), _pad32(Co)
        self.co_real = Co
        w5 = torch.zeros((self.Co, self.Ci) + k, device=w.device, dtype=torch.float32)
        w5[:Co, :Ci] = w.float().view((Co, Ci) + k)
        from difflet_b200.ops.fused import conv_weight

        self.w2 = conv_weight(w5.to(dt))
        bb = torch.zeros(self.Co, device=w.device, dtype=torch.float32)
        bb[:Co] = b.float()
        self.b = bb.to(dt)
        self.buf = None

    def ensure_buffer(self, slabs, T_max: int, rows: int, W: int, dt, halo: int):
        shape = (2 + T_max, rows + 2 * halo, W, self.Ci)
        if self.buf is None or tuple(self.buf.shape) != shape:
            self.buf = slabs.empty(shape, dt)
        return self.buf

    def reset(self):
        if self.buf is not None:
            self.buf[:2].zero_()

    def run(self, T: int, *, halo: int, resid=None):
        """Convolve the T frames at buf[2:2+T] (with their cached context) -> [1, T, rows, W, Co]."""
        from difflet_b200.ops import fused as F

        lo = 2 - (self.kt - 1)
        x = self.buf[lo:2 + T][None]
        padded = self.Co != self.co_real
        y = F.conv_cl(x, self.w2, self.b, kt=self.kt, kh=self.kh, kw=self.kw, valid_t=True,
                      valid_h=bool(halo) and self.kh > 1, resid=None if padded else resid)
        if self.kt > 1:  # the last two input frames become the cache of the next chunk
            tail = self.buf[T:T + 2]
            self.buf[:2].copy_(tail.clone() if T < 2 else tail)
        return self._trim(y, resid if padded else None)

    def _trim(self, y, resid=None):
        if self.Co == self.co_real:
            return y
        y = y[..., : self.co_real].contiguous()
        return y if resid is None else y + resid

    def pointwise(self, x, keep_padding: bool = False):
        """A 1x1x1 convolution of a plain [1, T, rows, W, C] tensor."""
        from difflet_b200.ops import fused as F

        if x.shape[-1] != self.Ci:
            x = torch.nn.functional.pad(x, (0, self.Ci - x.shape[-1]))
        y = F.conv_cl(x.contiguous(), self.w2, self.b, kt=1, kh=1, kw=1)
        return y if keep_padding else self._trim(y)


class WanVAEDecoder:
    """Causal Wan VAE decoder on the native kernels, channels-last, streaming one latent frame at a
    time, optionally split into row slabs over the ranks of a process group (``set_slabs``)."""

    def __init__(self, cfg: WanVAEConfig, weights: dict):
        self.cfg = cfg
        self.w = weights
        self._convs = None
        self.slabs = None

    @classmethod
    def random_init(cls, cfg: WanVAEConfig = WanVAEConfig(), *, device="cpu", dtype=torch.float32, seed=0):
        return cls(cfg, random_weights(cfg, device=device, dtype=dtype, seed=seed))

    @property
    def distributed(self) -> bool:
        return self.slabs is not None and self.slabs.world > 1

    def set_slabs(self, slabs) -> None:
        """Decode spatial row slabs over ``slabs`` (``parallel.slabs.make_slabs``)."""
        self.slabs = slabs
        self._convs = None

    def _prepare(self):
        if self._convs is None:
            dt = self.w["decoder.conv_in.weight"].dtype
            self._convs = {n[: -len(".weight")]: _Conv(self.w[n], self.w[n[: -len("weight")] + "bias"], dt)
                           for n in self.w if n.endswith(".weight") and self.w[n].dim() >= 4}
        return self._convs

    # -------------------------------------------------------------------------------- pieces
    def _gamma(self, name):
        return self.w[name].reshape(-1)

    def _fill(self, conv: _Conv, x, T, *, norm=None, silu=True, upsample=False):
        """Write the convolution's input frames (norm + SiLU of x, the upsampled x, or x itself)
        into its buffer, with halo rows to / from the neighbouring slabs."""
        from difflet_b200.ops import fused as F

        sl = self.slabs
        halo = sl.halo if conv.kh > 1 else 0
        rows = x.shape[2] * (2 if upsample else 1)
        W = x.shape[3] * (2 if upsample else 1)
        buf = conv.ensure_buffer(sl, self._t_max(rows), rows, W, x.dtype, halo)
        dst = buf[2:2 + T]
        x4 = x[0].contiguous()
        if x4.shape[-1] != conv.Ci:
            # channel-padded input (narrow test decoders only; the released Wan widths are all
            # multiples of 32): produce the real channels, then copy them into the padded buffer
            if getattr(sl, "heap", None) is not None:
                raise NotImplementedError("peer-memory slabs need channel counts that are multiples of 32")
            tmp = torch.zeros(T, rows + 2 * halo, W, x4.shape[-1], device=x4.device, dtype=x4.dtype)
            if norm is not None:
                F.vae_chan_norm(x4, self._gamma(norm), tmp, silu=silu, halo=halo)
            elif upsample:
                F.vae_upsample2x(x4, tmp, halo=halo)
            else:
                tmp[:, halo:halo + rows].copy_(x4)
            dst[..., : x4.shape[-1]].copy_(tmp)
        else:
            nb = sl.neighbours(buf, 2, rows) if halo else {}
            if norm is not None:
                F.vae_chan_norm(x4, self._gamma(norm), dst, silu=silu, halo=halo, **nb)
            elif upsample:
                F.vae_upsample2x(x4, dst, halo=halo, **nb)
            else:
                dst[:, halo:halo + rows].copy_(x4)
        if halo:
            sl.sync(buf, slice(2, 2 + T), rows)
        return halo

    def _t_max(self, rows: int) -> int:
        # frames per chunk at a resolution: 1 at the latent size, doubled by each temporal upsampler
        scale = max(1, rows // max(1, self._rows_latent))
        return {1: 1, 2: 2, 4: 4, 8: 4}.get(scale, 4)

    def _conv(self, name, x, T, resid=None, **fill):
        conv = self._convs[name]
        halo = self._fill(conv, x, T, **fill)
        return conv.run(T, halo=halo, resid=resid)

    def _res(self, x, n, T):
        sc = n + ".conv_shortcut"
        h = self._convs[sc].pointwise(x) if sc in self._convs else x
        y = self._conv(n + ".conv1", x, T, norm=n + ".norm1.gamma")
        return self._conv(n + ".conv2", y, T, resid=h, norm=n + ".norm2.gamma")

    def _attn(self, x, n, T):
        """Per-frame single-head spatial attention (mid block); K / V of every slab."""
        from difflet_b200.ops import fused as F

        _, T_, rows, W, C = x.shape
        nrm = torch.empty(T, rows, W, C, device=x.device, dtype=x.dtype)
        F.vae_chan_norm(x[0].contiguous(), self._gamma(n + ".norm.gamma"), nrm, silu=False)
        wq = self.w[n + ".to_qkv.weight"].reshape(3 * C, C)
        qkv = F.linear(nrm.reshape(-1, C), wq, self.w[n + ".to_qkv.bias"]).view(T, rows, W, 3, C)
        q, k, v = qkv[..., 0, :], qkv[..., 1, :], qkv[..., 2, :]
        rows_full = self.slabs.rows * (rows // max(1, self.slabs.local_rows()))
        k = self.slabs.gather_rows(k.contiguous(), rows_full)
        v = self.slabs.gather_rows(v.contiguous(), rows_full)
        ct = q.dtype
        o = torch.nn.functional.scaled_dot_product_attention(q.reshape(T, 1, -1, C), k.reshape(T, 1, -1, C).to(ct),
                                                             v.reshape(T, 1, -1, C).to(ct))
        wp = self.w[n + ".proj.weight"].reshape(C, C)
        y = F.linear(o.reshape(-1, C), wp, self.w[n + ".proj.bias"])
        return x + y.view(1, T, rows, W, C)

    def _resample(self, x, u, mode, first, T):
        if mode == "upsample3d":
            tc = self._convs[u + ".time_conv"]
            _, _, rows, W, C = x.shape
            buf = tc.ensure_buffer(self.slabs, self._t_max(rows), rows, W, x.dtype, 0)
            if first:  # no time convolution; the cache becomes the two frames ending with x
                buf[:2].zero_()
                buf[2 - min(2, T):2].copy_(x[0, -min(2, T):])
            else:
                buf[2:2 + T].copy_(x[0])
                y = tc.run(T, halo=0)  # [1, T, rows, W, 2C]
                x = y.view(1, T, rows, W, 2, C).permute(0, 1, 4, 2, 3, 5).reshape(1, 2 * T, rows, W, C)
                T = 2 * T
        y = self._conv(u + ".resample.1", x, T, upsample=True)
        return y, T

    def _chunk(self, z_slab, first: bool):
        """One latent frame: z_slab [1, 1, rows + 2 halo, w, 16] (halo rows from the full latent,
        zero outside the picture) -> frames [T, 8 rows, 8 w, 3]."""
        cv = self._convs
        sl = self.slabs
        halo = sl.halo
        rows = z_slab.shape[2] - 2 * halo
        # post_quant_conv (pointwise) straight into conv_in's input buffer, halo rows included
        zc = torch.nn.functional.pad(z_slab, (0, cv["post_quant_conv"].Ci - z_slab.shape[-1]))
        ci = cv["decoder.conv_in"]
        buf = ci.ensure_buffer(sl, 1, rows, z_slab.shape[3], z_slab.dtype, halo)
        pq = cv["post_quant_conv"].pointwise(zc, keep_padding=True)  # [1, 1, rows + 2 halo, w, 32]
        buf[2:3].copy_(pq[0])
        if halo:  # rows outside the picture stay zero (the convolution's zero padding)
            if sl.rank == 0:
                buf[2:3, 0].zero_()
            if sl.rank == sl.world - 1:
                buf[2:3, rows + 1].zero_()
        x = ci.run(1, halo=halo)
        T = 1
        x = self._res(x, "decoder.mid_block.resnets.0", T)
        x = self._attn(x, "decoder.mid_block.attentions.0", T)
        x = self._res(x, "decoder.mid_block.resnets.1", T)
        for i, (_, _, mode) in enumerate(_block_plan(self.cfg)):
            for j in range(self.cfg.num_res_blocks + 1):
                x = self._res(x, f"decoder.up_blocks.{i}.resnets.{j}", T)
            if mode is not None:
                x, T = self._resample(x, f"decoder.up_blocks.{i}.upsamplers.0", mode, first, T)
        y = self._conv("decoder.conv_out", x, T, norm="decoder.norm_out.gamma")
        return y[0].clamp_(-1, 1)

    # -------------------------------------------------------------------------------- decode
    @torch.no_grad()
    def decode_frames(self, z: torch.Tensor, frame_callback=None):
        """z [1, 16, T, h, w] normalised latents -> this rank's rows of every frame,
        [1 + 4 (T - 1), 8 rows, 8 w, 3] channels-last in [-1, 1]."""
        cfg = self.cfg
        if z.shape[0] != 1:
            raise ValueError("the streaming decoder takes one video at a time")
        self._prepare()
        if self.slabs is None:
            from difflet_b200.parallel.slabs import LocalSlabs

            self.slabs = LocalSlabs(z.shape[3], z.device)
        sl = self.slabs
        self._rows_latent = sl.local_rows()
        dt = self.w["decoder.conv_in.weight"].dtype
        mean = torch.tensor(cfg.latents_mean, device=z.device, dtype=torch.float32)
        std = torch.tensor(cfg.latents_std, device=z.device, dtype=torch.float32)
        zl = (z[0].float().permute(1, 2, 3, 0) * std + mean).to(dt)  # [T, h, w, 16]
        r0, r1 = sl.bounds(sl.rank)
        halo = sl.halo
        lo, hi = max(0, r0 - halo), min(zl.shape[1], r1 + halo)
        slab = torch.zeros(zl.shape[0], (r1 - r0) + 2 * halo, zl.shape[2], zl.shape[3], device=z.device, dtype=dt)
        slab[:, lo - (r0 - halo):hi - (r0 - halo)] = zl[:, lo:hi]
        for c in self._convs.values():
            c.reset()
        outs = []
        for t in range(zl.shape[0]):
            y = self._chunk(slab[t:t + 1][None], first=(t == 0))
            if frame_callback is not None:
                frame_callback(y)
            else:
                outs.append(y)
        for c in self._convs.values():
            c.reset()
        return torch.cat(outs, 0) if outs else None

    @torch.no_grad()
    def decode(self, z: torch.Tensor, frame_callback=None, channels_last: bool = False):
        """z [1, 16, T, h, w] -> video [1, 3, F, H, W] in [-1, 1] (``channels_last``: [1, F, H, W, 3]);
        under a slab split rank 0 returns the whole video, the other ranks None.  A batch of
        latents decodes one video after the other."""
        if z.shape[0] > 1:
            vids = [self.decode(z[b:b + 1], frame_callback, channels_last) for b in range(z.shape[0])]
            return None if vids[0] is None else torch.cat(vids, 0)
        frames = self.decode_frames(z, frame_callback)
        if frames is None:
            return None
        video = self.slabs.gather_video(frames, 8 * z.shape[3]) if self.distributed else frames
        if video is None:
            return None
        video = video[None]
        return video if channels_last else video.permute(0, 4, 1, 2, 3)
