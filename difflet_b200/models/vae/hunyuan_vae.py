"""Causal 3-D VAE decoder of HunyuanVideo (16 latent channels, 4x temporal, 8x spatial).

Architecture of diffusers' ``AutoencoderKLHunyuanVideo`` decoder, which the
reference decodes with fixed tiles and blending
(``difflet/models/hunyuan_video/vae/modeling_vae.py:85-489``,
``difflet/models/hunyuan_video/vae/tiling.py:44-145``): causal Conv3d with
replicate padding (past side in time, both sides in space), GroupNorm(32)
resnets, a mid-block attention that is causal across frames (a query frame sees
its own and earlier frames), up blocks whose upsamplers repeat the first frame
spatially only and the rest in (t, h, w), GroupNorm + SiLU + conv out.

Memory at 720p x 129 frames is bounded by decoding overlapping spatial tiles
(whole clip in time per tile) and blending the overlaps linearly.  Weights use
the diffusers names.  ``HunyuanVAEDecoder`` is the PyTorch statement of the
decoder (NCTHW, cuDNN convolutions: the oracle); ``HunyuanVAENative`` runs the
same tiles channels-last on the engine's kernels -- the tcgen05 implicit-GEMM
convolution (``csrc/conv.cu``, valid padding on a replicate-padded buffer),
clip GroupNorm (+ SiLU) and the causal upsampler (``csrc/vae_gn.cu``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as Fn


@dataclass(frozen=True)
class HunyuanVAEConfig:
    latent_channels: int = 16
    block_out_channels: tuple = (128, 256, 512, 512)
    layers_per_block: int = 2
    norm_groups: int = 32
    temporal_compression: int = 4
    scaling_factor: float = 0.476986
    tile_latent: int = 32          # spatial tile (latent pixels)
    tile_overlap: int = 8          # latent pixels of overlap between tiles


def _plan(cfg):
    ch = list(reversed(cfg.block_out_channels))
    n_t = {2: 1, 4: 2, 8: 3}[cfg.temporal_compression]
    out = []
    prev = ch[0]
    for i, c in enumerate(ch):
        final = i == len(ch) - 1
        up_s = not final
        up_t = (i >= len(ch) - 1 - n_t) and not final
        out.append((prev, c, up_s, up_t))
        prev = c
    return out


def weight_shapes(cfg: HunyuanVAEConfig) -> dict:
    s = {}

    def conv(n, ci, co, k=3):
        s[n + ".conv.weight"] = (co, ci, k, k, k)
        s[n + ".conv.bias"] = (co,)

    def norm(n, c):
        s[n + ".weight"], s[n + ".bias"] = (c,), (c,)

    def res(n, ci, co):
        norm(n + ".norm1", ci)
        conv(n + ".conv1", ci, co)
        norm(n + ".norm2", co)
        conv(n + ".conv2", co, co)
        if ci != co:
            conv(n + ".conv_shortcut", ci, co, 1)

    top = cfg.block_out_channels[-1]
    s["post_quant_conv.weight"], s["post_quant_conv.bias"] = (cfg.latent_channels, cfg.latent_channels, 1, 1, 1), (cfg.latent_channels,)
    conv("decoder.conv_in", cfg.latent_channels, top)
    res("decoder.mid_block.resnets.0", top, top)
    a = "decoder.mid_block.attentions.0"
    norm(a + ".group_norm", top)
    for n in ("to_q", "to_k", "to_v", "to_out.0"):
        s[f"{a}.{n}.weight"], s[f"{a}.{n}.bias"] = (top, top), (top,)
    res("decoder.mid_block.resnets.1", top, top)
    for i, (ci, co, up_s, _) in enumerate(_plan(cfg)):
        cur = ci
        for j in range(cfg.layers_per_block + 1):
            res(f"decoder.up_blocks.{i}.resnets.{j}", cur, co)
            cur = co
        if up_s:
            conv(f"decoder.up_blocks.{i}.upsamplers.0", co, co)
    norm("decoder.conv_norm_out", cfg.block_out_channels[0])
    conv("decoder.conv_out", cfg.block_out_channels[0], 3)
    return s


def _causal_conv(x, w, b):
    kt, kh, kw = w.shape[2:]
    x = Fn.pad(x, (kw // 2, kw // 2, kh // 2, kh // 2, kt - 1, 0), mode="replicate") if kt > 1 else x
    return Fn.conv3d(x, w, b)


class HunyuanVAEDecoder:
    def __init__(self, cfg: HunyuanVAEConfig, weights: dict):
        self.cfg, self.w = cfg, weights

    @classmethod
    def random_init(cls, cfg: HunyuanVAEConfig = HunyuanVAEConfig(), *, device="cpu", dtype=torch.float32, seed=0):
        g = torch.Generator(device=device).manual_seed(seed)
        w = {}
        for n, shape in weight_shapes(cfg).items():
            if len(shape) == 1:
                w[n] = (torch.ones if (n.endswith("weight") and "norm" in n) else torch.zeros)(shape, device=device, dtype=dtype)
            else:
                fan = 1
                for d in shape[1:]:
                    fan *= d
                w[n] = (torch.randn(shape, generator=g, device=device) * fan ** -0.5).to(dtype)
        return cls(cfg, w)

    def _gn(self, x, n, act=True):
        y = Fn.group_norm(x.float(), self.cfg.norm_groups, self.w[n + ".weight"].float(), self.w[n + ".bias"].float(),
                          eps=1e-6).to(x.dtype)
        return Fn.silu(y) if act else y

    def _conv(self, x, n):
        return _causal_conv(x, self.w[n + ".conv.weight"], self.w[n + ".conv.bias"])

    def _res(self, x, n):
        h = self._conv(x, n + ".conv_shortcut") if n + ".conv_shortcut.conv.weight" in self.w else x
        y = self._conv(self._gn(x, n + ".norm1"), n + ".conv1")
        y = self._conv(self._gn(y, n + ".norm2"), n + ".conv2")
        return y + h

    def _attn(self, x, n):
        B, C, T, H, W = x.shape
        y = self._gn(x, n + ".group_norm", act=False).permute(0, 2, 3, 4, 1).reshape(B, T * H * W, C)
        lin = lambda t, m: Fn.linear(t, self.w[f"{n}.{m}.weight"], self.w[f"{n}.{m}.bias"])  # noqa: E731
        q, k, v = (lin(y, m)[:, None] for m in ("to_q", "to_k", "to_v"))
        # frame-causal mask: token of frame f attends to frames <= f
        frame = torch.arange(T, device=x.device).repeat_interleave(H * W)
        mask = frame[None, :] <= frame[:, None]
        o = Fn.scaled_dot_product_attention(q, k, v, attn_mask=mask)[:, 0]
        o = lin(o, "to_out.0").view(B, T, H, W, C).permute(0, 4, 1, 2, 3)
        return x + o

    def _upsample(self, x, n, up_t):
        first = Fn.interpolate(x[:, :, :1], scale_factor=(1, 2, 2), mode="nearest")
        if x.shape[2] > 1:
            rest = Fn.interpolate(x[:, :, 1:], scale_factor=(2 if up_t else 1, 2, 2), mode="nearest")
            x = torch.cat([first, rest], 2)
        else:
            x = first
        return self._conv(x, n)

    def _decode_tile(self, z):
        x = Fn.conv3d(z, self.w["post_quant_conv.weight"], self.w["post_quant_conv.bias"])
        x = self._conv(x, "decoder.conv_in")
        x = self._res(x, "decoder.mid_block.resnets.0")
        x = self._attn(x, "decoder.mid_block.attentions.0")
        x = self._res(x, "decoder.mid_block.resnets.1")
        for i, (_, _, up_s, up_t) in enumerate(_plan(self.cfg)):
            for j in range(self.cfg.layers_per_block + 1):
                x = self._res(x, f"decoder.up_blocks.{i}.resnets.{j}")
            if up_s:
                x = self._upsample(x, f"decoder.up_blocks.{i}.upsamplers.0", up_t)
        x = self._gn(x, "decoder.conv_norm_out")
        return self._conv(x, "decoder.conv_out")

    @torch.no_grad()
    def decode(self, z: torch.Tensor) -> torch.Tensor:
        """z [B, 16, T, h, w] -> video [B, 3, 1 + 4 (T-1), 8h, 8w] in [-1, 1] (spatially tiled)."""
        cfg = self.cfg
        dt = self.w["decoder.conv_in.conv.weight"].dtype
        z = (z / cfg.scaling_factor).to(dt)
        B, C, T, h, w = z.shape
        tile, ov = cfg.tile_latent, cfg.tile_overlap
        if h <= tile and w <= tile:
            return self._decode_tile(z).clamp(-1, 1)
        step = tile - ov
        s = 8
        out = None
        weight = None
        for y0 in range(0, max(h - ov, 1), step):
            for x0 in range(0, max(w - ov, 1), step):
                y1, x1 = min(y0 + tile, h), min(x0 + tile, w)
                dec = self._decode_tile(z[:, :, :, y0:y1, x0:x1]).float()
                if out is None:
                    out = torch.zeros(B, 3, dec.shape[2], h * s, w * s, device=z.device)
                    weight = torch.zeros(1, 1, 1, h * s, w * s, device=z.device)
                # linear ramps over the overlap on interior edges
                ry = torch.ones(dec.shape[3], device=z.device)
                rx = torch.ones(dec.shape[4], device=z.device)
                r = ov * s
                if y0 > 0:
                    ry[:r] = torch.linspace(0, 1, r, device=z.device)
                if y1 < h:
                    ry[-r:] = torch.minimum(ry[-r:], torch.linspace(1, 0, r, device=z.device))
                if x0 > 0:
                    rx[:r] = torch.linspace(0, 1, r, device=z.device)
                if x1 < w:
                    rx[-r:] = torch.minimum(rx[-r:], torch.linspace(1, 0, r, device=z.device))
                m = (ry[:, None] * rx[None, :]).clamp_min(1e-4)[None, None, None]
                out[:, :, :, y0 * s:y1 * s, x0 * s:x1 * s] += dec * m
                weight[:, :, :, y0 * s:y1 * s, x0 * s:x1 * s] += m
        return (out / weight).clamp(-1, 1).to(dt)


# ------------------------------------------------------------------------------------------------
# Channels-last decoder on the native kernels
# ------------------------------------------------------------------------------------------------
def _pad32(n: int) -> int:
    return -(-n // 32) * 32


class _NConv:
    """A convolution in kernel layout, input / output channels padded to multiples of 32."""

    def __init__(self, w, b, dt):
        from difflet_b200.ops.fused import conv_weight

        Co, Ci = w.shape[:2]
        self.k = tuple(w.shape[2:])
        self.ci, self.co = Ci, Co
        self.Ci, self.Co = _pad32(Ci), _pad32(Co)
        w5 = torch.zeros((self.Co, self.Ci) + self.k, device=w.device, dtype=torch.float32)
        w5[:Co, :Ci] = w.float()
        self.w2 = conv_weight(w5.to(dt))
        bb = torch.zeros(self.Co, device=w.device, dtype=torch.float32)
        bb[:Co] = b.float()
        self.b = bb.to(dt)


class HunyuanVAENative(HunyuanVAEDecoder):
    """The HunyuanVideo decoder channels-last [N, T, H, W, C] on the native kernels (any device:
    on the CPU every op runs its PyTorch oracle).  Each 3x3x3 causal convolution reads a buffer
    [N, T + 2, H + 2, W + 2, C] whose interior the producer writes (GroupNorm + SiLU, the causal
    upsampler, or a copy), then ``pad_replicate`` fills the two leading frames and the one-pixel
    border the way the reference's replicate padding does, and the convolution runs with valid
    padding in T, H and W.  The mid-block attention (one 512-wide head, frame-causal mask) stays
    on PyTorch SDPA."""

    def __init__(self, cfg: HunyuanVAEConfig, weights: dict):
        super().__init__(cfg, weights)
        self._convs = None
        self._norms = None

    def _prep(self):
        if self._convs is None:
            dt = self.w["decoder.conv_in.conv.weight"].dtype
            self._convs = {n[: -len(".conv.weight")]: _NConv(self.w[n], self.w[n[: -len("weight")] + "bias"], dt)
                           for n in self.w if n.endswith(".conv.weight")}
            self._norms = {n[: -len(".weight")]: (self.w[n].float().contiguous(),
                                                  self.w[n[: -len("weight")] + "bias"].float().contiguous())
                           for n in self.w if n.endswith(".weight") and self.w[n].dim() == 1}
        return self._convs

    def _gn_into(self, x, name, silu, y, offs=(0, 0, 0)):
        from difflet_b200.ops import fused as F

        g, b = self._norms[name]
        st = F.gn_stats(x, self.cfg.norm_groups, 1e-6)
        return F.gn_apply(x, st, g, b, self.cfg.norm_groups, silu=silu, y=y, offs=offs)

    def _conv3(self, name, fill, T, H, W, resid=None, like=None):
        """3x3x3 causal conv of the (T, H, W) volume that ``fill(buf, offs)`` writes."""
        from difflet_b200.ops import fused as F

        cv = self._convs[name]
        alloc = torch.zeros if cv.Ci != cv.ci else torch.empty  # padded channels must read as zero
        buf = alloc(1, T + 2, H + 2, W + 2, cv.Ci, device=like.device, dtype=like.dtype)
        fill(buf, (2, 1, 1))
        F.pad_replicate(buf, (2, 1, 1), (T, H, W))
        padded = cv.Co != cv.co
        y = F.conv_cl(buf, cv.w2, cv.b, kt=3, kh=3, kw=3, valid_t=True, valid_h=True, valid_w=True,
                      resid=None if padded else resid)
        if padded:
            y = y[..., : cv.co].contiguous()
            if resid is not None:
                y = y + resid
        return y

    def _pointwise(self, name, x):
        from difflet_b200.ops import fused as F

        cv = self._convs[name]
        return F.conv_cl(x, cv.w2, cv.b, kt=1, kh=1, kw=1)[..., : cv.co].contiguous()

    def _nres(self, x, n):
        _, T, H, W, _ = x.shape
        h = self._pointwise(n + ".conv_shortcut", x) if n + ".conv_shortcut" in self._convs else x
        y = self._conv3(n + ".conv1", lambda buf, o: self._gn_into(x, n + ".norm1", True, buf, o), T, H, W, like=x)
        return self._conv3(n + ".conv2", lambda buf, o: self._gn_into(y, n + ".norm2", True, buf, o), T, H, W,
                           resid=h, like=x)

    def _nattn(self, x, n):
        _, T, H, W, C = x.shape
        y = self._gn_into(x, n + ".group_norm", False, torch.empty_like(x)).reshape(1, T * H * W, C)
        lin = lambda t, m: Fn.linear(t, self.w[f"{n}.{m}.weight"], self.w[f"{n}.{m}.bias"])  # noqa: E731
        q, k, v = (lin(y, m)[:, None] for m in ("to_q", "to_k", "to_v"))
        frame = torch.arange(T, device=x.device).repeat_interleave(H * W)
        mask = frame[None, :] <= frame[:, None]
        o = Fn.scaled_dot_product_attention(q, k, v, attn_mask=mask)[:, 0]
        return x + lin(o, "to_out.0").view(1, T, H, W, C)

    def _nup(self, x, n, up_t):
        from difflet_b200.ops import fused as F

        _, T, H, W, _ = x.shape
        To = 2 * T - 1 if up_t else T
        return self._conv3(n, lambda buf, o: F.upsample_causal(x, up_t, buf, o), To, 2 * H, 2 * W, like=x)

    def _decode_tile(self, z):
        """z [B, 16, T, h, w] -> [B, 3, T', 8h, 8w] (the parent's tiling and blending call this)."""
        self._prep()
        outs = []
        for bi in range(z.shape[0]):
            x = z[bi:bi + 1].permute(0, 2, 3, 4, 1).contiguous()  # [1, T, h, w, 16]
            pq = self.w["post_quant_conv.weight"]
            x = Fn.linear(x, pq.reshape(pq.shape[0], -1), self.w["post_quant_conv.bias"])
            _, T, H, W, c = x.shape
            x = self._conv3("decoder.conv_in", lambda buf, o: buf[:, 2:2 + T, 1:1 + H, 1:1 + W, :c].copy_(x),
                            T, H, W, like=x)
            x = self._nres(x, "decoder.mid_block.resnets.0")
            x = self._nattn(x, "decoder.mid_block.attentions.0")
            x = self._nres(x, "decoder.mid_block.resnets.1")
            for i, (_, _, up_s, up_t) in enumerate(_plan(self.cfg)):
                for j in range(self.cfg.layers_per_block + 1):
                    x = self._nres(x, f"decoder.up_blocks.{i}.resnets.{j}")
                if up_s:
                    x = self._nup(x, f"decoder.up_blocks.{i}.upsamplers.0", up_t)
            _, T, H, W, _ = x.shape
            x = self._conv3("decoder.conv_out", lambda buf, o: self._gn_into(x, "decoder.conv_norm_out", True, buf, o),
                            T, H, W, like=x)
            outs.append(x.permute(0, 4, 1, 2, 3))
        return torch.cat(outs, 0)


__all__ = ["HunyuanVAEConfig", "HunyuanVAEDecoder", "HunyuanVAENative", "weight_shapes"]

