"""LTX-2 audio-video DiT on the sm_100a fused kernels.

The architecture the reference runs through diffusers' ``LTX2VideoTransformer3DModel``
(difflet/models/ltx_2/modeling_ltx_2.py:154-584): a video stream (32 heads x 128 =
4096 wide) and an audio stream (32 x 64 = 2048) through 48 joint blocks.  Per block
and stream: RMSNorm + adaLN (per-block ``scale_shift_table`` + timestep projection)
-> self-attention (q/k RMSNorm across heads, "split" rotary over the whole inner
dimension) -> gated residual; RMSNorm -> text cross-attention -> residual; then the
two cross-modal attentions, audio->video (queries from video, keys / values from
audio) and video->audio, on time-only rotary positions, gated by their own adaLN
vectors; RMSNorm + adaLN -> GELU-tanh MLP -> gated residual.  Output: LayerNorm +
adaLN-continuous (``scale_shift_table`` + embedded timestep) and a projection per
stream.  Guidance hooks of the reference pipeline: ``perturb_blocks`` replaces the
self-attention of those blocks by its values (spatio-temporal guidance) and
``isolate_modalities`` drops the cross-modal attentions (modality guidance).

B200 specifics as for the other families: fused q|k|v GEMMs, q/k norm + rotary +
head scatter in one kernel (per-head rotary tables), gated residuals in the GEMM
epilogue, the text cross-attention K/V of every block computed once per prompt
(``prepare_context``), all blocks' modulation in one GEMV per stream.  Video
attention (head dim 128) runs on the tcgen05 flash-attention kernel; the audio
stream's head dim 64 goes to the library attention.

Weights use diffusers' module names in ``to_diffusers`` / ``from_diffusers`` (the
checkpoint keys the quantization targets name); no LTX-2 checkpoint is available
offline, so the mapping is exercised through round trips and random init.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch

from difflet_b200.ops import fused as F


@dataclass(frozen=True)
class LTX2Config:
    in_channels: int = 128          # video latent channels (patch 1)
    audio_in_channels: int = 128    # audio latent channels x mel bins (8 x 16)
    heads: int = 32
    head_dim: int = 128
    audio_heads: int = 32
    audio_head_dim: int = 64
    layers: int = 48
    text_dim: int = 3840            # Gemma-3 hidden size
    text_len: int = 1024
    timestep_dim: int = 256
    mlp_ratio: int = 4
    theta: float = 10000.0
    eps: float = 1e-6
    max_pos: tuple = (20, 2048, 2048)   # rotary position normalisers (t, h, w)
    audio_max_pos: int = 20
    vae_scale_t: int = 8
    vae_scale: int = 32
    audio_mel_bins: int = 16
    audio_channels: int = 8

    @property
    def dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def audio_dim(self) -> int:
        return self.audio_heads * self.audio_head_dim


LTX2_PRESETS = {
    "ltx-2": LTX2Config(),
    "tiny-ltx2": LTX2Config(heads=2, head_dim=128, audio_heads=2, audio_head_dim=64, layers=2, text_dim=64,
                            text_len=16, in_channels=32, audio_in_channels=32, audio_channels=2, audio_mel_bins=16),
}


def get_ltx2_config(name: str, **kw) -> LTX2Config:
    return replace(LTX2_PRESETS[name], **kw)


# ----------------------------------------------------------------------------- rotary tables
def _freqs(n: int, theta: float) -> torch.Tensor:
    """n rotary frequencies spread geometrically over [pi/2, theta * pi/2] (float64)."""
    if n == 0:
        return torch.zeros(0, dtype=torch.float64)
    return (theta ** torch.linspace(0.0, 1.0, n, dtype=torch.float64)) * (math.pi / 2)


def rope_angles(coords: torch.Tensor, max_pos, inner_dim: int, theta: float) -> torch.Tensor:
    """coords [S, n_axes, 2] ([start, end) per axis) -> angles [S, inner_dim / 2] (float64).

    Each axis gets ``(inner_dim / 2) // n_axes`` frequencies applied to its
    midpoint normalised to [-1, 1] by ``max_pos``; leftover pairs (when n_axes does
    not divide) are identity rotations placed first.  The table covers the whole
    inner dimension, so heads see different frequencies (head h: pairs
    [h * dh/2, (h + 1) * dh/2))."""
    S, n_axes, _ = coords.shape
    pairs = inner_dim // 2
    per = pairs // n_axes
    mids = coords.to(torch.float64).mean(-1)  # [S, n_axes]
    parts = [torch.zeros(S, pairs - per * n_axes, dtype=torch.float64)]
    for a in range(n_axes):
        frac = mids[:, a] / float(max_pos[a]) * 2.0 - 1.0
        parts.append(frac[:, None] * _freqs(per, theta)[None, :])
    return torch.cat(parts, 1)


def video_coords(frames: int, h: int, w: int, cfg: LTX2Config, fps: float = 24.0) -> torch.Tensor:
    """[S, 3, 2] pixel-space patch bounds (time in seconds, causal first frame) of a latent grid."""
    t = torch.arange(frames, dtype=torch.float64)
    tt = torch.stack([t, t + 1], -1) * cfg.vae_scale_t
    tt = (tt + 1 - cfg.vae_scale_t).clamp(min=0) / fps
    hh = torch.stack([torch.arange(h), torch.arange(h) + 1], -1).double() * cfg.vae_scale
    ww = torch.stack([torch.arange(w), torch.arange(w) + 1], -1).double() * cfg.vae_scale
    g = torch.zeros(frames, h, w, 3, 2, dtype=torch.float64)
    g[..., 0, :] = tt[:, None, None, :]
    g[..., 1, :] = hh[None, :, None, :]
    g[..., 2, :] = ww[None, None, :, :]
    return g.reshape(-1, 3, 2)


def audio_coords(frames: int, hop_s: float = 0.04) -> torch.Tensor:
    """[S, 1, 2] audio latent frame bounds in seconds."""
    t = torch.arange(frames, dtype=torch.float64)
    return (torch.stack([t, t + 1], -1) * hop_s)[:, None, :]


# ----------------------------------------------------------------------------- model
_BLOCK_SHAPES = {
    # video self-attention
    "v_qkv.w": ("3v", "v"), "v_qkv.b": ("3v",), "v_qn": ("v",), "v_kn": ("v",), "v_o.w": ("v", "v"), "v_o.b": ("v",),
    # audio self-attention
    "a_qkv.w": ("3a", "a"), "a_qkv.b": ("3a",), "a_qn": ("a",), "a_kn": ("a",), "a_o.w": ("a", "a"), "a_o.b": ("a",),
    # text cross-attention (keys / values from the caption-projected text of the same width)
    "v_cq.w": ("v", "v"), "v_cq.b": ("v",), "v_cqn": ("v",), "v_ckv.w": ("2v", "v"), "v_ckv.b": ("2v",),
    "v_ckn": ("v",), "v_co.w": ("v", "v"), "v_co.b": ("v",),
    "a_cq.w": ("a", "a"), "a_cq.b": ("a",), "a_cqn": ("a",), "a_ckv.w": ("2a", "a"), "a_ckv.b": ("2a",),
    "a_ckn": ("a",), "a_co.w": ("a", "a"), "a_co.b": ("a",),
    # audio -> video (queries video, keys / values audio; inner width = audio width)
    "a2v_q.w": ("a", "v"), "a2v_q.b": ("a",), "a2v_qn": ("a",), "a2v_kv.w": ("2a", "a"), "a2v_kv.b": ("2a",),
    "a2v_kn": ("a",), "a2v_o.w": ("v", "a"), "a2v_o.b": ("v",),
    # video -> audio
    "v2a_q.w": ("a", "a"), "v2a_q.b": ("a",), "v2a_qn": ("a",), "v2a_kv.w": ("2a", "v"), "v2a_kv.b": ("2a",),
    "v2a_kn": ("a",), "v2a_o.w": ("a", "a"), "v2a_o.b": ("a",),
    # MLPs
    "v_up.w": ("4v", "v"), "v_up.b": ("4v",), "v_down.w": ("v", "4v"), "v_down.b": ("v",),
    "a_up.w": ("4a", "a"), "a_up.b": ("4a",), "a_down.w": ("a", "4a"), "a_down.b": ("a",),
    # modulation tables
    "sst": (6, "v"), "asst": (6, "a"), "v_av": (3, "v"), "a_av": (3, "a"),
}


class LTX2Transformer:
    def __init__(self, cfg: LTX2Config, weights: dict[str, torch.Tensor]):
        self.cfg = cfg
        self.w = weights
        self.par = None
        self._rope = {}
        self._ones = {}

    @property
    def device(self):
        return next(iter(self.w.values())).device

    @property
    def dtype(self):
        return self.w["proj_in.w"].dtype

    def to(self, device=None, dtype=None):
        for k, v in self.w.items():
            self.w[k] = v.to(device=device, dtype=dtype if v.is_floating_point() and v.element_size() > 1 else None)
        self._rope.clear()
        return self

    # ------------------------------------------------------------------ weights
    @staticmethod
    def weight_shapes(cfg: LTX2Config) -> dict[str, tuple]:
        v, a, T = cfg.dim, cfg.audio_dim, cfg.timestep_dim
        dims = {"v": v, "a": a, "2v": 2 * v, "3v": 3 * v, "4v": cfg.mlp_ratio * v, "2a": 2 * a, "3a": 3 * a,
                "4a": cfg.mlp_ratio * a}
        s = {
            "proj_in.w": (v, cfg.in_channels), "proj_in.b": (v,),
            "audio_proj_in.w": (a, cfg.audio_in_channels), "audio_proj_in.b": (a,),
            "cap.w1": (v, cfg.text_dim), "cap.b1": (v,), "cap.w2": (v, v), "cap.b2": (v,),
            "acap.w1": (a, cfg.text_dim), "acap.b1": (a,), "acap.w2": (a, a), "acap.b2": (a,),
            "t.w1": (v, T), "t.b1": (v,), "t.w2": (v, v), "t.b2": (v,), "t.mod.w": (6 * v, v), "t.mod.b": (6 * v,),
            "at.w1": (a, T), "at.b1": (a,), "at.w2": (a, a), "at.b2": (a,), "at.mod.w": (6 * a, a),
            "at.mod.b": (6 * a,),
            "av.v.w": (3 * v, v), "av.v.b": (3 * v,), "av.a.w": (3 * a, a), "av.a.b": (3 * a,),
            "sst_out": (2, v), "proj_out.w": (cfg.in_channels, v), "proj_out.b": (cfg.in_channels,),
            "asst_out": (2, a), "audio_proj_out.w": (cfg.audio_in_channels, a),
            "audio_proj_out.b": (cfg.audio_in_channels,),
        }
        for i in range(cfg.layers):
            for k, shp in _BLOCK_SHAPES.items():
                s[f"blk.{i}.{k}"] = tuple(dims[d] if isinstance(d, str) else d for d in shp)
        return s

    @classmethod
    def random_init(cls, cfg: LTX2Config, *, device="cpu", dtype=torch.float32, seed: int = 0, std: float = 0.02):
        g = torch.Generator(device="cpu")
        g.manual_seed(seed)
        w = {}
        for name, shape in cls.weight_shapes(cfg).items():
            t = torch.randn(shape, generator=g, dtype=torch.float64) * std
            if name.endswith("n") and len(shape) == 1 and name.rsplit(".", 1)[-1] in (
                    "v_qn", "v_kn", "a_qn", "a_kn", "v_cqn", "v_ckn", "a_cqn", "a_ckn", "a2v_qn", "a2v_kn",
                    "v2a_qn", "v2a_kn"):
                t = t + 1.0
            w[name] = t.to(device=device, dtype=dtype)
        return cls(cfg, w)

    # ------------------------------------------------------------------ tables
    def _ones_gate(self, B, width):
        key = (B, width)
        if key not in self._ones:
            dt = torch.float64 if self.dtype == torch.float64 else torch.float32
            self._ones[key] = torch.ones(B, width, device=self.device, dtype=dt)
        return self._ones[key]

    def rope(self, key, coords, max_pos, inner):
        if key not in self._rope:
            ang = rope_angles(coords, max_pos, inner, self.cfg.theta)
            dt = torch.float64 if self.dtype == torch.float64 else torch.float32
            self._rope[key] = (ang.cos().to(self.device, dt).contiguous(), ang.sin().to(self.device, dt).contiguous())
        return self._rope[key]

    # ------------------------------------------------------------------ conditioning
    def _mlp(self, x, w1, b1, w2, b2, act):
        h = F.linear(x, self.w[w1], self.w[b1], act=act)
        return F.linear(h, self.w[w2], self.w[b2])

    def prepare_context(self, text: torch.Tensor, audio_text: torch.Tensor | None = None):
        """Caption projections and every block's text K/V (normed), once per prompt:
        returns per block ((k_v, v_v), (k_a, v_a)) [B, H, L, dh]."""
        cfg, w = self.cfg, self.w
        audio_text = text if audio_text is None else audio_text
        B, L, _ = text.shape
        ctx_v = self._mlp(text.reshape(B * L, -1), "cap.w1", "cap.b1", "cap.w2", "cap.b2", "gelu")
        ctx_a = self._mlp(audio_text.reshape(B * L, -1), "acap.w1", "acap.b1", "acap.w2", "acap.b2", "gelu")
        out = []
        for i in range(cfg.layers):
            p = f"blk.{i}."
            pair = []
            for st, ctx, H, dh, D in (("v", ctx_v, cfg.heads, cfg.head_dim, cfg.dim),
                                      ("a", ctx_a, cfg.audio_heads, cfg.audio_head_dim, cfg.audio_dim)):
                kv = F.linear(ctx, w[p + st + "_ckv.w"], w[p + st + "_ckv.b"])
                k = torch.empty(B, H, L, dh, device=ctx.device, dtype=ctx.dtype)
                v = torch.empty_like(k)
                F.qkv_scatter(kv, q_off=-1, k_off=0, v_off=D, S_src=L, H=H, dh=dh, q_dst=None, k_dst=[k], v_dst=[v],
                              S_dst=L, norm_mode=2, wk=w[p + st + "_ckn"], eps=cfg.eps, heads_per_rank=H)
                pair.append((k, v))
            out.append(tuple(pair))
        return out

    def time_embed(self, timestep: torch.Tensor):
        """timestep [B] in [0, 1] -> (temb_v, temb_a, mod_v [B, 6v], mod_a [B, 6a], av_v [B, 3v], av_a [B, 3a])."""
        cfg = self.cfg
        tf = F.timestep_embed(timestep * 1000.0, cfg.timestep_dim)
        tv = F.gemv(self.w["t.w2"], F.gemv(self.w["t.w1"], tf, self.w["t.b1"], silu_out=True), self.w["t.b2"])
        ta = F.gemv(self.w["at.w2"], F.gemv(self.w["at.w1"], tf, self.w["at.b1"], silu_out=True), self.w["at.b2"])
        mv = F.gemv(self.w["t.mod.w"], tv, self.w["t.mod.b"], silu_in=True)
        ma = F.gemv(self.w["at.mod.w"], ta, self.w["at.mod.b"], silu_in=True)
        av_v = F.gemv(self.w["av.v.w"], tv, self.w["av.v.b"], silu_in=True)
        av_a = F.gemv(self.w["av.a.w"], ta, self.w["av.a.b"], silu_in=True)
        return tv, ta, mv, ma, av_v, av_a

    # ------------------------------------------------------------------ attention helpers
    def _self_attn(self, x, n, p, st, B, S, H, dh, D, cos, sin, perturbed, mod_shift, mod_scale, gate):
        cfg, w = self.cfg, self.w
        F.ln_modulate(x, shift=mod_shift, scale=mod_scale, eps=cfg.eps, rms=True, rows_per_batch=S, out=n)
        qkv = F.linear(n, w[p + st + "_qkv.w"], w[p + st + "_qkv.b"])
        q = torch.empty(B, H, S, dh, device=x.device, dtype=x.dtype)
        k, v = torch.empty_like(q), torch.empty_like(q)
        F.qkv_scatter(qkv, q_off=0, k_off=D, v_off=2 * D, S_src=S, H=H, dh=dh, q_dst=[q], k_dst=[k], v_dst=[v], S_dst=S,
                      norm_mode=2, wq=w[p + st + "_qn"], wk=w[p + st + "_kn"], eps=cfg.eps, cos=cos, sin=sin,
                      rope_half=True, heads_per_rank=H)
        o2 = torch.empty(B * S, D, device=x.device, dtype=x.dtype)
        ov = o2.view(B, S, H, dh).permute(0, 2, 1, 3)  # token-major output written by the kernel
        if perturbed:  # spatio-temporal guidance: the attention passes its values through
            ov.copy_(v)
        else:
            F.attention(q, k, v, 1.0 / math.sqrt(dh), out=ov)
        F.linear(o2, w[p + st + "_o.w"], w[p + st + "_o.b"], out=x, gate=gate, resid=x, rows_per_batch=S)

    def _cross_text(self, x, n, p, st, B, S, H, dh, D, kv, kv_lo, kv_hi):
        cfg, w = self.cfg, self.w
        F.ln_modulate(x, eps=cfg.eps, rms=True, out=n)
        qin = F.linear(n, w[p + st + "_cq.w"], w[p + st + "_cq.b"])
        q = torch.empty(B, H, S, dh, device=x.device, dtype=x.dtype)
        F.qkv_scatter(qin, q_off=0, k_off=-1, v_off=-1, S_src=S, H=H, dh=dh, q_dst=[q], k_dst=None, v_dst=None,
                      S_dst=S, norm_mode=2, wq=w[p + st + "_cqn"], eps=cfg.eps, heads_per_rank=H)
        k, v = kv
        o = F.attention(q, k, v, 1.0 / math.sqrt(dh), kv_lo=kv_lo, kv_hi=kv_hi)
        F.linear(o.permute(0, 2, 1, 3).reshape(B * S, D), w[p + st + "_co.w"], w[p + st + "_co.b"], out=x,
                 gate=self._ones_gate(B, D), resid=x, rows_per_batch=S)

    def _cross_modal(self, xq, nq, xkv_normed, p, name, B, Sq, Skv, Dq, mshift, mscale, gate, cos_q, sin_q, cos_k,
                     sin_k):
        """Cross-modal attention (inner width = audio width, audio head dim)."""
        cfg, w = self.cfg, self.w
        H, dh, Di = cfg.audio_heads, cfg.audio_head_dim, cfg.audio_dim
        F.ln_modulate(xq, shift=mshift, scale=mscale, eps=cfg.eps, rms=True, rows_per_batch=Sq, out=nq)
        qin = F.linear(nq, w[p + name + "_q.w"], w[p + name + "_q.b"])
        kvin = F.linear(xkv_normed, w[p + name + "_kv.w"], w[p + name + "_kv.b"])
        q = torch.empty(B, H, Sq, dh, device=xq.device, dtype=xq.dtype)
        k = torch.empty(B, H, Skv, dh, device=xq.device, dtype=xq.dtype)
        v = torch.empty_like(k)
        F.qkv_scatter(qin, q_off=0, k_off=-1, v_off=-1, S_src=Sq, H=H, dh=dh, q_dst=[q], k_dst=None, v_dst=None,
                      S_dst=Sq, norm_mode=2, wq=w[p + name + "_qn"], eps=cfg.eps, cos=cos_q, sin=sin_q, rope_half=True,
                      heads_per_rank=H)
        F.qkv_scatter(kvin, q_off=-1, k_off=0, v_off=Di, S_src=Skv, H=H, dh=dh, q_dst=None, k_dst=[k], v_dst=[v],
                      S_dst=Skv, norm_mode=2, wk=w[p + name + "_kn"], eps=cfg.eps, cos=cos_k, sin=sin_k,
                      rope_half=True, heads_per_rank=H)
        o = F.attention(q, k, v, 1.0 / math.sqrt(dh))
        F.linear(o.permute(0, 2, 1, 3).reshape(B * Sq, Di), w[p + name + "_o.w"], w[p + name + "_o.b"], out=xq,
                 gate=gate, resid=xq, rows_per_batch=Sq)

    # ------------------------------------------------------------------ forward
    def forward(self, video_tokens, audio_tokens, timestep, context, *, vcoords, acoords, text_valid=None,
                perturb_blocks=(), isolate_modalities=False, cond=None):
        """video_tokens [B, Sv, in_ch], audio_tokens [B, Sa, audio_in_ch], timestep [B] in [0, 1],
        context = ``prepare_context(...)``; vcoords [Sv, 3, 2], acoords [Sa, 1, 2] (seconds /
        pixels).  Returns (video velocity [B, Sv, in_ch], audio velocity [B, Sa, audio_in_ch])."""
        cfg, w = self.cfg, self.w
        B, Sv, _ = video_tokens.shape
        Sa = audio_tokens.shape[1]
        V, A = cfg.dim, cfg.audio_dim
        Hv, dv, Ha, da = cfg.heads, cfg.head_dim, cfg.audio_heads, cfg.audio_head_dim
        tv, ta, mv, ma, av_v, av_a = cond if cond is not None else self.time_embed(timestep)
        cos_v, sin_v = self.rope(("v", Sv), vcoords, cfg.max_pos, V)
        cos_a, sin_a = self.rope(("a", Sa), acoords, (cfg.audio_max_pos,), A)
        # cross-modal rotary: time only, at the audio (inner) width
        cos_vt, sin_vt = self.rope(("vt", Sv), vcoords[:, :1], (cfg.audio_max_pos,), A)
        kv_lo = kv_hi = None
        if text_valid is not None:
            kv_hi = text_valid.to(device=video_tokens.device, dtype=torch.int32)
            kv_lo = torch.zeros_like(kv_hi)
        hv = F.linear(video_tokens.reshape(B * Sv, -1), w["proj_in.w"], w["proj_in.b"])
        ha = F.linear(audio_tokens.reshape(B * Sa, -1), w["audio_proj_in.w"], w["audio_proj_in.b"])
        nv = torch.empty_like(hv)
        na = torch.empty_like(ha)
        nv2 = torch.empty_like(hv)
        na2 = torch.empty_like(ha)
        mvv = mv.view(B, 6, V)
        maa = ma.view(B, 6, A)
        avv = av_v.view(B, 3, V)
        ava = av_a.view(B, 3, A)
        for i in range(cfg.layers):
            p = f"blk.{i}."
            sv = (w[p + "sst"][None].to(mvv.dtype) + mvv)  # [B, 6, V] f32
            sa = (w[p + "asst"][None].to(maa.dtype) + maa)
            cv = (w[p + "v_av"][None].to(avv.dtype) + avv)
            ca = (w[p + "a_av"][None].to(ava.dtype) + ava)
            pert = i in perturb_blocks
            self._self_attn(hv, nv, p, "v", B, Sv, Hv, dv, V, cos_v, sin_v, pert, sv[:, 0], sv[:, 1],
                            sv[:, 2].contiguous())
            self._self_attn(ha, na, p, "a", B, Sa, Ha, da, A, cos_a, sin_a, pert, sa[:, 0], sa[:, 1],
                            sa[:, 2].contiguous())
            kv_v, kv_a = context[i]
            self._cross_text(hv, nv, p, "v", B, Sv, Hv, dv, V, kv_v, kv_lo, kv_hi)
            self._cross_text(ha, na, p, "a", B, Sa, Ha, da, A, kv_a, kv_lo, kv_hi)
            if not isolate_modalities:
                # both directions read the pre-update streams
                F.ln_modulate(ha, eps=cfg.eps, rms=True, out=na2)
                F.ln_modulate(hv, eps=cfg.eps, rms=True, out=nv2)
                self._cross_modal(hv, nv, na2, p, "a2v", B, Sv, Sa, V, cv[:, 0], cv[:, 1], cv[:, 2].contiguous(),
                                  cos_vt, sin_vt, cos_a, sin_a)
                self._cross_modal(ha, na, nv2, p, "v2a", B, Sa, Sv, A, ca[:, 0], ca[:, 1], ca[:, 2].contiguous(),
                                  cos_a, sin_a, cos_vt, sin_vt)
            for x, n, st, S, mod in ((hv, nv, "v", Sv, sv), (ha, na, "a", Sa, sa)):
                F.ln_modulate(x, shift=mod[:, 3], scale=mod[:, 4], eps=cfg.eps, rms=True, rows_per_batch=S, out=n)
                h = F.linear(n, w[p + st + "_up.w"], w[p + st + "_up.b"], act="gelu")
                F.linear(h, w[p + st + "_down.w"], w[p + st + "_down.b"], out=x, gate=mod[:, 5].contiguous(), resid=x,
                         rows_per_batch=S)
        outs = []
        for x, S, sst, temb, wo, bo in ((hv, Sv, "sst_out", tv, "proj_out.w", "proj_out.b"),
                                        (ha, Sa, "asst_out", ta, "audio_proj_out.w", "audio_proj_out.b")):
            fm = w[sst][None].to(temb.dtype) + temb[:, None]  # [B, 2, D]: shift, scale
            n = F.ln_modulate(x, shift=fm[:, 0], scale=fm[:, 1], eps=cfg.eps, rows_per_batch=S)
            outs.append(F.linear(n, w[wo], w[bo]).view(B, S, -1))
        return outs[0], outs[1]

    __call__ = forward


def pack_video(lat: torch.Tensor) -> torch.Tensor:
    """[B, C, T, H, W] -> [B, T*H*W, C] (patch size 1)."""
    B, C = lat.shape[:2]
    return lat.reshape(B, C, -1).transpose(1, 2)


def unpack_video(tok: torch.Tensor, grid) -> torch.Tensor:
    B, S, C = tok.shape
    return tok.transpose(1, 2).reshape(B, C, *grid)


def pack_audio(lat: torch.Tensor) -> torch.Tensor:
    """[B, C, T, mel] -> [B, T, C*mel]."""
    B, C, T, M = lat.shape
    return lat.permute(0, 2, 1, 3).reshape(B, T, C * M)


def unpack_audio(tok: torch.Tensor, channels: int) -> torch.Tensor:
    B, T, CM = tok.shape
    return tok.view(B, T, channels, CM // channels).permute(0, 2, 1, 3)


__all__ = ["LTX2Config", "LTX2Transformer", "audio_coords", "get_ltx2_config", "pack_audio", "pack_video",
           "rope_angles", "unpack_audio", "unpack_video", "video_coords"]
