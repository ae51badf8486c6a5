"""MiniMax-H3 joint video + audio DiT on the sm_100a fused kernels.

Architecture of the reference's ``MiniMaxH3Transformer3DModel``
(difflet/models/minimax_h3/modeling_minimax_h3.py:55-739): ONE packed sequence
[text | condition video | audio | video] through 50 blocks of full self-attention
(56 heads x 128 = 7168 inner, wider than the 5376 residual) and SwiGLU MLPs (14336),
no cross-attention; per-head RMS q/k norms; rotary on the first 96 channels of each
head (three axes t, h, w x 16 shared frequencies, rotate-half); AdaLN per row chosen
from a (timestep, modality) table: row index ``timestep_index * 3 + tag``, one
[18 D] projection of the timestep embedding per block; a 2-block token refiner on
the projected text; RMSNorm output modulated per timestep; two output heads.

B200 mapping: the per-row modulation rows are gathered inside the LN kernel and the
GEMM epilogue (``row_map``), so each block is one GEMM per linear over the whole
packed sequence; q/k norm + partial rotary + head scatter are one kernel; SwiGLU is
fused into the up-projection's epilogue (weight rows interleaved at load); the
attention over the packed sequence runs on the tcgen05 kernel.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch

from difflet_b200.ops import fused as F

MODALITIES = 3


@dataclass(frozen=True)
class MiniMaxH3Config:
    hidden: int = 5376
    heads: int = 56
    head_dim: int = 128
    layers: int = 50
    refiner_layers: int = 2
    ffn: int = 14336
    in_channels: int = 24
    patch: tuple = (1, 2, 2)
    audio_in_channels: int = 32
    text_dim: int = 5120
    freq_dim: int = 256
    time_hidden: int = 5376
    time_dim: int = 2688
    rope_freq_dim: int = 16
    theta: float = 10000.0
    eps: float = 1e-5
    qk_eps: float = 1e-5
    final_eps: float = 1e-5

    @property
    def inner(self) -> int:
        return self.heads * self.head_dim

    @property
    def patch_dim(self) -> int:
        return self.in_channels * self.patch[0] * self.patch[1] * self.patch[2]


PRESETS = {
    "minimax-h3": MiniMaxH3Config(),
    "tiny-minimax-h3": MiniMaxH3Config(hidden=256, heads=2, layers=2, refiner_layers=1, ffn=512, in_channels=4,
                                       audio_in_channels=8, text_dim=64, time_hidden=256, time_dim=128),
}


def get_minimax_config(name: str, **kw) -> MiniMaxH3Config:
    return replace(PRESETS[name], **kw)


def rope_table(position_ids: torch.Tensor, cfg: MiniMaxH3Config) -> torch.Tensor:
    """[S, 3] (t, h, w) positions -> angles [S, 3 * rope_freq_dim] (float64): the unique half
    of the rotate-half table (the released model repeats it for the two halves)."""
    n = cfg.rope_freq_dim
    inv = 1.0 / (cfg.theta ** (torch.arange(0, 2 * n, 2, dtype=torch.float64) / (2 * n)))
    f = position_ids.to(torch.float64)[:, :, None] * inv[None, None, :]   # [S, 3, n]
    return f.reshape(position_ids.shape[0], 3 * n)


def _block_shapes(cfg: MiniMaxH3Config, adaln: bool) -> dict:
    D, I, Fh = cfg.hidden, cfg.inner, cfg.ffn
    s = {"n1": (D,), "qkv.w": (3 * I, D), "qn": (cfg.head_dim,), "kn": (cfg.head_dim,), "o.w": (D, I),
         "n2": (D,), "up.w": (2 * Fh, D), "down.w": (D, Fh)}
    if adaln:
        s["ada.w"] = (6 * D * MODALITIES, cfg.time_dim)
        s["ada.b"] = (6 * D * MODALITIES,)
    return s


class MiniMaxH3Transformer:
    def __init__(self, cfg: MiniMaxH3Config, weights: dict):
        self.cfg, self.w = cfg, weights
        self._rope = {}

    @property
    def device(self):
        return self.w["proj_in.w"].device

    @property
    def dtype(self):
        return self.w["qkv.w" if "qkv.w" in self.w else "blk.0.qkv.w"].dtype

    @staticmethod
    def weight_shapes(cfg: MiniMaxH3Config) -> dict:
        D = cfg.hidden
        s = {"proj_in.w": (D, cfg.patch_dim), "proj_in.b": (D,), "audio_proj_in.w": (D, cfg.audio_in_channels),
             "audio_proj_in.b": (D,), "ctx.w": (D, cfg.text_dim), "ctx.b": (D,),
             "t.w1": (cfg.time_hidden, cfg.freq_dim), "t.b1": (cfg.time_hidden,),
             "t.w2": (cfg.time_dim, cfg.time_hidden), "t.b2": (cfg.time_dim,),
             "ref.final": (D,), "out.norm": (D,), "out.w": (2 * D, cfg.time_dim), "out.b": (2 * D,),
             "proj_out.w": (cfg.patch_dim, D), "proj_out.b": (cfg.patch_dim,),
             "audio_proj_out.w": (cfg.audio_in_channels, D), "audio_proj_out.b": (cfg.audio_in_channels,)}
        for j in range(cfg.refiner_layers):
            for k, v in _block_shapes(cfg, False).items():
                s[f"ref.{j}.{k}"] = v
        for i in range(cfg.layers):
            for k, v in _block_shapes(cfg, True).items():
                s[f"blk.{i}.{k}"] = v
        return s

    @classmethod
    def random_init(cls, cfg: MiniMaxH3Config, *, device="cpu", dtype=torch.float32, seed=0, std=0.02):
        g = torch.Generator().manual_seed(seed)
        w = {}
        for k, shp in cls.weight_shapes(cfg).items():
            t = torch.randn(shp, generator=g, dtype=torch.float64) * std
            if len(shp) == 1 and k.split(".")[-1] in ("n1", "n2", "qn", "kn", "final", "norm"):
                t = t + 1.0
            w[k] = t.to(device=device, dtype=dtype)
        return cls(cfg, w)

    def to(self, device=None, dtype=None):
        for k, v in self.w.items():
            self.w[k] = v.to(device=device, dtype=dtype)
        self._rope.clear()
        return self

    # ------------------------------------------------------------------ pieces
    def time_embed(self, timestep: torch.Tensor) -> torch.Tensor:
        """Distinct timesteps [T] in [0, 1] (unscaled) -> temb [T, time_dim] f32."""
        tf = F.timestep_embed(timestep.float() if timestep.is_cuda else timestep, self.cfg.freq_dim)
        return F.gemv(self.w["t.w2"], F.gemv(self.w["t.w1"], tf, self.w["t.b1"], silu_out=True), self.w["t.b2"])

    def modulation(self, temb: torch.Tensor, i: int) -> torch.Tensor:
        """Block i's AdaLN table [T * 3, 6, D] (f32): rows timestep-major, modality-minor."""
        T = temb.shape[0]
        m = F.gemv(self.w[f"blk.{i}.ada.w"], temb, self.w[f"blk.{i}.ada.b"], silu_in=True)  # [T, 18 D]
        return m.view(T * MODALITIES, 6, self.cfg.hidden)

    def _attn_mlp(self, h, p, B, S, cos, sin, mod=None, row_map=None, kv_hi=None):
        cfg, w = self.cfg, self.w
        D, I, H, dh = cfg.hidden, cfg.inner, cfg.heads, cfg.head_dim
        n = F.ln_modulate(h, w=w[p + "n1"], eps=cfg.eps, rms=True, row_map=row_map,
                          shift=None if mod is None else mod[:, 0], scale=None if mod is None else mod[:, 1])
        qkv = F.linear(n, w[p + "qkv.w"])
        q = torch.empty(B, H, S, dh, device=h.device, dtype=h.dtype)
        k, v = torch.empty_like(q), torch.empty_like(q)
        F.qkv_scatter(qkv, q_off=0, k_off=I, v_off=2 * I, S_src=S, H=H, dh=dh, q_dst=[q], k_dst=[k], v_dst=[v],
                      S_dst=S, norm_mode=1, wq=w[p + "qn"], wk=w[p + "kn"], eps=cfg.qk_eps, cos=cos, sin=sin,
                      rope_half=True, heads_per_rank=H)
        o = torch.empty(B * S, I, device=h.device, dtype=h.dtype)
        lo = hi = None
        if kv_hi is not None:
            hi = kv_hi
            lo = torch.zeros_like(hi)
        F.attention(q, k, v, 1.0 / math.sqrt(dh), out=o.view(B, S, H, dh).permute(0, 2, 1, 3), kv_lo=lo, kv_hi=hi)
        if mod is None:
            F.linear(o, w[p + "o.w"], out=h, gate=self._ones(), resid=h, rows_per_batch=B * S)
        else:
            F.linear(o, w[p + "o.w"], out=h, gate=mod[:, 2], resid=h, gate_row_map=row_map)
        n = F.ln_modulate(h, w=w[p + "n2"], eps=cfg.eps, rms=True, row_map=row_map,
                          shift=None if mod is None else mod[:, 3], scale=None if mod is None else mod[:, 4])
        u = F.linear(n, w[p + "up.w"], act="swiglu")
        if mod is None:
            F.linear(u, w[p + "down.w"], out=h, gate=self._ones(), resid=h, rows_per_batch=B * S)
        else:
            F.linear(u, w[p + "down.w"], out=h, gate=mod[:, 5], resid=h, gate_row_map=row_map)

    def _ones(self):
        key = "ones"
        if key not in self._rope:
            dt = torch.float64 if self.dtype == torch.float64 else torch.float32
            self._rope[key] = torch.ones(1, self.cfg.hidden, device=self.device, dtype=dt)
        return self._rope[key]

    def rope(self, layout_key, position_ids):
        if layout_key not in self._rope:
            ang = rope_table(position_ids, self.cfg)
            dt = torch.float64 if self.dtype == torch.float64 else torch.float32
            self._rope[layout_key] = (ang.cos().to(self.device, dt).contiguous(),
                                      ang.sin().to(self.device, dt).contiguous())
        return self._rope[layout_key]

    def refine_text(self, text: torch.Tensor, text_valid=None) -> torch.Tensor:
        cfg, w = self.cfg, self.w
        B, L, _ = text.shape
        h = F.linear(text.reshape(B * L, -1), w["ctx.w"], w["ctx.b"])
        pos = torch.zeros(L, 3)
        pos[:, 0] = torch.arange(L)
        # the refiner has no rotary: identity tables
        cos = torch.ones(L, 3 * cfg.rope_freq_dim, device=h.device,
                         dtype=torch.float64 if self.dtype == torch.float64 else torch.float32)
        sin = torch.zeros_like(cos)
        hi = None if text_valid is None else text_valid.to(device=h.device, dtype=torch.int32)
        for j in range(cfg.refiner_layers):
            self._attn_mlp(h, f"ref.{j}.", B, L, cos, sin, kv_hi=hi)
        return F.ln_modulate(h, w=w["ref.final"], eps=cfg.final_eps, rms=True).view(B, L, -1)

    # ------------------------------------------------------------------ forward
    def forward(self, video_rows, audio_rows, text, timestep, timestep_indices, layout, *, text_valid=None,
                temb=None):
        """video_rows [B, Nv, patch_dim], audio_rows [B, Na, audio_in], text [B, L, text_dim];
        timestep [T] distinct values, timestep_indices [S] (slot of every packed row);
        ``layout`` from ``layout.build_layout``.  Returns (video [B, Nv, patch_dim], audio [B, Na, audio_in])."""
        cfg, w = self.cfg, self.w
        B = video_rows.shape[0]
        S, D = layout.sequence_length, cfg.hidden
        dev = video_rows.device
        cos, sin = self.rope(("layout", S, int(layout.text_indices.numel())), layout.position_ids)
        txt = self.refine_text(text, text_valid)
        ve = F.linear(video_rows.reshape(-1, video_rows.shape[-1]), w["proj_in.w"], w["proj_in.b"])
        ae = F.linear(audio_rows.reshape(-1, audio_rows.shape[-1]), w["audio_proj_in.w"], w["audio_proj_in.b"])
        h = torch.zeros(B, S, D, device=dev, dtype=ve.dtype)
        h[:, layout.text_indices.to(dev)] = txt.to(h.dtype)
        h[:, layout.video_indices.to(dev)] = ve.view(B, -1, D)
        h[:, layout.audio_indices.to(dev)] = ae.view(B, -1, D)
        h2 = h.view(B * S, D)
        if temb is None:
            temb = self.time_embed(timestep)
        tidx = timestep_indices.to(dev).long()
        adaln = (tidx * MODALITIES + layout.token_tags.to(dev).long()).to(torch.int32)
        row_map = adaln.repeat(B).contiguous()
        for i in range(cfg.layers):
            mod = self.modulation(temb, i)
            self._attn_mlp(h2, f"blk.{i}.", B, S, cos, sin, mod=mod, row_map=row_map)
        so = F.gemv(w["out.w"], temb, w["out.b"], silu_in=True)  # [T, 2D]: shift, scale
        nmap = tidx.to(torch.int32).repeat(B).contiguous()
        n = F.ln_modulate(h2, w=w["out.norm"], eps=cfg.final_eps, rms=True, shift=so[:, :D], scale=so[:, D:],
                          row_map=nmap).view(B, S, D)
        vo = F.linear(n[:, layout.video_indices.to(dev)].reshape(-1, D), w["proj_out.w"], w["proj_out.b"])
        ao = F.linear(n[:, layout.audio_indices.to(dev)].reshape(-1, D), w["audio_proj_out.w"], w["audio_proj_out.b"])
        return vo.view(B, -1, cfg.patch_dim), ao.view(B, -1, cfg.audio_in_channels)

    __call__ = forward


__all__ = ["MiniMaxH3Config", "MiniMaxH3Transformer", "get_minimax_config", "rope_table"]
