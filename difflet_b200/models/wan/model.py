"""Wan 2.1 / 2.2 video DiT on the sm_100a fused kernels.

Architecture as in the reference (``difflet/models/wan/modeling_wan.py:113-1115``)
and diffusers' ``WanTransformer3DModel``: Conv3d (1, 2, 2) patch embedding;
time embedding -> ``temb`` and a shared ``[6, D]`` projection that each block adds
to its own ``scale_shift_table``; per block: adaLN LayerNorm -> self-attention
(fused QKV, RMS q/k norm ACROSS heads, 3-axis RoPE t/h/w = 44/42/42) -> gated
residual; affine LayerNorm -> cross-attention to the text (RMS q/k norm across
heads) -> residual; adaLN LayerNorm -> GELU-tanh FFN -> gated residual; final
adaLN (table + temb) and projection, unpatchify.

B200 specifics:
  * the text context (text embedder) and every block's cross-attention K/V depend
    only on the prompt: they are computed once per generation and cached
    (``prepare_context``) instead of every step
  * all 40 blocks' modulation vectors are one f32 add per step
  * Ulysses sequence parallelism: self-attention q/k/v are scattered straight into
    the owning ranks' buffers and the attention epilogue stores rows back to their
    owners; cross-attention is local (all heads of the local queries against the
    replicated text K/V)
"""

from __future__ import annotations

import math
from dataclasses import dataclass, replace

import torch

from difflet_b200.layers.rope import multi_axis_angles, rope_tables, video_ids
from difflet_b200.ops import fused as F


@dataclass(frozen=True)
class WanConfig:
    in_channels: int = 16
    out_channels: int = 16
    hidden: int = 5120
    heads: int = 40
    head_dim: int = 128
    ffn: int = 13824
    layers: int = 40
    text_dim: int = 4096
    text_len: int = 512
    timestep_dim: int = 256
    patch: tuple = (1, 2, 2)
    theta: float = 10000.0
    eps: float = 1e-6
    vae_scale: int = 8
    vae_scale_t: int = 4

    @property
    def axes_dim(self) -> tuple:
        hw = 2 * (self.head_dim // 6)
        return (self.head_dim - 2 * hw, hw, hw)

    @property
    def patch_dim(self) -> int:
        return self.in_channels * self.patch[0] * self.patch[1] * self.patch[2]


WAN_PRESETS = {
    "wan2.1-t2v-14b": WanConfig(),
    "wan2.2-t2v-a14b": WanConfig(),  # two experts of this shape
    "wan2.1-t2v-1.3b": WanConfig(hidden=1536, heads=12, ffn=8960, layers=30),
    "tiny-wan": WanConfig(hidden=256, heads=2, ffn=512, layers=2, text_dim=64, text_len=16),
}


def get_wan_config(name: str, **kw) -> WanConfig:
    return replace(WAN_PRESETS[name], **kw)


class WanTransformer:
    def __init__(self, cfg: WanConfig, weights: dict[str, torch.Tensor]):
        self.cfg = cfg
        self.w = weights
        self.par = None
        self.tp = None  # tensor-parallel context (heads / FFN columns sharded; see parallel/tp.py)
        self._ws = {}
        self._rope = {}
        self._ones = {}

    @property
    def device(self):
        return self.w["patch.w"].device

    @property
    def dtype(self):
        return self.w["patch.w"].dtype

    def to(self, device=None, dtype=None):
        self.w = {k: (v.to(device=device) if k.endswith("sst") else v.to(device=device, dtype=dtype))
                  for k, v in self.w.items()}
        self._ws.clear()
        self._rope.clear()
        return self

    @staticmethod
    def weight_shapes(cfg: WanConfig) -> dict[str, tuple]:
        D, Fh = cfg.hidden, cfg.ffn
        s = {"patch.w": (D, cfg.patch_dim), "patch.b": (D,),
             "t.w1": (D, cfg.timestep_dim), "t.b1": (D,), "t.w2": (D, D), "t.b2": (D,),
             "tproj.w": (6 * D, D), "tproj.b": (6 * D,),
             "txt.w1": (D, cfg.text_dim), "txt.b1": (D,), "txt.w2": (D, D), "txt.b2": (D,),
             "sst": (cfg.layers, 6, D), "out.sst": (2, D),
             "final.w": (cfg.out_channels * cfg.patch[0] * cfg.patch[1] * cfg.patch[2], D),
             "final.b": (cfg.out_channels * cfg.patch[0] * cfg.patch[1] * cfg.patch[2],)}
        for i in range(cfg.layers):
            p = f"blk.{i}."
            s.update({p + "qkv.w": (3 * D, D), p + "qkv.b": (3 * D,), p + "qn": (D,), p + "kn": (D,),
                      p + "o.w": (D, D), p + "o.b": (D,), p + "n2.w": (D,), p + "n2.b": (D,),
                      p + "cq.w": (D, D), p + "cq.b": (D,), p + "ckv.w": (2 * D, D), p + "ckv.b": (2 * D,),
                      p + "cqn": (D,), p + "ckn": (D,), p + "co.w": (D, D), p + "co.b": (D,),
                      p + "up.w": (Fh, D), p + "up.b": (Fh,), p + "down.w": (D, Fh), p + "down.b": (D,)})
        return s

    @classmethod
    def random_init(cls, cfg: WanConfig, *, device="cpu", dtype=torch.float32, seed=0, std=0.02):
        g = torch.Generator(device=device).manual_seed(seed)
        w = {}
        for name, shape in cls.weight_shapes(cfg).items():
            t = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std
            if name.endswith("n") and not name.endswith(".b") or name.endswith("n2.w"):
                t = t + 1.0
            if name.endswith("sst"):
                w[name] = (torch.randn(shape, generator=g, device=device) / math.sqrt(cfg.hidden)).to(
                    torch.float64 if dtype == torch.float64 else torch.float32)
            else:
                w[name] = t.to(dtype)
        return cls(cfg, w)

    @classmethod
    def from_diffusers_state_dict(cls, cfg, sd, *, device=None, dtype=None):
        from difflet_b200.models.wan.weights import convert_diffusers_wan

        m = cls(cfg, convert_diffusers_wan(cfg, sd))
        if device is not None or dtype is not None:
            m.to(device, dtype)
        return m

    # ------------------------------------------------------------------ helpers
    def rope(self, grid):
        grid = tuple(grid)
        if grid not in self._rope:
            ids = video_ids(*grid)
            if self.dtype == torch.float64:
                ang = multi_axis_angles(ids, self.cfg.axes_dim, self.cfg.theta)
                self._rope[grid] = (ang.cos().contiguous(), ang.sin().contiguous())
            else:
                self._rope[grid] = rope_tables(ids, self.cfg.axes_dim, self.cfg.theta, device=self.device)
        return self._rope[grid]

    def _qk_norm(self, buf, q_off: int, k_off: int) -> dict:
        """Across-heads q/k RMS arguments of ``qkv_scatter``.  Under TP each rank holds D/T of
        the row: the per-row sums of squares over its heads are summed over the tp ranks first
        (a [rows, 2] f32 all-reduce), then every rank normalises with the full-row RMS."""
        if self.tp is None:
            return {"norm_mode": 2}
        width = self.cfg.hidden // self.tp.world
        rs = F.row_sumsq(buf, q_off, k_off, width)
        self.tp.allreduce_rows(rs)
        return {"norm_mode": 3, "row_sumsq": rs, "norm_total": self.cfg.hidden}

    def _row_linear(self, xin, wt, bias, out, gate, rpb):
        """Output projections fused with ``out += gate * (.)`` (row-parallel under TP)."""
        if self.tp is not None:
            self.tp.row_linear(xin, wt, bias, out=out, gate=gate, resid=out, rows_per_batch=rpb)
        else:
            F.linear(xin, wt, bias, out=out, gate=gate, resid=out, rows_per_batch=rpb)

    def _ones_gate(self, B):
        if B not in self._ones:
            dt = torch.float64 if self.dtype == torch.float64 else torch.float32
            self._ones[B] = torch.ones(B, self.cfg.hidden, device=self.device, dtype=dt)
        return self._ones[B]

    def _workspace(self, B, S_loc):
        key = (B, S_loc)
        if key in self._ws:
            return self._ws[key]
        cfg, par, tp = self.cfg, self.par, self.tp
        D, H, dh = cfg.hidden, cfg.heads, cfg.head_dim
        T = tp.world if tp is not None else 1
        Dl, Ht = D // T, H // T  # this rank's attention columns / heads
        world = par.world if par is not None else 1
        S = S_loc * world
        dev, dt = self.device, self.dtype
        e = lambda *s: torch.empty(s, device=dev, dtype=dt)  # noqa: E731
        pe = (lambda *s: par.empty(s, dt)) if par is not None else e  # noqa: E731
        if par is not None:  # context parallelism splits this rank's tensor-parallel heads
            par.check_heads(Ht)
        # the residual stream is written by every rank's TP reducer: symmetric memory under TP
        x = tp.empty((B * S_loc, D), dt) if tp is not None else e(B * S_loc, D)
        ws = {"S": S, "x": x, "norm": e(B * S_loc, D), "qkv": e(B * S_loc, 3 * Dl),
              "mlp": e(B * S_loc, cfg.ffn // T), "cq": e(B, Ht, S_loc, dh), "cqin": e(B * S_loc, Dl),
              "cattn": e(B, S_loc, Dl), "attn": pe(B, S_loc, Dl)}
        if par is not None:  # the CP mode decides the q/k/v layout
            ws["q"], ws["k"], ws["v"] = par.layout(B, Ht, dh, S_loc, S, dt)
        else:
            ws["q"], ws["k"], ws["v"] = e(B, Ht, S, dh), e(B, Ht, S, dh), e(B, Ht, S, dh)
        self._ws[key] = ws
        return ws

    # ------------------------------------------------------------------ text / time
    def prepare_context(self, text: torch.Tensor, text_valid=None):
        """Text embedder + every block's cross-attention K/V (normed): computed once per
        prompt.  text [B, L, text_dim] -> list of (k, v) [B, H, L, dh]."""
        cfg, w = self.cfg, self.w
        B, L, _ = text.shape
        T = self.tp.world if self.tp is not None else 1
        D, H, dh = cfg.hidden // T, cfg.heads // T, cfg.head_dim  # this rank's columns / heads
        if text_valid is not None:  # zero the padding rows (reference pad-zeroing)
            mask = torch.arange(L, device=text.device)[None, :] < text_valid.to(text.device)[:, None]
            text = text * mask[..., None].to(text.dtype)
        h = F.linear(text.reshape(B * L, -1), w["txt.w1"], w["txt.b1"], act="gelu")
        ctx = F.linear(h, w["txt.w2"], w["txt.b2"])
        kvs = []
        kv = torch.empty(B * L, 2 * D, device=ctx.device, dtype=ctx.dtype)
        for i in range(cfg.layers):
            p = f"blk.{i}."
            F.linear(ctx, w[p + "ckv.w"], w[p + "ckv.b"], out=kv)
            k = torch.empty(B, H, L, dh, device=ctx.device, dtype=ctx.dtype)
            v = torch.empty_like(k)
            F.qkv_scatter(kv, q_off=-1, k_off=0, v_off=D, S_src=L, H=H, dh=dh, q_dst=None, k_dst=[k], v_dst=[v],
                          S_dst=L, wk=w[p + "ckn"], eps=cfg.eps, heads_per_rank=H, **self._qk_norm(kv, -1, 0))
            kvs.append((k, v))
        return kvs

    def time_embed(self, timestep):
        """timestep [B] in [0, 1000] -> (temb [B, D] f32, per-block modulation [L, B, 6, D] f32)."""
        cfg, w = self.cfg, self.w
        tf = F.timestep_embed(timestep, cfg.timestep_dim)
        h = F.gemv(w["t.w1"], tf, w["t.b1"], silu_out=True)
        temb = F.gemv(w["t.w2"], h, w["t.b2"])
        tproj = F.gemv(w["tproj.w"], temb, w["tproj.b"], silu_in=True)
        B = temb.shape[0]
        mods = (w["sst"][:, None] + tproj.view(1, B, 6, cfg.hidden).to(w["sst"].dtype)).contiguous()
        return temb, mods

    # ------------------------------------------------------------------ forward
    def forward(self, x_tokens, timestep, context, *, grid, mods=None, temb=None, out=None):
        """x_tokens [B, S(local), C*pt*ph*pw]; timestep [B] in [0, 1000]; context = the
        cached per-block (k, v) from ``prepare_context``; grid = (t, h, w) token grid.
        ``out`` (optional, [B, S(local), out_dim] bf16): where the final projection stores the
        prediction (a CFG-parallel exchange buffer)."""
        cfg, w, par, tp = self.cfg, self.w, self.par, self.tp
        B, S_loc, _ = x_tokens.shape
        T = tp.world if tp is not None else 1
        D, H, dh = cfg.hidden // T, cfg.heads // T, cfg.head_dim  # this rank's columns / heads
        world = par.world if par is not None else 1
        rank = par.rank if par is not None else 0
        Hl = par.heads_local(H) if par is not None else H
        ws = self._workspace(B, S_loc)
        S = ws["S"]
        cos, sin = self.rope(grid)
        if mods is None:
            temb, mods = self.time_embed(timestep)
        eps = cfg.eps
        x = ws["x"]
        F.linear(x_tokens.reshape(B * S_loc, -1), w["patch.w"], w["patch.b"], out=x)
        norm, q, k, v = ws["norm"], ws["q"], ws["k"], ws["v"]
        pos = rank * S_loc
        ones = self._ones_gate(B)

        if par is not None:
            tgt = par.scatter_kwargs(q, k, v, 0, pos, S_loc, S, H)
        else:
            tgt = dict(q_dst=[q], k_dst=[k], v_dst=[v], S_dst=S, seq_off=pos, heads_per_rank=H)

        for i in range(cfg.layers):
            p = f"blk.{i}."
            m = mods[i]  # [B, 6, D]: shift, scale, gate, c_shift, c_scale, c_gate
            F.ln_modulate(x, shift=m[:, 0], scale=m[:, 1], eps=eps, rows_per_batch=S_loc, out=norm)
            F.linear(norm, w[p + "qkv.w"], w[p + "qkv.b"], out=ws["qkv"])
            F.qkv_scatter(ws["qkv"], q_off=0, k_off=D, v_off=2 * D, S_src=S_loc, H=H, dh=dh, **tgt,
                          wq=w[p + "qn"], wk=w[p + "kn"], eps=eps, cos=cos, sin=sin, rope_pos_off=pos,
                          **self._qk_norm(ws["qkv"], 0, D))
            self._self_attention(ws, B, S_loc, Hl)
            self._row_linear(ws["attn"].view(B * S_loc, D), w[p + "o.w"], w[p + "o.b"], x, m[:, 2], S_loc)
            # cross-attention (local queries, all heads, cached text K/V)
            F.ln_modulate(x, w=w[p + "n2.w"], b=w[p + "n2.b"], eps=eps, out=norm)
            F.linear(norm, w[p + "cq.w"], w[p + "cq.b"], out=ws["cqin"])
            F.qkv_scatter(ws["cqin"], q_off=0, k_off=-1, v_off=-1, S_src=S_loc, H=H, dh=dh, q_dst=[ws["cq"]],
                          k_dst=None, v_dst=None, S_dst=S_loc, wq=w[p + "cqn"], eps=eps, heads_per_rank=H,
                          **self._qk_norm(ws["cqin"], 0, -1))
            ck, cv = context[i]
            F.attention(ws["cq"], ck, cv, 1.0 / math.sqrt(dh), out=ws["cattn"].view(B, S_loc, H, dh).permute(0, 2, 1, 3))
            self._row_linear(ws["cattn"].view(B * S_loc, D), w[p + "co.w"], w[p + "co.b"], x, ones, S_loc)
            # feed-forward
            F.ln_modulate(x, shift=m[:, 3], scale=m[:, 4], eps=eps, rows_per_batch=S_loc, out=norm)
            F.linear(norm, w[p + "up.w"], w[p + "up.b"], out=ws["mlp"], act="gelu")
            self._row_linear(ws["mlp"], w[p + "down.w"], w[p + "down.b"], x, m[:, 5], S_loc)
        if temb is None:
            temb, _ = self.time_embed(timestep)
        fm = (w["out.sst"][None] + temb[:, None].to(w["out.sst"].dtype)).contiguous()  # [B, 2, D]: shift, scale
        F.ln_modulate(x, shift=fm[:, 0], scale=fm[:, 1], eps=eps, rows_per_batch=S_loc, out=norm)
        out = F.linear(norm, w["final.w"], w["final.b"], out=None if out is None else out.view(B * S_loc, -1))
        return out.view(B, S_loc, -1)

    __call__ = forward

    def _self_attention(self, ws, B, S_loc, Hl):
        par = self.par
        q, k, v = ws["q"], ws["k"], ws["v"]
        dh = self.cfg.head_dim
        scale = 1.0 / math.sqrt(dh)
        if par is not None:
            target = ws["attn"].view(B * S_loc, -1)
            par.attention(q, k, v, scale, target, B, 0, S_loc, target.shape[1])
            return
        S = q.shape[2]
        F.attention(q, k, v, scale, out=ws["attn"].view(B, S, Hl, dh).permute(0, 2, 1, 3))


def patchify(lat: torch.Tensor, patch=(1, 2, 2)) -> torch.Tensor:
    """[B, C, T, H, W] -> [B, (T/pt)(H/ph)(W/pw), C pt ph pw] (Conv3d kernel = stride order)."""
    B, C, T, Hh, Ww = lat.shape
    pt, ph, pw = patch
    x = lat.view(B, C, T // pt, pt, Hh // ph, ph, Ww // pw, pw)
    return x.permute(0, 2, 4, 6, 1, 3, 5, 7).reshape(B, (T // pt) * (Hh // ph) * (Ww // pw), C * pt * ph * pw)


def unpatchify(tok: torch.Tensor, grid, patch=(1, 2, 2), channels=16) -> torch.Tensor:
    B = tok.shape[0]
    t, h, w = grid
    pt, ph, pw = patch
    x = tok.view(B, t, h, w, channels, pt, ph, pw)
    return x.permute(0, 4, 1, 5, 2, 6, 3, 7).reshape(B, channels, t * pt, h * ph, w * pw)
