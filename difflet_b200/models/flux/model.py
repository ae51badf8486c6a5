"""FLUX MMDiT, written for the sm_100a fused kernels.

Architecture as in the reference (``difflet/models/flux/modeling_flux.py:219-613``,
double block ``:736-867``, single block ``:616-733``) and diffusers'
``FluxTransformer2DModel``: 19 double-stream blocks (separate text / image
weights, joint attention over ``[text ; image]``), 38 single-stream blocks
(parallel attention + MLP, one output projection), adaLN-Zero modulation from
``temb = t_emb + guidance_emb + pooled_text_emb``, per-head RMS q/k norm and
3-axis RoPE.

B200 layout (weights are converted once at load time):
  * every block's adaLN linear is one row range of a single ``[N_mod, D]``
    matrix -> one GEMV per step produces all shift / scale / gate vectors (f32)
  * double block: fused ``[3D, D]`` QKV per stream; q/k RMSNorm + RoPE +
    head-major scatter into one joint q/k/v buffer in a single pass (the text
    rows land at positions [0, S_txt), image rows after them)
  * single block: one ``[7D, D]`` GEMM producing ``[q | mlp | k | v]`` with
    GELU-tanh applied to the mlp column window; attention writes its output
    back into the q slot, so ``proj_out`` reads the contiguous ``[attn | mlp]``
    view (row stride 7D) -- the reference's ``cat`` disappears
  * every output projection fuses bias + ``residual + gate * y`` in the GEMM
    epilogue (in place on the residual stream)
The same code runs on CPU tensors through the PyTorch oracle of each op.
Sequence parallelism (Ulysses) plugs in through ``par`` (see
``difflet_b200/parallel/ulysses.py``): q/k/v scatter and the attention output
go straight to the owning ranks' symmetric buffers.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from difflet_b200.layers.rope import flux_ids, rope_tables
from difflet_b200.models.flux.config import FluxConfig
from difflet_b200.ops import fused as F


class FluxTransformer:
    def __init__(self, config: FluxConfig, weights: dict[str, torch.Tensor]):
        self.cfg = config
        self.w = weights
        self._ws = {}
        self._rope = {}
        self.par = None  # sequence-parallel context (None = single device)

    # ------------------------------------------------------------------ weights
    @property
    def device(self):
        return next(iter(self.w.values())).device

    @property
    def dtype(self):
        return self.w["x_embed.w"].dtype

    def to(self, device=None, dtype=None):
        self.w = {k: v.to(device=device, dtype=dtype if v.is_floating_point() else None) for k, v in self.w.items()}
        self._ws.clear()
        self._rope.clear()
        return self

    def named_tensors(self):
        return self.w.items()

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.w.values())

    @staticmethod
    def weight_shapes(cfg: FluxConfig) -> dict[str, tuple]:
        D, F_, dh = cfg.hidden, cfg.mlp_hidden, cfg.head_dim
        s = {
            "x_embed.w": (D, cfg.in_channels), "x_embed.b": (D,),
            "ctx_embed.w": (D, cfg.text_dim), "ctx_embed.b": (D,),
            "t_embed.w1": (D, cfg.timestep_dim), "t_embed.b1": (D,), "t_embed.w2": (D, D), "t_embed.b2": (D,),
            "p_embed.w1": (D, cfg.pooled_dim), "p_embed.b1": (D,), "p_embed.w2": (D, D), "p_embed.b2": (D,),
            "mod.w": (cfg.mod_rows, D), "mod.b": (cfg.mod_rows,),
            "final.w": (cfg.out_channels, D), "final.b": (cfg.out_channels,),
        }
        if cfg.guidance_embed:
            s.update({"g_embed.w1": (D, cfg.timestep_dim), "g_embed.b1": (D,), "g_embed.w2": (D, D), "g_embed.b2": (D,)})
        for i in range(cfg.double_blocks):
            p = f"double.{i}."
            for st in ("img", "txt"):
                s[p + st + "_qkv.w"] = (3 * D, D)
                s[p + st + "_qkv.b"] = (3 * D,)
                s[p + st + "_qnorm"] = (dh,)
                s[p + st + "_knorm"] = (dh,)
                s[p + st + "_out.w"] = (D, D)
                s[p + st + "_out.b"] = (D,)
                s[p + st + "_up.w"] = (F_, D)
                s[p + st + "_up.b"] = (F_,)
                s[p + st + "_down.w"] = (D, F_)
                s[p + st + "_down.b"] = (D,)
        for j in range(cfg.single_blocks):
            p = f"single.{j}."
            s[p + "fused.w"] = (3 * D + F_, D)
            s[p + "fused.b"] = (3 * D + F_,)
            s[p + "qnorm"] = (dh,)
            s[p + "knorm"] = (dh,)
            s[p + "proj.w"] = (D, D + F_)
            s[p + "proj.b"] = (D,)
        return s

    @classmethod
    def random_init(cls, cfg: FluxConfig, *, device="cpu", dtype=torch.float32, seed: int = 0, std: float = 0.02):
        """Seeded N(0, std) weights (RMSNorm gains 1 + N(0, std)), generated on ``device``."""
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        w = {}
        for name, shape in cls.weight_shapes(cfg).items():
            t = torch.randn(shape, generator=g, device=device, dtype=torch.float32 if dtype == torch.float64 else dtype)
            t.mul_(std)
            if name.endswith("norm"):
                t.add_(1.0)
            w[name] = t.to(dtype)
        return cls(cfg, w)

    @classmethod
    def from_diffusers_state_dict(cls, cfg: FluxConfig, sd: dict[str, torch.Tensor], *, device=None, dtype=None):
        """Convert a diffusers ``FluxTransformer2DModel`` state dict to the fused layout."""
        from difflet_b200.models.flux.weights import convert_diffusers_flux

        w = convert_diffusers_flux(cfg, sd)
        m = cls(cfg, w)
        if device is not None or dtype is not None:
            m.to(device, dtype)
        return m

    # ------------------------------------------------------------------ buffers
    def _workspace(self, B: int, S_txt: int, S_img: int):
        key = (B, S_txt, S_img)
        ws = self._ws.get(key)
        if ws is not None:
            return ws
        cfg = self.cfg
        D, F_, H, dh = cfg.hidden, cfg.mlp_hidden, cfg.heads, cfg.head_dim
        dev, dt = self.device, self.dtype
        par = self.par
        world = par.world if par is not None else 1
        S_txt_g, S_img_g = S_txt * world, S_img * world
        S = S_txt_g + S_img_g
        S_loc = S_txt + S_img
        e = lambda *shape: torch.empty(shape, device=dev, dtype=dt)  # noqa: E731
        ws = {"S": S, "S_txt_g": S_txt_g, "S_img_g": S_img_g}
        ws["x"] = e(B, S_loc, D)  # residual stream [txt_local ; img_local] per batch
        if B == 1:
            ws["x_txt"] = ws["x"][0, :S_txt]
            ws["x_img"] = ws["x"][0, S_txt:]
        else:
            ws["x_txt"] = e(B * S_txt, D)
            ws["x_img"] = e(B * S_img, D)
        ws["norm"] = e(B * S_loc, D)
        ws["qkv_img"] = e(B * S_img, 3 * D)
        ws["qkv_txt"] = e(B * S_txt, 3 * D)
        ws["mlp"] = e(B * max(S_img, S_txt), F_)
        Hl = H // world
        # buffers that peers store into (q/k/v, attention outputs) come from the
        # sequence-parallel context's symmetric heap
        pe = (lambda *shape: par.empty(shape, dt)) if par is not None else e  # noqa: E731
        if par is not None:
            par.check_heads(H)
        ws["fused"] = pe(B * S_loc, 3 * D + F_)
        ws["q"] = pe(B, Hl, S, dh)
        ws["k"] = pe(B, Hl, S, dh)
        ws["v"] = pe(B, Hl, S, dh)
        ws["attn"] = pe(B, S_loc, D)
        self._ws[key] = ws
        return ws

    def rope(self, S_txt: int, h_tok: int, w_tok: int):
        key = (S_txt, h_tok, w_tok)
        if key not in self._rope:
            ids = flux_ids(S_txt, h_tok, w_tok)
            cos, sin = rope_tables(ids, self.cfg.axes_dim, self.cfg.theta, device=self.device)
            if self.dtype == torch.float64:  # float64 oracle: keep the tables exact
                from difflet_b200.layers.rope import multi_axis_angles

                ang = multi_axis_angles(ids, self.cfg.axes_dim, self.cfg.theta)
                cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
            self._rope[key] = (cos, sin)
        return self._rope[key]

    # ------------------------------------------------------------------ pieces
    def temb(self, timestep: torch.Tensor, guidance: torch.Tensor | None, pooled: torch.Tensor) -> torch.Tensor:
        """temb [B, D] (f32): t-embedder + guidance-embedder + pooled-text embedder."""
        cfg, w = self.cfg, self.w
        tf = F.timestep_embed(timestep * 1000.0, cfg.timestep_dim)
        h = F.gemv(w["t_embed.w1"], tf, w["t_embed.b1"], silu_out=True)
        temb = F.gemv(w["t_embed.w2"], h, w["t_embed.b2"])
        if cfg.guidance_embed:
            g = guidance if guidance is not None else torch.full_like(timestep, 3.5)
            gf = F.timestep_embed(g * 1000.0, cfg.timestep_dim)
            h = F.gemv(w["g_embed.w1"], gf, w["g_embed.b1"], silu_out=True)
            temb = temb + F.gemv(w["g_embed.w2"], h, w["g_embed.b2"])
        h = F.gemv(w["p_embed.w1"], pooled, w["p_embed.b1"], silu_out=True)
        temb = temb + F.gemv(w["p_embed.w2"], h, w["p_embed.b2"])
        return temb

    def modulation(self, temb: torch.Tensor) -> torch.Tensor:
        """All blocks' adaLN vectors in one GEMV: f32 [B, N_mod] = W_mod silu(temb) + b."""
        par = self.par
        if par is not None and hasattr(par, "shard_gemv") and temb.is_cuda:
            out = par.shard_gemv(self.w["mod.w"], temb, self.w["mod.b"], silu_in=True)
            if out is not None:
                return out
        return F.gemv(self.w["mod.w"], temb, self.w["mod.b"], silu_in=True)

    # ------------------------------------------------------------------ forward
    def forward(self, x_tokens, txt, pooled, timestep, guidance=None, *, img_hw=None, mod=None):
        """x_tokens [B, S_img(local), in_ch]; txt [B, S_txt(local), text_dim]; pooled [B, pooled_dim];
        timestep [B] in [0, 1]; returns the velocity [B, S_img(local), out_ch]."""
        cfg, w = self.cfg, self.w
        B, S_img, _ = x_tokens.shape
        S_txt = txt.shape[1]
        D, H, dh, F_ = cfg.hidden, cfg.heads, cfg.head_dim, cfg.mlp_hidden
        ws = self._workspace(B, S_txt, S_img)
        par = self.par
        world = par.world if par is not None else 1
        rank = par.rank if par is not None else 0
        S, S_txt_g = ws["S"], ws["S_txt_g"]
        S_img_g = ws["S_img_g"]
        if img_hw is None:
            side = int(round(math.sqrt(S_img_g)))
            img_hw = (side, S_img_g // side)
        cos, sin = self.rope(S_txt_g, img_hw[0], img_hw[1])
        Hl = H // world
        if mod is None:
            mod = self.modulation(self.temb(timestep, guidance, pooled))
        eps = cfg.eps

        x_img, x_txt = ws["x_img"], ws["x_txt"]
        # embedders
        F.linear(x_tokens.reshape(B * S_img, -1), w["x_embed.w"], w["x_embed.b"], out=x_img.reshape(B * S_img, D))
        F.linear(txt.reshape(B * S_txt, -1), w["ctx_embed.w"], w["ctx_embed.b"], out=x_txt.reshape(B * S_txt, D))
        x_img2 = x_img.reshape(B * S_img, D)
        x_txt2 = x_txt.reshape(B * S_txt, D)
        norm = ws["norm"]
        q, k, v = ws["q"], ws["k"], ws["v"]
        txt_pos = rank * S_txt       # global position of this rank's first text row
        img_pos = S_txt_g + rank * S_img

        def dst(t):
            return par.peer_views(t) if par is not None else [t]

        def mslice(off):
            return mod[:, off:off + D]

        for i in range(cfg.double_blocks):
            p = f"double.{i}."
            for st, xs, n_rows, qkv_buf, pos in (("img", x_img2, S_img, ws["qkv_img"], img_pos),
                                                  ("txt", x_txt2, S_txt, ws["qkv_txt"], txt_pos)):
                o = cfg.double_mod_offset(i, st)
                nb = norm[: B * n_rows]
                F.ln_modulate(xs, shift=mslice(o), scale=mslice(o + D), eps=eps, rows_per_batch=n_rows, out=nb)
                F.linear(nb, w[p + st + "_qkv.w"], w[p + st + "_qkv.b"], out=qkv_buf)
                F.qkv_scatter(qkv_buf, q_off=0, k_off=D, v_off=2 * D, S_src=n_rows, H=H, dh=dh,
                              q_dst=dst(q), k_dst=dst(k), v_dst=dst(v), S_dst=S, seq_off=pos,
                              norm_mode=1, wq=w[p + st + "_qnorm"], wk=w[p + st + "_knorm"], eps=eps,
                              cos=cos, sin=sin, rope_pos_off=pos, heads_per_rank=Hl)
            self._attention(ws, B, S_txt, S_img, D, Hl, dh)
            for st, xs, n_rows, rows in (("img", x_img2, S_img, slice(S_txt, S_txt + S_img)),
                                         ("txt", x_txt2, S_txt, slice(0, S_txt))):
                o = cfg.double_mod_offset(i, st)
                self._rows_gemm(ws["attn"], rows, B, n_rows, w[p + st + "_out.w"], w[p + st + "_out.b"],
                                xs, mslice(o + 2 * D))
                nb = norm[: B * n_rows]
                F.ln_modulate(xs, shift=mslice(o + 3 * D), scale=mslice(o + 4 * D), eps=eps, rows_per_batch=n_rows, out=nb)
                mb = ws["mlp"][: B * n_rows]
                F.linear(nb, w[p + st + "_up.w"], w[p + st + "_up.b"], out=mb, act="gelu")
                F.linear(mb, w[p + st + "_down.w"], w[p + st + "_down.b"], out=xs, gate=mslice(o + 5 * D),
                         resid=xs, rows_per_batch=n_rows)

        # double -> single: the residual stream becomes [txt ; img] per batch
        if B > 1:
            ws["x"][:, :S_txt] = x_txt.view(B, S_txt, D)
            ws["x"][:, S_txt:] = x_img.view(B, S_img, D)
        S_loc = S_txt + S_img
        x2 = ws["x"].view(B * S_loc, D)
        fused = ws["fused"]
        for j in range(cfg.single_blocks):
            p = f"single.{j}."
            o = cfg.single_mod_offset(j)
            F.ln_modulate(x2, shift=mslice(o), scale=mslice(o + D), eps=eps, rows_per_batch=S_loc, out=norm)
            F.linear(norm, w[p + "fused.w"], w[p + "fused.b"], out=fused, act="gelu", act_lo=D, act_hi=D + F_)
            # columns: [q | mlp | k | v]; text rows first within each batch
            for b in range(B):
                rows = fused[b * S_loc:(b + 1) * S_loc]
                for seg, n_rows, pos, base in (("txt", S_txt, txt_pos, 0), ("img", S_img, img_pos, S_txt)):
                    F.qkv_scatter(rows[base:base + n_rows], q_off=0, k_off=D + F_, v_off=2 * D + F_,
                                  S_src=n_rows, H=H, dh=dh, q_dst=dst(q[b:b + 1]), k_dst=dst(k[b:b + 1]),
                                  v_dst=dst(v[b:b + 1]), S_dst=S, seq_off=pos, norm_mode=1,
                                  wq=w[p + "qnorm"], wk=w[p + "knorm"], eps=eps, cos=cos, sin=sin,
                                  rope_pos_off=pos, heads_per_rank=Hl)
            self._attention(ws, B, S_txt, S_img, D, Hl, dh, out_rows=fused)
            F.linear(fused[:, : D + F_], w[p + "proj.w"], w[p + "proj.b"], out=x2, gate=mslice(o + 2 * D),
                     resid=x2, rows_per_batch=S_loc)

        # final adaLN-continuous (scale, shift) on the image rows + projection
        o = cfg.final_mod_offset()
        out = torch.empty(B * S_img, cfg.out_channels, device=x_tokens.device, dtype=x_tokens.dtype)
        for b in range(B):
            xi = ws["x"][b, S_txt:]
            nb = norm[:S_img]
            F.ln_modulate(xi, shift=mod[b:b + 1, o + D:o + 2 * D], scale=mod[b:b + 1, o:o + D], eps=eps, out=nb)
            F.linear(nb, w["final.w"], w["final.b"], out=out[b * S_img:(b + 1) * S_img])
        return out.view(B, S_img, cfg.out_channels)

    __call__ = forward

    # ------------------------------------------------------------------ helpers
    def _attention(self, ws, B, S_txt, S_img, D, Hl, dh, out_rows=None):
        """Joint attention over the full sequence; output lands token-major in
        ``ws['attn']`` (double blocks) or in the q slot of ``out_rows`` (single)."""
        par = self.par
        q, k, v = ws["q"], ws["k"], ws["v"]
        scale = 1.0 / math.sqrt(dh)
        if par is not None:
            target = ws["attn"].view(B * (S_txt + S_img), D) if out_rows is None else out_rows
            par.attention(q, k, v, scale, target, B, S_txt, S_img, target.shape[1])
            return
        S = q.shape[2]
        if out_rows is None:
            o = ws["attn"].view(B, S, Hl, dh).permute(0, 2, 1, 3)
        else:
            ld = out_rows.shape[1]
            o = out_rows.as_strided((B, Hl, S, dh), (S * ld, dh, ld, 1))
        F.attention(q, k, v, scale, out=o)

    @staticmethod
    def _rows_gemm(attn, rows, B, n_rows, wt, bias, xs, gate):
        """Output projection of one stream's rows of the attention output, fused with
        ``x += gate * (o W^T + b)``."""
        D = xs.shape[-1]
        if B == 1:
            F.linear(attn[0, rows], wt, bias, out=xs, gate=gate, resid=xs, rows_per_batch=n_rows)
            return
        for b in range(B):
            xb = xs[b * n_rows:(b + 1) * n_rows]
            F.linear(attn[b, rows], wt, bias, out=xb, gate=gate[b:b + 1], resid=xb, rows_per_batch=n_rows)


def pack_latents(lat: torch.Tensor, patch: int = 2) -> torch.Tensor:
    """[B, C, H, W] -> [B, (H/p)(W/p), C p p] (channel-major within a patch)."""
    B, C, Hh, Ww = lat.shape
    x = lat.view(B, C, Hh // patch, patch, Ww // patch, patch)
    return x.permute(0, 2, 4, 1, 3, 5).reshape(B, (Hh // patch) * (Ww // patch), C * patch * patch)


def unpack_latents(tok: torch.Tensor, h: int, w: int, patch: int = 2) -> torch.Tensor:
    """[B, (H/p)(W/p), C p p] -> [B, C, H, W]."""
    B, _, Cpp = tok.shape
    C = Cpp // (patch * patch)
    x = tok.view(B, h // patch, w // patch, C, patch, patch)
    return x.permute(0, 3, 1, 4, 2, 5).reshape(B, C, h, w)
