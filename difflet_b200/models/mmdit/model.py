"""MMDiT on the sm_100a fused kernels: FLUX, HunyuanVideo and Qwen-Image.

Architecture (reference: FLUX ``difflet/models/flux/modeling_flux.py:219-949``,
HunyuanVideo ``difflet/models/hunyuan_video/modeling_hunyuan_video.py:316-1390``,
Qwen-Image ``difflet/models/qwen_image/modeling_qwen_image.py:155-819``):
dual-stream blocks (separate text / image weights, joint attention over the
concatenated sequence), optional single-stream blocks (parallel attention + MLP
with one output projection), adaLN-Zero modulation from ``temb``, per-head RMS
q/k norm, multi-axis RoPE.

B200 layout (weights are converted once at load time):
  * every block's adaLN linear is a row range of one ``[N_mod, D]`` matrix -> one
    GEMV per step (row-sharded over ranks under sequence parallelism) or one
    GEMM per image for all steps
  * dual block: fused ``[3D, D]`` QKV per stream; q/k RMSNorm + RoPE + head-major
    scatter straight into the joint q/k/v buffers (the Ulysses all-to-all when
    the buffers are peers')
  * single block: one ``[7D, D]`` GEMM producing ``[q | mlp | k | v]`` with
    GELU-tanh on the mlp window; attention writes into the q slot, so the output
    projection reads ``[attn | mlp]`` in place (row stride 7D)
  * output projections fuse bias + ``residual + gate * y`` in the GEMM epilogue
The joint sequence is ``[seg0 ; seg1]`` (FLUX / Qwen: text first; HunyuanVideo:
video first); a right-padded text stream at the end becomes the attention key
window ``[0, S_img + n_valid)``.  The same code runs on CPU tensors (oracle).
"""

from __future__ import annotations

import math

import torch

from difflet_b200.layers.rope import joint_ids, multi_axis_angles, rope_tables
from difflet_b200.models.mmdit.config import MMDiTConfig
from difflet_b200.ops import fused as F


class MMDiT:
    def __init__(self, config: MMDiTConfig, weights: dict[str, torch.Tensor]):
        self.cfg = config
        self.w = weights
        self._ws = {}
        self._rope = {}
        self.par = None  # sequence-parallel context (None = single device)
        self.tp = None   # tensor-parallel context: weights hold this rank's heads / MLP columns

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
    def weight_shapes(cfg: MMDiTConfig) -> dict[str, tuple]:
        D, F_, dh = cfg.hidden, cfg.mlp_hidden, cfg.head_dim
        s = {
            "x_embed.w": (D, cfg.in_channels), "x_embed.b": (D,),
            "t_embed.w1": (D, cfg.timestep_dim), "t_embed.b1": (D,), "t_embed.w2": (D, D), "t_embed.b2": (D,),
            "mod.w": (cfg.mod_rows, D), "mod.b": (cfg.mod_rows,),
            "final.w": (cfg.out_channels, D), "final.b": (cfg.out_channels,),
        }
        if cfg.refiner_layers == 0:
            s.update({"ctx_embed.w": (D, cfg.text_dim), "ctx_embed.b": (D,)})
        if cfg.pooled_dim:
            s.update({"p_embed.w1": (D, cfg.pooled_dim), "p_embed.b1": (D,), "p_embed.w2": (D, D), "p_embed.b2": (D,)})
        if cfg.guidance_embed:
            s.update({"g_embed.w1": (D, cfg.timestep_dim), "g_embed.b1": (D,), "g_embed.w2": (D, D), "g_embed.b2": (D,)})
        if cfg.txt_norm:
            s["txt_norm"] = (cfg.text_dim,)
        if cfg.refiner_layers:
            s.update({"ref.t.w1": (D, cfg.timestep_dim), "ref.t.b1": (D,), "ref.t.w2": (D, D), "ref.t.b2": (D,),
                      "ref.p.w1": (D, cfg.text_dim), "ref.p.b1": (D,), "ref.p.w2": (D, D), "ref.p.b2": (D,),
                      "ref.proj.w": (D, cfg.text_dim), "ref.proj.b": (D,)})
            for i in range(cfg.refiner_layers):
                p = f"ref.{i}."
                s.update({p + "n1.w": (D,), p + "n1.b": (D,), p + "qkv.w": (3 * D, D), p + "qkv.b": (3 * D,),
                          p + "out.w": (D, D), p + "out.b": (D,), p + "n2.w": (D,), p + "n2.b": (D,),
                          p + "up.w": (F_, D), p + "up.b": (F_,), p + "down.w": (D, F_), p + "down.b": (D,),
                          p + "ada.w": (2 * D, D), p + "ada.b": (2 * D,)})
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
    def random_init(cls, cfg: MMDiTConfig, *, device="cpu", dtype=torch.float32, seed: int = 0, std: float = 0.02):
        """Seeded N(0, std) weights (norm gains 1 + N(0, std)), generated on ``device``."""
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        w = {}
        for name, shape in cls.weight_shapes(cfg).items():
            t = torch.randn(shape, generator=g, device=device, dtype=torch.float32 if dtype == torch.float64 else dtype)
            t.mul_(std)
            if name.endswith("norm") or name.endswith("n1.w") or name.endswith("n2.w"):
                t.add_(1.0)
            w[name] = t.to(dtype)
        return cls(cfg, w)

    @classmethod
    def from_diffusers_state_dict(cls, cfg: MMDiTConfig, sd: dict[str, torch.Tensor], *, device=None, dtype=None):
        from difflet_b200.models.mmdit.weights import convert_diffusers

        m = cls(cfg, convert_diffusers(cfg, sd))
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
        tp = self.tp
        T = tp.world if tp is not None else 1
        Dl, Fl = D // T, F_ // T  # this rank's attention / MLP columns
        world = par.world if par is not None else 1
        S_txt_g, S_img_g = S_txt * world, S_img * world
        S = S_txt_g + S_img_g
        S_loc = S_txt + S_img
        n = {"txt": S_txt, "img": S_img}
        ng = {"txt": S_txt_g, "img": S_img_g}
        s0, s1 = cfg.streams
        e = lambda *shape: torch.empty(shape, device=dev, dtype=dt)  # noqa: E731
        ws = {"S": S, "S_txt_g": S_txt_g, "S_img_g": S_img_g, "n": n,
              # local row offset of each stream inside [seg0_local ; seg1_local]
              "row": {s0: 0, s1: n[s0]},
              # global position of this rank's first row of each stream
              "pos": {s0: (par.rank if par else 0) * n[s0], s1: ng[s0] + (par.rank if par else 0) * n[s1]}}
        # residual stream [seg0_local ; seg1_local] per batch (replicated in peer memory under TP)
        ws["x"] = tp.empty((B, S_loc, D), dt) if tp is not None else e(B, S_loc, D)
        if B == 1:
            for st in ("txt", "img"):
                r0 = ws["row"][st]
                ws["x_" + st] = ws["x"][0, r0:r0 + n[st]]
        else:
            xe = (lambda *shape: tp.empty(shape, dt)) if tp is not None else e  # noqa: E731
            ws["x_txt"] = xe(B * S_txt, D)
            ws["x_img"] = xe(B * S_img, D)
        sp = tp is not None and tp.sp
        ws["norm"] = tp.empty((B * S_loc, D), dt) if sp else e(B * S_loc, D)  # all-gathered under SP
        ws["qkv_img"] = e(B * S_img, 3 * Dl)
        ws["qkv_txt"] = e(B * S_txt, 3 * Dl)
        ws["mlp"] = e(B * S_loc, Fl)  # [img rows ; txt rows]: both streams' MLPs live at once
        pe = (lambda *shape: par.empty(shape, dt)) if par is not None else e  # noqa: E731
        if par is not None:  # context parallelism splits this rank's tensor-parallel heads
            par.check_heads(H // T)
        ws["fused"] = pe(B * S_loc, 3 * Dl + Fl) if cfg.single_blocks else None
        if par is not None:  # the CP mode decides the q/k/v layout (heads x full sequence, or local rows)
            ws["q"], ws["k"], ws["v"] = par.layout(B, H // T, dh, S_loc, S, dt)
        else:
            Ht = H // T
            ws["q"], ws["k"], ws["v"] = e(B, Ht, S, dh), e(B, Ht, S, dh), e(B, Ht, S, dh)
        ws["attn"] = pe(B, S_loc, Dl)
        self._ws[key] = ws
        return ws

    def rope(self, S_txt_g: int, grid: tuple):
        key = (S_txt_g, tuple(grid))
        if key not in self._rope:
            ids = joint_ids(self.cfg.family, S_txt_g, grid, self.cfg.order)
            if self.dtype == torch.float64:  # float64 oracle: keep the tables exact
                ang = multi_axis_angles(ids, self.cfg.axes_dim, self.cfg.theta)
                cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
            else:
                cos, sin = rope_tables(ids, self.cfg.axes_dim, self.cfg.theta, device=self.device)
            self._rope[key] = (cos.to(self.device), sin.to(self.device))
        return self._rope[key]

    # ------------------------------------------------------------------ embeddings
    def _mlp_embed(self, x, prefix, act_out="silu"):
        w = self.w
        h = F.gemv(w[prefix + ".w1"], x, w[prefix + ".b1"], silu_out=(act_out == "silu"))
        return F.gemv(w[prefix + ".w2"], h, w[prefix + ".b2"])

    def temb(self, timestep, guidance=None, pooled=None) -> torch.Tensor:
        """temb [B, D] (f32): timestep (+ guidance) (+ pooled-text) embedders."""
        cfg = self.cfg
        temb = self._mlp_embed(F.timestep_embed(timestep * 1000.0, cfg.timestep_dim), "t_embed")
        if cfg.guidance_embed:
            g = guidance if guidance is not None else torch.full_like(timestep, 3.5)
            temb = temb + self._mlp_embed(F.timestep_embed(g * 1000.0, cfg.timestep_dim), "g_embed")
        if cfg.pooled_dim:
            temb = temb + self._mlp_embed(pooled, "p_embed")
        return temb

    def modulation(self, temb: torch.Tensor) -> torch.Tensor:
        """All blocks' adaLN vectors in one GEMV: f32 [B, N_mod] = W_mod silu(temb) + b."""
        par = self.par if self.par is not None else self.tp
        if par is not None and hasattr(par, "shard_gemv") and temb.is_cuda:
            out = par.shard_gemv(self.w["mod.w"], temb, self.w["mod.b"], silu_in=True)
            if out is not None:
                return out
        return F.gemv(self.w["mod.w"], temb, self.w["mod.b"], silu_in=True)

    def teacache_probe(self, x_tokens, mod) -> torch.Tensor:
        """TeaCache signal source: block 0's modulated image input
        ``LN(x_embed(x)) * (1 + scale) + shift`` (one GEMM + one fused LN)."""
        cfg, w = self.cfg, self.w
        B, S_img, _ = x_tokens.shape
        D = cfg.hidden
        h = F.linear(x_tokens.reshape(B * S_img, -1), w["x_embed.w"], w["x_embed.b"])
        o = cfg.double_mod_offset(0, "img") if cfg.double_blocks else cfg.single_mod_offset(0)
        return F.ln_modulate(h, shift=mod[:, o:o + D], scale=mod[:, o + D:o + 2 * D], eps=cfg.eps,
                             rows_per_batch=S_img)

    def refine_text(self, txt, timestep, txt_valid=None):
        """HunyuanVideo token refiner: text self-attention blocks gated by (timestep,
        mean-pooled text).  txt [B, S, text_dim] -> [B, S, D] (replicated on every rank)."""
        cfg, w = self.cfg, self.w
        B, S, _ = txt.shape
        D, H, dh = cfg.hidden, cfg.heads, cfg.head_dim
        dev = txt.device
        valid = txt_valid if txt_valid is not None else torch.full((B,), S, device=dev, dtype=torch.int32)
        ct = torch.float64 if txt.dtype == torch.float64 else torch.float32
        mask = (torch.arange(S, device=dev)[None, :] < valid[:, None].to(dev)).to(ct)
        pooled = (txt.to(ct) * mask[..., None]).sum(1) / mask.sum(1, keepdim=True).clamp_min(1.0)
        tf = F.timestep_embed(timestep * 1000.0, cfg.timestep_dim)
        temb = self._mlp_embed(tf, "ref.t") + self._mlp_embed(pooled, "ref.p")
        h = F.linear(txt.reshape(B * S, -1), w["ref.proj.w"], w["ref.proj.b"])
        q = torch.empty(B, H, S, dh, device=dev, dtype=h.dtype)
        k, v = torch.empty_like(q), torch.empty_like(q)
        o = torch.empty(B, S, D, device=dev, dtype=h.dtype)
        lo = torch.zeros(B, device=dev, dtype=torch.int32)
        hi = valid.to(device=dev, dtype=torch.int32)
        for i in range(cfg.refiner_layers):
            p = f"ref.{i}."
            gates = F.gemv(w[p + "ada.w"], temb, w[p + "ada.b"], silu_in=True)  # [gate_msa | gate_mlp]
            n = F.ln_modulate(h, w=w[p + "n1.w"], b=w[p + "n1.b"], eps=cfg.eps)
            qkv = F.linear(n, w[p + "qkv.w"], w[p + "qkv.b"])
            F.qkv_scatter(qkv, q_off=0, k_off=D, v_off=2 * D, S_src=S, H=H, dh=dh, q_dst=[q], k_dst=[k], v_dst=[v],
                          S_dst=S, norm_mode=0, heads_per_rank=H)
            F.attention(q, k, v, 1.0 / math.sqrt(dh), out=o.view(B, S, H, dh).permute(0, 2, 1, 3), kv_lo=lo, kv_hi=hi)
            F.linear(o.view(B * S, D), w[p + "out.w"], w[p + "out.b"], out=h, gate=gates[:, :D], resid=h,
                     rows_per_batch=S)
            n = F.ln_modulate(h, w=w[p + "n2.w"], b=w[p + "n2.b"], eps=cfg.eps)
            u = F.linear(n, w[p + "up.w"], w[p + "up.b"], act="silu")
            F.linear(u, w[p + "down.w"], w[p + "down.b"], out=h, gate=gates[:, D:], resid=h, rows_per_batch=S)
        return h.view(B, S, D)

    # ------------------------------------------------------------------ forward
    def forward(self, x_tokens, txt, pooled=None, timestep=None, guidance=None, *, img_hw=None, grid=None,
                mod=None, txt_valid=None):
        """x_tokens [B, S_img(local), in_ch]; txt [B, S_txt(local), text_dim] (the full,
        replicated text for models with a token refiner); timestep [B] in [0, 1].
        ``grid`` = (t, h, w) token grid (``img_hw`` = (h, w) for images);
        ``txt_valid`` [B] = valid text length of a right-padded text stream.
        Returns the velocity [B, S_img(local), out_ch]."""
        cfg, w = self.cfg, self.w
        par = self.par
        world = par.world if par is not None else 1
        rank = par.rank if par is not None else 0
        B, S_img, _ = x_tokens.shape
        D, H, dh, F_ = cfg.hidden, cfg.heads, cfg.head_dim, cfg.mlp_hidden
        eps = cfg.eps
        if cfg.refiner_layers:
            txt_d = self.refine_text(txt, timestep, txt_valid)  # [B, S_txt_full, D]
            if par is not None:
                txt_d = par.shard_tokens(txt_d)
            S_txt = txt_d.shape[1]
        else:
            S_txt = txt.shape[1]
        ws = self._workspace(B, S_txt, S_img)
        S, S_txt_g, S_img_g = ws["S"], ws["S_txt_g"], ws["S_img_g"]
        if grid is None:
            if img_hw is None:
                side = int(round(math.sqrt(S_img_g)))
                img_hw = (side, S_img_g // side)
            grid = (1, img_hw[0], img_hw[1])
        cos, sin = self.rope(S_txt_g, grid)
        tp = self.tp
        T = tp.world if tp is not None else 1
        # heads / attention / MLP columns held by this rank (tensor parallelism); context
        # parallelism then splits the rank's Ht heads (Ulysses) or its rows (ring / gather-KV)
        # over the cp group: the q/k/v scatter and the attention epilogue address cp peers only
        Ht, Dl, Fl = H // T, D // T, F_ // T
        Hl = par.heads_local(Ht) if par is not None else Ht
        S_loc = S_txt + S_img

        sp = tp is not None and tp.sp
        if sp and B != 1:
            raise NotImplementedError("sequence parallelism runs batch 1 here (use cfg-parallel for CFG)")

        def ln(xin, out, **kw):
            """Norm + modulation; under SP this rank's rows, all-gathered into every rank's ``out``."""
            if sp:
                return tp.ln_gather(xin, out, **kw)
            return F.ln_modulate(xin, out=out, **kw)

        def row_linear(xin, wt, bias, out, gate, rpb):
            """Row-parallel (under TP) output projection fused with out += gate * (.)"""
            if tp is not None:
                tp.row_linear(xin, wt, bias, out=out, gate=gate, resid=out, rows_per_batch=rpb)
            else:
                F.linear(xin, wt, bias, out=out, gate=gate, resid=out, rows_per_batch=rpb)
        if mod is None:
            mod = self.modulation(self.temb(timestep, guidance, pooled))
        kv_lo = kv_hi = None
        if txt_valid is not None and cfg.order == "img_txt":
            kv_hi = (S_img_g + txt_valid.to(torch.int64)).to(device=x_tokens.device, dtype=torch.int32)
            kv_lo = torch.zeros_like(kv_hi)
        x_img, x_txt = ws["x_img"], ws["x_txt"]
        F.linear(x_tokens.reshape(B * S_img, -1), w["x_embed.w"], w["x_embed.b"], out=x_img.reshape(B * S_img, D))
        if cfg.refiner_layers:
            x_txt.reshape(B * S_txt, D).copy_(txt_d.reshape(B * S_txt, D))
        else:
            t2 = txt.reshape(B * S_txt, -1)
            if cfg.txt_norm:
                t2 = F.ln_modulate(t2, w=w["txt_norm"], rms=True, eps=eps)
            F.linear(t2, w["ctx_embed.w"], w["ctx_embed.b"], out=x_txt.reshape(B * S_txt, D))
        xs_of = {"img": x_img.reshape(B * S_img, D), "txt": x_txt.reshape(B * S_txt, D)}
        n_of, row_of, pos_of = ws["n"], ws["row"], ws["pos"]
        norm = ws["norm"]
        q, k, v = ws["q"], ws["k"], ws["v"]

        def dst(q_, k_, v_, row, pos):
            """qkv_scatter destinations for rows at local offset ``row`` / global position ``pos``."""
            if par is not None:
                return par.scatter_kwargs(q_, k_, v_, row, pos, S_loc, S, Ht)
            return dict(q_dst=[q_], k_dst=[k_], v_dst=[v_], S_dst=S, seq_off=pos, heads_per_rank=Ht)

        def mslice(off):
            return mod[:, off:off + D]

        # per-stream slices of the norm / MLP buffers, so both streams' GEMMs can share one launch
        off_of = {"img": 0, "txt": n_of["img"]}
        ns = {st: norm[B * off_of[st]:B * (off_of[st] + n_of[st])] for st in ("img", "txt")}
        ms = {st: ws["mlp"][B * off_of[st]:B * (off_of[st] + n_of[st])] for st in ("img", "txt")}
        group_rows = tp is None and B == 1  # row GEMMs straight into the residual stream (no TP reducer)
        for i in range(cfg.double_blocks):
            p = f"double.{i}."
            mo = {st: cfg.double_mod_offset(i, st) for st in ("img", "txt")}
            calls = []
            for st in ("img", "txt"):
                xs, nr, pos = xs_of[st], n_of[st], pos_of[st]
                ln(xs, ns[st], shift=mslice(mo[st]), scale=mslice(mo[st] + D), eps=eps, rows_per_batch=nr)
                # qkv projection with q/k RMSNorm + RoPE + head scatter (the Ulysses all-to-all under
                # CP) in its epilogue
                calls.append(dict(x=ns[st], w=w[p + st + "_qkv.w"], b=w[p + st + "_qkv.b"], out=ws["qkv_" + st],
                                  scatter=dict(q_off=0, k_off=Dl, v_off=2 * Dl, S_src=nr, H=Ht, dh=dh,
                                               **dst(q, k, v, row_of[st], pos), norm_mode=1,
                                               wq=w[p + st + "_qnorm"], wk=w[p + st + "_knorm"], eps=eps, cos=cos,
                                               sin=sin, rope_pos_off=pos)))
            F.linear_group(calls)
            self._attention(ws, B, S_txt, S_img, D, Hl, dh, kv_lo=kv_lo, kv_hi=kv_hi)
            if group_rows:
                F.linear_group([dict(x=ws["attn"][0, row_of[st]:row_of[st] + n_of[st]], w=w[p + st + "_out.w"],
                                     b=w[p + st + "_out.b"], out=xs_of[st], gate=mslice(mo[st] + 2 * D),
                                     resid=xs_of[st], rows_per_batch=n_of[st]) for st in ("img", "txt")])
            else:
                for st in ("img", "txt"):
                    rows = slice(row_of[st], row_of[st] + n_of[st])
                    self._rows_gemm(ws["attn"], rows, B, n_of[st], w[p + st + "_out.w"], w[p + st + "_out.b"],
                                    xs_of[st], mslice(mo[st] + 2 * D), row_linear)
            for st in ("img", "txt"):
                ln(xs_of[st], ns[st], shift=mslice(mo[st] + 3 * D), scale=mslice(mo[st] + 4 * D), eps=eps,
                   rows_per_batch=n_of[st])
            F.linear_group([dict(x=ns[st], w=w[p + st + "_up.w"], b=w[p + st + "_up.b"], out=ms[st], act="gelu")
                            for st in ("img", "txt")])
            if group_rows:
                F.linear_group([dict(x=ms[st], w=w[p + st + "_down.w"], b=w[p + st + "_down.b"], out=xs_of[st],
                                     gate=mslice(mo[st] + 5 * D), resid=xs_of[st], rows_per_batch=n_of[st])
                                for st in ("img", "txt")])
            else:
                for st in ("img", "txt"):
                    row_linear(ms[st], w[p + st + "_down.w"], w[p + st + "_down.b"], xs_of[st],
                               mslice(mo[st] + 5 * D), n_of[st])

        if sp:  # dual -> single: the rows each rank owns change; replicate the residual stream once
            for st in ("txt", "img"):
                tp.sync_rows(xs_of[st])
        if B > 1:  # dual -> single: the residual stream becomes [seg0 ; seg1] per batch
            for st in ("txt", "img"):
                r0 = row_of[st]
                ws["x"][:, r0:r0 + n_of[st]] = xs_of[st].view(B, n_of[st], D)
        x2 = ws["x"].view(B * S_loc, D)
        fused = ws["fused"]
        s0, s1 = cfg.streams
        for j in range(cfg.single_blocks):
            p = f"single.{j}."
            o = cfg.single_mod_offset(j)
            ln(x2, norm, shift=mslice(o), scale=mslice(o + D), eps=eps, rows_per_batch=S_loc)
            # [q | mlp | k | v] projection: GELU on the MLP columns (kept in `fused` next to the
            # attention output slot), q/k/v normalised, rotated and scattered by head in the epilogue
            if par is None:  # positions equal local rows
                place = dict(q_dst=[q], k_dst=[k], v_dst=[v], S_dst=S, seq_off=0, rope_pos_off=0, heads_per_rank=Ht)
            else:  # this rank's [seg0 ; seg1] rows: each segment placed as the CP mode lays it out
                place = dst(q, k, v, row_of[s0], pos_of[s0])
                place.update(rope_pos_off=pos_of[s0], seg_rows=n_of[s0],
                             seg1_seq_off=dst(q, k, v, row_of[s1], pos_of[s1])["seq_off"], seg1_rope_off=pos_of[s1])
            F.linear_qkv(norm, w[p + "fused.w"], w[p + "fused.b"], out=fused, act="gelu", act_lo=Dl, act_hi=Dl + Fl,
                         scatter=dict(q_off=0, k_off=Dl + Fl, v_off=2 * Dl + Fl, S_src=S_loc, H=Ht, dh=dh,
                                      norm_mode=1, wq=w[p + "qnorm"], wk=w[p + "knorm"], eps=eps, cos=cos, sin=sin,
                                      **place))
            self._attention(ws, B, S_txt, S_img, D, Hl, dh, out_rows=fused, kv_lo=kv_lo, kv_hi=kv_hi)
            row_linear(fused[:, : Dl + Fl], w[p + "proj.w"], w[p + "proj.b"], x2, mslice(o + 2 * D), S_loc)

        if sp:  # the final layer reads every image row
            tp.sync_rows(x2)
        # final adaLN-continuous (scale, shift) on the image rows + projection
        o = cfg.final_mod_offset()
        out = torch.empty(B * S_img, cfg.out_channels, device=x_tokens.device, dtype=x_tokens.dtype)
        ri = row_of["img"]
        for b in range(B):
            xi = ws["x"][b, ri:ri + S_img] if (B == 1 or cfg.single_blocks) else xs_of["img"][b * S_img:(b + 1) * S_img]
            nb = norm[:S_img]
            F.ln_modulate(xi, shift=mod[b:b + 1, o + D:o + 2 * D], scale=mod[b:b + 1, o:o + D], eps=eps, out=nb)
            F.linear(nb, w["final.w"], w["final.b"], out=out[b * S_img:(b + 1) * S_img])
        return out.view(B, S_img, cfg.out_channels)

    __call__ = forward

    # ------------------------------------------------------------------ helpers
    def _attention(self, ws, B, S_txt, S_img, D, Hl, dh, out_rows=None, kv_lo=None, kv_hi=None):
        """Joint attention over the full sequence; output lands token-major in
        ``ws['attn']`` (dual blocks) or in the q slot of ``out_rows`` (single)."""
        par = self.par
        q, k, v = ws["q"], ws["k"], ws["v"]
        scale = 1.0 / math.sqrt(dh)
        if par is not None:
            target = ws["attn"].view(B * (S_txt + S_img), -1) if out_rows is None else out_rows
            n0 = ws["n"][self.cfg.streams[0]]
            n1 = ws["n"][self.cfg.streams[1]]
            par.attention(q, k, v, scale, target, B, n0, n1, target.shape[1], kv_lo=kv_lo, kv_hi=kv_hi)
            return
        S = q.shape[2]
        if out_rows is None:
            o = ws["attn"].view(B, S, Hl, dh).permute(0, 2, 1, 3)
        else:
            ld = out_rows.shape[1]
            o = out_rows.as_strided((B, Hl, S, dh), (S * ld, dh, ld, 1))
        F.attention(q, k, v, scale, out=o, kv_lo=kv_lo, kv_hi=kv_hi)

    @staticmethod
    def _rows_gemm(attn, rows, B, n_rows, wt, bias, xs, gate, row_linear):
        """Output projection of one stream's rows of the attention output, fused with
        ``x += gate * (o W^T + b)`` (row-parallel under TP)."""
        if B == 1:
            row_linear(attn[0, rows], wt, bias, xs, gate, n_rows)
            return
        for b in range(B):
            xb = xs[b * n_rows:(b + 1) * n_rows]
            row_linear(attn[b, rows], wt, bias, xb, gate[b:b + 1], n_rows)


def pack_latents(lat: torch.Tensor, patch: int = 2) -> torch.Tensor:
    """[B, C, H, W] -> [B, (H/p)(W/p), C p p]  or  [B, C, T, H, W] -> [B, T (H/p)(W/p), C p p]."""
    if lat.dim() == 5:
        B, C, T, Hh, Ww = lat.shape
        x = lat.view(B, C, T, Hh // patch, patch, Ww // patch, patch)
        return x.permute(0, 2, 3, 5, 1, 4, 6).reshape(B, T * (Hh // patch) * (Ww // patch), C * patch * patch)
    B, C, Hh, Ww = lat.shape
    x = lat.view(B, C, Hh // patch, patch, Ww // patch, patch)
    return x.permute(0, 2, 4, 1, 3, 5).reshape(B, (Hh // patch) * (Ww // patch), C * patch * patch)


def unpack_latents(tok: torch.Tensor, h: int, w: int, patch: int = 2, t: int | None = None) -> torch.Tensor:
    """Inverse of ``pack_latents`` ([B, C, H, W], or [B, C, T, H, W] when ``t`` is given)."""
    B, _, Cpp = tok.shape
    C = Cpp // (patch * patch)
    if t is not None:
        x = tok.view(B, t, h // patch, w // patch, C, patch, patch)
        return x.permute(0, 4, 1, 2, 5, 3, 6).reshape(B, C, t, h, w)
    x = tok.view(B, h // patch, w // patch, C, patch, patch)
    return x.permute(0, 3, 1, 4, 2, 5).reshape(B, C, h, w)
