"""LTX-2 text-to-audio+video application.

Denoising loop of the reference orchestrator (difflet/models/ltx_2/pipeline.py:
249-830): flow-matching sigmas ``linspace(1, 1/N)`` shifted by the resolution-
dependent ``mu`` (LTX-2's line: 0.95 at 1024 tokens to 2.05 at 4096), video and
audio latents stepped together with one velocity each.  Guidance is combined in x0
space (x0 = x - sigma v): classifier-free guidance ``c + (s - 1)(c - u)``,
spatio-temporal guidance ``+ stg (c - perturbed)`` (self-attention of the given
blocks replaced by its values), modality guidance ``+ (m - 1)(c - isolated)`` (no
cross-modal attention), optional guidance rescale; each with its own audio scale.
The text embeddings come from a deterministic stand-in for Gemma-3 (no encoder
weights offline).  CFG runs both branches in one batch of 2, or on two GPUs
(cfg axis) with each rank holding one branch and the prediction exchanged.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from difflet_b200.models.flux.pipeline import SyntheticTextEncoder
from difflet_b200.models.ltx_2.model import (LTX2Transformer, audio_coords, pack_audio, pack_video, unpack_audio,
                                             unpack_video, video_coords)


def ltx2_mu(seq_len: int, base_seq=1024, max_seq=4096, base_shift=0.95, max_shift=2.05) -> float:
    m = (max_shift - base_shift) / (max_seq - base_seq)
    return base_shift + m * (seq_len - base_seq)


def _rescale(guided, cond, phi):
    dims = tuple(range(1, guided.dim()))
    std_c = cond.std(dim=dims, keepdim=True)
    std_g = guided.std(dim=dims, keepdim=True)
    return phi * guided * (std_c / std_g) + (1 - phi) * guided


class LTX2Application:
    def __init__(self, transformer: LTX2Transformer, decoders=None, *, text_encoder=None, cfg_par=None,
                 fps: float = 24.0):
        self.dit = transformer
        self.cfg = transformer.cfg
        self.decoders = decoders
        self.cfg_par = cfg_par
        self.fps = fps
        self.text_encoder = text_encoder or SyntheticTextEncoder(self.cfg.text_len, self.cfg.text_dim, 1)

    def latent_shape(self, height, width, num_frames):
        c = self.cfg
        f = (num_frames - 1) // c.vae_scale_t + 1
        ta = max(1, round(num_frames / self.fps * 25))
        return (c.in_channels, f, height // c.vae_scale, width // c.vae_scale), (c.audio_channels, ta, c.audio_mel_bins)

    def _encode(self, prompts):
        emb, _ = self.text_encoder(prompts)
        valid = torch.tensor([max(1, min(self.cfg.text_len, len(p.split()) * 2 + 1)) for p in prompts])
        return emb, valid

    @torch.no_grad()
    def generate(self, prompt: str, negative_prompt: str = "", *, height=512, width=768, num_frames=121,
                 num_inference_steps=40, guidance_scale=4.0, audio_guidance_scale=None, stg_scale=0.0,
                 audio_stg_scale=None, spatio_temporal_guidance_blocks=None, modality_scale=1.0,
                 audio_modality_scale=None, guidance_rescale=0.0, seed=0, output_type="np", latents=None,
                 audio_latents=None, return_latents=False, callback=None):
        dit, cfg = self.dit, self.cfg
        dev, dt = dit.device, dit.dtype
        ags = guidance_scale if audio_guidance_scale is None else audio_guidance_scale
        astg = stg_scale if audio_stg_scale is None else audio_stg_scale
        amod = modality_scale if audio_modality_scale is None else audio_modality_scale
        do_cfg = guidance_scale > 1.0 or ags > 1.0
        do_stg = stg_scale > 0.0 or astg > 0.0
        do_mod = modality_scale > 1.0 or amod > 1.0
        if do_stg and not spatio_temporal_guidance_blocks:
            raise ValueError("LTX-2 STG requires spatio_temporal_guidance_blocks when stg_scale is nonzero")
        if self.cfg_par is not None and (do_stg or do_mod or guidance_rescale > 0.0):
            raise ValueError("LTX-2 CFG-parallel does not support STG, modality guidance or guidance rescale")
        vshape, ashape = self.latent_shape(height, width, num_frames)
        g = torch.Generator().manual_seed(int(seed))
        x = latents if latents is not None else torch.randn(1, *vshape, generator=g)
        xa = audio_latents if audio_latents is not None else torch.randn(1, *ashape, generator=g)
        xv = pack_video(x.float()).to(dev)          # [1, Sv, C] f32 master latents
        xa = pack_audio(xa.float()).to(dev)         # [1, Sa, C*mel]
        grid = vshape[1:]
        vc = video_coords(*grid, cfg, fps=self.fps)
        ac = audio_coords(ashape[1])
        prompts = [negative_prompt, prompt] if do_cfg else [prompt]
        text, valid = self._encode(prompts)
        cfg_par = self.cfg_par
        if do_cfg and cfg_par is not None:  # this rank evaluates one branch
            text, valid = text[cfg_par.rank:cfg_par.rank + 1], valid[cfg_par.rank:cfg_par.rank + 1]
        ctx = dit.prepare_context(text.to(dev, dt))
        valid = valid.to(dev)
        Sv = xv.shape[1]
        sig = np.linspace(1.0, 1.0 / num_inference_steps, num_inference_steps)
        mu = ltx2_mu(Sv)
        sig = math.exp(mu) / (math.exp(mu) + (1.0 / sig - 1.0))
        sigmas = np.concatenate([sig, [0.0]])
        nb = text.shape[0]
        for i in range(num_inference_steps):
            s, s_next = float(sigmas[i]), float(sigmas[i + 1])
            t = torch.full((nb,), s, device=dev, dtype=torch.float32 if dt != torch.float64 else dt)
            cond = dit.time_embed(t)
            vin = xv.to(dt).expand(nb, -1, -1).contiguous()
            ain = xa.to(dt).expand(nb, -1, -1).contiguous()
            pv, pa = dit(vin, ain, t, ctx, vcoords=vc, acoords=ac, text_valid=valid, cond=cond)
            if do_cfg and cfg_par is not None:
                # x0-space CFG equals u + s (c - u) on the velocities: one fused exchange per stream
                xv = xv + (s_next - s) * cfg_par.combine(pv.contiguous(), guidance_scale)
                xa = xa + (s_next - s) * cfg_par.combine(pa.contiguous(), ags)
                if callback is not None:
                    callback(i, xv)
                continue
            pv, pa = pv.float(), pa.float()
            x0v = xv - s * pv
            x0a = xa - s * pa
            if do_cfg:
                uv, cv = x0v.chunk(2)
                ua, ca = x0a.chunk(2)
                gv = cv + (guidance_scale - 1.0) * (cv - uv)
                ga = ca + (ags - 1.0) * (ca - ua)
            else:
                cv, ca = x0v, x0a
                gv, ga = cv, ca
            if do_stg or do_mod:
                pos = slice(nb - 1, nb)
                tp = t[pos]
                cond1 = tuple(c[pos] for c in cond)
                ctx1 = [tuple((k[pos], v[pos]) for k, v in pair) for pair in ctx]
                if do_stg:
                    sv, sa = dit(xv.to(dt), xa.to(dt), tp, ctx1, vcoords=vc, acoords=ac, text_valid=valid[pos],
                                 cond=cond1, perturb_blocks=tuple(spatio_temporal_guidance_blocks))
                    gv = gv + stg_scale * (cv - (xv - s * sv.float()))
                    ga = ga + astg * (ca - (xa - s * sa.float()))
                if do_mod:
                    iv, ia = dit(xv.to(dt), xa.to(dt), tp, ctx1, vcoords=vc, acoords=ac, text_valid=valid[pos],
                                 cond=cond1, isolate_modalities=True)
                    gv = gv + (modality_scale - 1.0) * (cv - (xv - s * iv.float()))
                    ga = ga + (amod - 1.0) * (ca - (xa - s * ia.float()))
            if guidance_rescale > 0.0:
                gv = _rescale(gv, cv, guidance_rescale)
                ga = _rescale(ga, ca, guidance_rescale)
            vel_v = (xv - gv) / s
            vel_a = (xa - ga) / s
            xv = xv + (s_next - s) * vel_v
            xa = xa + (s_next - s) * vel_a
            if callback is not None:  # per-step observer (video latents)
                callback(i, xv)
        lat_v = unpack_video(xv, grid)
        lat_a = unpack_audio(xa, cfg.audio_channels)
        if return_latents or self.decoders is None:
            return {"latents": lat_v, "audio_latents": lat_a}
        d = self.decoders
        video = d.decode_video(lat_v.to(dt))[0]               # [3, F, H, W]
        wav = d.vocode(d.decode_mel(lat_a.to(dt)))[0].float()  # [stereo, samples]
        frames = ((video.float().clamp(-1, 1) + 1) * 127.5).round().to(torch.uint8).permute(1, 2, 3, 0).cpu()
        return {"frames": frames.numpy() if output_type == "np" else frames, "audio": wav.cpu().numpy(),
                "fps": self.fps, "sample_rate": d.cfg.sample_rate}


__all__ = ["LTX2Application", "ltx2_mu"]
