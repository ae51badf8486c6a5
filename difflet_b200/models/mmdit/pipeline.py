"""Text-to-video / text-to-image applications for the MMDiT families beyond FLUX.

* HunyuanVideo (``difflet/models/hunyuan_video/pipeline.py``): guidance-distilled
  (embedded guidance, one pass per step), LLM text states with a padding mask
  (-> attention key window) plus CLIP pooled vector, flow-matching Euler with a
  static shift, causal 3-D VAE (tiled).
* HunyuanVideo 1.5 (``difflet/models/hunyuan_video/pipeline15.py``): true CFG
  (default 6.0), token-refined Qwen2.5-VL text, 1x1x1 patches of 32-channel
  latents concatenated with the (zero) condition latents and mask.
* Qwen-Image (``difflet/models/qwen_image/pipeline.py``): true CFG with the
  norm-preserving combine ``(u + s (c - u)) * |c| / |u + s (c - u)|``, Qwen2.5-VL
  text (padding trimmed), flow-matching Euler with the resolution-dependent
  shift, Wan-style VAE on a single frame.

Latents stay on the device in fp32; CFG runs as a batched [uncond, cond] pass
on one GPU or, with ``cfg_parallel_enabled``, one branch per rank exchanged by
the fused peer kernel; Ulysses shards the tokens.
"""

from __future__ import annotations


import torch

from difflet_b200.models.flux.pipeline import SyntheticTextEncoder
from difflet_b200.models.mmdit.model import MMDiT, pack_latents, unpack_latents
from difflet_b200.ops import fused as F
from difflet_b200.schedulers import FlowMatchEulerScheduler


def qwen_time_shift_mu(seq_len: int, base_seq=256, max_seq=8192, base_shift=0.5, max_shift=0.9) -> float:
    m = (max_shift - base_shift) / (max_seq - base_seq)
    return seq_len * m + (base_shift - m * base_seq)


class MMDiTApplication:
    def __init__(self, dit: MMDiT, vae=None, *, text_encoder=None, text_len=256, flow_shift: float | None = 7.0,
                 cfg_par=None, true_cfg: bool = False, cfg_rescale: bool = False, cond_channels: int = 0):
        self.dit = dit
        self.cfg = dit.cfg
        self.vae = vae
        self.text_len = text_len
        self.text_encoder = text_encoder or SyntheticTextEncoder(text_len, self.cfg.text_dim, max(1, self.cfg.pooled_dim))
        self.flow_shift = flow_shift
        self.cfg_par = cfg_par
        self.true_cfg = true_cfg
        self.cfg_rescale = cfg_rescale
        self.cond_channels = cond_channels  # extra zero channels concatenated to the latents (HV 1.5)
        self.teacache = None
        self.last_step_ms: list[float] = []

    @property
    def device(self):
        return self.dit.device

    def _sched(self, steps, seq_len):
        if self.flow_shift is None:  # dynamic (Qwen-Image)
            return FlowMatchEulerScheduler().set_timesteps(steps, mu=qwen_time_shift_mu(seq_len))
        return FlowMatchEulerScheduler(shift=self.flow_shift, use_dynamic_shifting=False).set_timesteps(steps)

    @torch.no_grad()
    def generate(self, *, prompt=None, negative_prompt="", prompt_embeds=None, pooled_prompt_embeds=None,
                 negative_prompt_embeds=None, negative_pooled_prompt_embeds=None, text_valid=None,
                 negative_text_valid=None, height=720, width=1280, num_frames=None, num_inference_steps=50,
                 guidance_scale=6.0, true_cfg_scale=None, seed=0, latents=None, output_type="uint8", callback=None):
        cfg, dev, dt = self.cfg, self.device, self.dit.dtype
        video = num_frames is not None and num_frames > 1
        if prompt_embeds is None:
            prompts = [prompt] if isinstance(prompt, str) else list(prompt)
            prompt_embeds, pooled_prompt_embeds = self.text_encoder(prompts)
            negative_prompt_embeds, negative_pooled_prompt_embeds = self.text_encoder([negative_prompt] * len(prompts))
        B = prompt_embeds.shape[0]
        s = cfg.vae_scale
        lh, lw = height // s, width // s
        T = (num_frames - 1) // cfg.vae_scale_t + 1 if video else 1
        grid = (T // cfg.patch_t, lh // cfg.patch, lw // cfg.patch)
        S_img = grid[0] * grid[1] * grid[2]
        use_cfg = self.true_cfg and (true_cfg_scale or guidance_scale) and (true_cfg_scale or guidance_scale) > 1.0
        scale = true_cfg_scale or guidance_scale
        cfg_par = self.cfg_par if use_cfg else None
        txt_c = prompt_embeds.to(dev, dt, non_blocking=True)
        txt_u = (negative_prompt_embeds if negative_prompt_embeds is not None else torch.zeros_like(prompt_embeds)).to(dev, dt)
        pool_c = pooled_prompt_embeds.to(dev, torch.float32) if (cfg.pooled_dim and pooled_prompt_embeds is not None) else None
        pool_u = (negative_pooled_prompt_embeds.to(dev, torch.float32)
                  if (cfg.pooled_dim and negative_pooled_prompt_embeds is not None) else pool_c)
        tv_c = text_valid.to(dev) if text_valid is not None else None
        tv_u = negative_text_valid.to(dev) if negative_text_valid is not None else tv_c
        if cfg_par is not None:
            txt, pool, tv = (txt_c, pool_c, tv_c) if cfg_par.is_cond else (txt_u, pool_u, tv_u)
        elif use_cfg:
            txt = torch.cat([txt_u, txt_c])
            pool = None if pool_c is None else torch.cat([pool_u, pool_c])
            tv = None if tv_c is None else torch.cat([tv_u, tv_c])
        else:
            txt, pool, tv = txt_c, pool_c, tv_c
        Bm = txt.shape[0]
        if latents is None:
            g = torch.Generator().manual_seed(seed)
            shape = (B, cfg.latent_channels, T, lh, lw) if video else (B, cfg.latent_channels, lh, lw)
            latents = torch.randn(*shape, generator=g)
        lat = latents.to(dev, torch.float32, non_blocking=True)
        x32 = pack_latents(lat, cfg.patch).contiguous()
        par = self.dit.par
        if par is not None:
            x32 = par.shard_tokens(x32).contiguous()
            if not cfg.refiner_layers:
                txt = par.shard_tokens(txt).contiguous()
        sched = self._sched(num_inference_steps, S_img)
        gvec = torch.full((Bm,), float(guidance_scale), device=dev)
        for i in range(num_inference_steps):
            t = float(sched.timesteps[i]) / 1000.0
            tvec = torch.full((Bm,), t, device=dev)
            x_in = x32.to(dt)
            if self.cond_channels:
                x_in = torch.cat([x_in, torch.zeros(*x_in.shape[:2], self.cond_channels, device=dev, dtype=dt)], -1)
            if use_cfg and cfg_par is None:
                x_in = torch.cat([x_in, x_in])
            if self.teacache is not None and self.teacache.should_skip(i, x_in, None):
                v = self.teacache.skip_noise_pred()
            else:
                v = self.dit(x_in, txt, pool, tvec, gvec, grid=grid, txt_valid=tv)
                if self.teacache is not None:
                    self.teacache.record_full_step(i, v)
            if cfg_par is not None:
                v32 = cfg_par.combine(v, scale)
            elif use_cfg:
                u, c = v[:B].float(), v[B:].float()
                v32 = u + scale * (c - u)
                if self.cfg_rescale:
                    v32 = v32 * (c.norm(dim=-1, keepdim=True) / v32.norm(dim=-1, keepdim=True).clamp_min(1e-12))
            else:
                v32 = v.float()
            x32.add_(v32, alpha=sched.dt(i))
            if callback is not None:
                callback(i, x32)
        x_full = par.gather_tokens(x32) if par is not None else x32
        out_lat = unpack_latents(x_full, lh, lw, cfg.patch, t=T if video else None)
        if output_type == "latent":
            return out_lat
        import torch.distributed as dist

        if dist.is_initialized() and dist.get_rank() != 0:
            return None
        if self.vae is None:
            raise RuntimeError("no VAE loaded; use output_type='latent'")
        z = out_lat if out_lat.dim() == 5 else out_lat[:, :, None]
        img = self.vae.decode(z)
        if output_type == "float":
            return img
        img = ((img.float() * 0.5 + 0.5).clamp(0, 1) * 255).round().to(torch.uint8)
        return img.permute(0, 2, 3, 4, 1) if video else img[:, :, 0].permute(0, 2, 3, 1)

    __call__ = generate
