"""Wan text-to-video application: two-expert denoise loop with UniPC, CFG, causal VAE.

Reference behaviour: ``difflet/models/wan/pipeline.py:32-582`` and
``difflet/backends/cuda/wan/application.py:52-336``: UMT5 text padded to 512
(padding rows zeroed), fp32 latents, UniPC flow-matching steps, Wan 2.2's two
experts switched at ``boundary_ratio * 1000`` (high-noise expert first) with
``guidance_scale`` / ``guidance_scale_2``, true CFG, VAE decode.

B200 design:
  * latents stay on the device in fp32 as token shards (Ulysses): UniPC is
    elementwise, so each rank steps only its own tokens
  * per prompt and expert, the text embedder and all 40 blocks' cross-attention
    K/V are computed once (not per step)
  * CFG: batched ``[uncond, cond]`` on one GPU; with ``cfg_parallel_enabled``
    each branch runs on its own rank group and one kernel reads the partner's
    prediction over NVLink and forms ``u + s (c - u)`` (PeerCfg)
  * VAE decode streams latent frames through the causal decoder
"""

from __future__ import annotations

import torch

from difflet_b200.models.flux.pipeline import SyntheticTextEncoder
from difflet_b200.models.wan.model import WanTransformer, patchify, unpatchify
from difflet_b200.schedulers.unipc import UniPCScheduler


class WanApplication:
    def __init__(self, experts: list[WanTransformer], vae=None, *, boundary_ratio: float = 0.875,
                 flow_shift: float = 12.0, text_encoder=None, cfg_par=None, seq_par=None):
        self.experts = experts
        self.cfg = experts[0].cfg
        self.vae = vae
        self.boundary_ratio = boundary_ratio
        self.flow_shift = flow_shift
        self.text_encoder = text_encoder or SyntheticTextEncoder(self.cfg.text_len, self.cfg.text_dim, 1)
        self.cfg_par = cfg_par
        self.seq_par = seq_par
        for e in experts:
            e.par = seq_par
        self.last_step_ms: list[float] = []
        self.teacache = None

    @property
    def device(self):
        return self.experts[0].device

    def _encode(self, prompts):
        emb, _ = self.text_encoder(prompts)
        return emb

    def _expert_for(self, t: float) -> int:
        if len(self.experts) == 1:
            return 0
        return 0 if t >= self.boundary_ratio * 1000.0 else 1

    @torch.no_grad()
    def generate(self, *, prompt=None, negative_prompt="", prompt_embeds=None, negative_prompt_embeds=None,
                 height: int = 720, width: int = 1280, num_frames: int = 81, num_inference_steps: int = 40,
                 guidance_scale: float = 5.0, guidance_scale_2: float | None = None, seed: int = 0, latents=None,
                 output_type: str = "uint8", text_valid=None, time_steps: bool = False, callback=None):
        cfg = self.cfg
        dev = self.device
        dt = self.experts[0].dtype
        if prompt_embeds is None:
            prompts = [prompt] if isinstance(prompt, str) else list(prompt)
            prompt_embeds = self._encode(prompts)
            negative_prompt_embeds = self._encode([negative_prompt] * len(prompts))
        if negative_prompt_embeds is None:
            negative_prompt_embeds = torch.zeros_like(prompt_embeds)
        B = prompt_embeds.shape[0]
        T = (num_frames - 1) // cfg.vae_scale_t + 1
        lh, lw = height // cfg.vae_scale, width // cfg.vae_scale
        grid = (T // cfg.patch[0], lh // cfg.patch[1], lw // cfg.patch[2])
        cond = prompt_embeds.to(dev, dt, non_blocking=True)
        uncond = negative_prompt_embeds.to(dev, dt, non_blocking=True)
        use_cfg = guidance_scale is not None and guidance_scale > 1.0
        cfg_par = self.cfg_par if use_cfg else None
        # per-expert cached text context (text embedder + all blocks' cross K/V)
        contexts = []
        for e in self.experts:
            if cfg_par is not None:
                contexts.append(e.prepare_context(cond if cfg_par.is_cond else uncond, text_valid))
            elif use_cfg:
                cu, cc = e.prepare_context(uncond, text_valid), e.prepare_context(cond, text_valid)
                contexts.append([(torch.cat([ku, kc]), torch.cat([vu, vc])) for (ku, vu), (kc, vc) in zip(cu, cc)])
            else:
                contexts.append(e.prepare_context(cond, text_valid))
        if latents is None:
            g = torch.Generator().manual_seed(seed)
            latents = torch.randn(B, cfg.in_channels, T, lh, lw, generator=g)
        x32 = patchify(latents.to(dev, torch.float32, non_blocking=True), cfg.patch)
        if self.seq_par is not None:
            x32 = self.seq_par.shard_tokens(x32)
        x32 = x32.contiguous()
        sched = UniPCScheduler(shift=self.flow_shift).set_timesteps(num_inference_steps)
        self.last_step_ms = []
        for i in range(num_inference_steps):
            ev = None
            if time_steps and x32.is_cuda:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record()
            t = float(sched.timesteps[i])
            ei = self._expert_for(t)
            gs = guidance_scale if ei == 0 or guidance_scale_2 is None else guidance_scale_2
            expert = self.experts[ei]
            x_in = x32.to(dt)
            if use_cfg and cfg_par is None:
                x_in = torch.cat([x_in, x_in])
            tvec = torch.full((x_in.shape[0],), t, device=dev, dtype=torch.float32)
            if self.teacache is not None and self.teacache.should_skip(i, x_in, None):
                v = self.teacache.skip_noise_pred()
            else:
                v = expert(x_in, tvec, contexts[ei], grid=grid)
                if self.teacache is not None:
                    self.teacache.record_full_step(i, v)
            if cfg_par is not None:
                v32 = cfg_par.combine(v, gs)
            elif use_cfg:
                u, c = v[:B].float(), v[B:].float()
                v32 = u + gs * (c - u)
            else:
                v32 = v.float()
            x32 = sched.step(v32, x32)
            if ev is not None:
                ev[1].record()
                self.last_step_ms.append(ev)
            if callback is not None:
                callback(i, x32)
        if time_steps and x32.is_cuda:
            torch.cuda.synchronize()
            self.last_step_ms = [a.elapsed_time(b) for a, b in self.last_step_ms]
        x_full = self.seq_par.gather_tokens(x32) if self.seq_par is not None else x32
        lat = unpatchify(x_full, grid, cfg.patch, cfg.out_channels)
        if output_type == "latent":
            return lat
        if self.vae is None:
            raise RuntimeError("no VAE loaded; use output_type='latent'")
        import torch.distributed as dist

        if dist.is_initialized() and dist.get_rank() != 0:
            return None
        video = self.vae.decode(lat)  # [B, 3, F, H, W] in [-1, 1]
        if output_type == "float":
            return video
        return ((video.float() * 0.5 + 0.5).clamp(0, 1) * 255).round().to(torch.uint8).permute(0, 2, 3, 4, 1)

    __call__ = generate
