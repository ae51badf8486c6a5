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
    each branch runs on its own rank group; either way ONE kernel per step forms
    ``u + s (c - u)`` (reading the partner's prediction over NVLink under CFG
    parallelism, PeerCfg) and applies the UniPC corrector + predictor to the fp32
    latents (``schedulers/guided.py``, ``csrc/sched.cu``)
  * VAE decode streams latent frames through the causal decoder
"""

from __future__ import annotations

import torch

from difflet_b200.models.flux.pipeline import SyntheticTextEncoder
from difflet_b200.models.wan.model import WanTransformer, patchify, unpatchify
from difflet_b200.schedulers.guided import GuidedSampler
from difflet_b200.schedulers.unipc import UniPCScheduler


class WanRun:
    """One generation's device state: cached text contexts per expert, the latent token shard and
    its fused sampler (CFG combine + UniPC in one kernel), the DiT input buffer and schedule.
    ``step(i)`` runs denoise step ``i``; ``latents()`` gathers and unpatchifies the result."""

    def __init__(self, app, *, cond, uncond, text_valid, grid, latents, steps, guidance_scale, guidance_scale_2):
        self.app = app
        self.grid = grid
        self.steps = steps
        self.gs, self.gs2 = guidance_scale, guidance_scale_2
        cfg = app.cfg
        dev = app.device
        dt = app.experts[0].dtype
        self.use_cfg = guidance_scale is not None and guidance_scale > 1.0
        self.cfg_par = app.cfg_par if self.use_cfg else None
        self.batched_cfg = self.use_cfg and self.cfg_par is None
        self.contexts = []
        for e in app.experts:
            if self.cfg_par is not None:
                self.contexts.append(e.prepare_context(cond if self.cfg_par.is_cond else uncond, text_valid))
            elif self.batched_cfg:
                cu, cc = e.prepare_context(uncond, text_valid), e.prepare_context(cond, text_valid)
                self.contexts.append([(torch.cat([ku, kc]), torch.cat([vu, vc])) for (ku, vu), (kc, vc) in zip(cu, cc)])
            else:
                self.contexts.append(e.prepare_context(cond, text_valid))
        x32 = patchify(latents.to(dev, torch.float32, non_blocking=True), cfg.patch)
        if app.seq_par is not None:
            x32 = app.seq_par.shard_tokens(x32)
        self.B = x32.shape[0]
        self.x32 = x32.contiguous()
        # DiT input: the sampler writes the bf16 mirror of the latents into the first B rows
        # (batched CFG feeds the same latents to both branches: the mirror is copied once per step)
        nb = 2 * self.B if self.batched_cfg else self.B
        self.x_in = torch.empty((nb,) + tuple(self.x32.shape[1:]), device=dev, dtype=dt)
        self.x_in[: self.B].copy_(self.x32)
        if self.batched_cfg:
            self.x_in[self.B:].copy_(self.x_in[: self.B])
        self.sched = UniPCScheduler(shift=app.flow_shift).set_timesteps(steps)
        self.sampler = GuidedSampler(self.sched, self.x32, self.x_in[: self.B])
        self.tvec = torch.empty(nb, device=dev, dtype=torch.float32)
        self.out_shape = (nb, self.x32.shape[1], cfg.out_channels * cfg.patch[0] * cfg.patch[1] * cfg.patch[2])

    def step(self, i: int) -> None:
        app = self.app
        t = float(self.sched.timesteps[i])
        ei = app._expert_for(t)
        gs = self.gs if ei == 0 or self.gs2 is None else self.gs2
        expert = app.experts[ei]
        self.tvec.fill_(t)
        tc = app.teacache
        if tc is not None and tc.should_skip(i, self.x_in, None):
            v = tc.skip_noise_pred()
        else:
            out = self.cfg_par.next_pred_buffer(self.out_shape, self.x_in.dtype) if self.cfg_par is not None else None
            v = expert(self.x_in, self.tvec, self.contexts[ei], grid=self.grid, out=out)
            if tc is not None:
                tc.record_full_step(i, v)
        B = self.B
        if self.cfg_par is not None:
            self.cfg_par.step(v, gs, self.sampler)   # exchange + combine + UniPC, one kernel
        elif self.batched_cfg:
            self.sampler.step(v[:B], v[B:], gs)      # combine + UniPC, one kernel
            self.x_in[B:].copy_(self.x_in[:B])
        else:
            self.sampler.step(v)

    def latents(self):
        app = self.app
        x_full = app.seq_par.gather_tokens(self.x32) if app.seq_par is not None else self.x32
        return unpatchify(x_full, self.grid, app.cfg.patch, app.cfg.out_channels)


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

    def prepare(self, *, prompt=None, negative_prompt="", prompt_embeds=None, negative_prompt_embeds=None,
                height: int = 720, width: int = 1280, num_frames: int = 81, num_inference_steps: int = 40,
                guidance_scale: float = 5.0, guidance_scale_2: float | None = None, seed: int = 0, latents=None,
                text_valid=None) -> WanRun:
        """Text contexts, initial latents and sampler of one generation (``WanRun``)."""
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
        if latents is None:
            g = torch.Generator().manual_seed(seed)
            latents = torch.randn(B, cfg.in_channels, T, lh, lw, generator=g)
        return WanRun(self, cond=cond, uncond=uncond, text_valid=text_valid, grid=grid, latents=latents,
                      steps=num_inference_steps, guidance_scale=guidance_scale, guidance_scale_2=guidance_scale_2)

    @torch.no_grad()
    def generate(self, *, prompt=None, negative_prompt="", prompt_embeds=None, negative_prompt_embeds=None,
                 height: int = 720, width: int = 1280, num_frames: int = 81, num_inference_steps: int = 40,
                 guidance_scale: float = 5.0, guidance_scale_2: float | None = None, seed: int = 0, latents=None,
                 output_type: str = "uint8", text_valid=None, time_steps: bool = False, callback=None):
        run = self.prepare(prompt=prompt, negative_prompt=negative_prompt, prompt_embeds=prompt_embeds,
                           negative_prompt_embeds=negative_prompt_embeds, height=height, width=width,
                           num_frames=num_frames, num_inference_steps=num_inference_steps,
                           guidance_scale=guidance_scale, guidance_scale_2=guidance_scale_2, seed=seed,
                           latents=latents, text_valid=text_valid)
        self.last_step_ms = []
        timed = time_steps and run.x32.is_cuda
        for i in range(num_inference_steps):
            ev = None
            if timed:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record()
            run.step(i)
            if ev is not None:
                ev[1].record()
                self.last_step_ms.append(ev)
            if callback is not None:
                callback(i, run.x32)
        if timed:
            torch.cuda.synchronize()
            self.last_step_ms = [a.elapsed_time(b) for a, b in self.last_step_ms]
        lat = run.latents()
        if output_type == "latent":
            return lat
        if self.vae is None:
            raise RuntimeError("no VAE loaded; use output_type='latent'")
        video = self.decode(lat)
        if video is None or output_type == "float":
            return video
        return ((video.float() * 0.5 + 0.5).clamp(0, 1) * 255).round().to(torch.uint8).permute(0, 2, 3, 4, 1)

    def decode(self, lat):
        """Causal VAE decode.  Under a multi-GPU world every rank decodes a slab of rows (halo rows
        exchanged over NVLink by the producer kernels) and rank 0 returns the video [B, 3, F, H, W]
        in [-1, 1] (the other ranks None)."""
        import torch.distributed as dist

        from difflet_b200.utils.host_vae import for_vae, vae_device

        if vae_device(self.vae) is not None and vae_device(self.vae).type == "cpu" and lat.is_cuda:  # --host-vae
            if dist.is_initialized() and dist.get_rank() != 0:
                return None
            return self.vae.decode(for_vae(self.vae, lat))
        if dist.is_initialized() and dist.get_world_size() > 1 and hasattr(self.vae, "set_slabs"):
            rows = lat.shape[3]
            if self.vae.slabs is None or self.vae.slabs.rows != rows or self.vae.slabs.world == 1:
                from difflet_b200.parallel.slabs import make_slabs

                self.vae.set_slabs(make_slabs(rows, lat.device))
            return self.vae.decode(lat)
        if dist.is_initialized() and dist.get_rank() != 0:
            return None
        return self.vae.decode(lat)

    __call__ = generate
