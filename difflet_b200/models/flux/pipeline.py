"""FLUX text-to-image application: denoise loop + VAE decode, fully device-resident.

Reference behaviour: ``difflet/backends/cuda/flux/application.py:26-160`` (a
diffusers ``FluxPipeline`` around the DiT) and ``difflet/models/flux/pipeline.py:46-460``:
flow-matching Euler with the resolution-dependent shift ``mu``, embedded
guidance (FLUX.1-dev is guidance-distilled: no CFG pass), latents packed 2x2.

B200 design:
  * latents live on the device in fp32 (plus a bf16 mirror the DiT reads);
    the Euler update is one kernel
  * the adaLN modulation for ALL steps is computed up front in one tcgen05
    GEMM (``[steps*B, D] x [N_mod, D]^T``, f32 out): the 6.5 GB modulation
    matrix is read once per image instead of once per step
  * the DiT step can be captured in a CUDA graph (static workspace buffers)
  * ``par`` (Ulysses sequence parallelism) shards the token sequence over GPUs
"""

from __future__ import annotations

import hashlib
import time
from dataclasses import dataclass

import torch

from difflet_b200.models.flux.config import FluxConfig
from difflet_b200.models.flux.model import FluxTransformer, pack_latents, unpack_latents
from difflet_b200.ops import fused as F
from difflet_b200.schedulers import FlowMatchEulerScheduler, flux_time_shift_mu


class SyntheticTextEncoder:
    """Deterministic stand-in for T5 / CLIP when no encoder weights are available:
    a prompt maps (by SHA-256 seed) to N(0, 1) hidden states and pooled vector of
    the encoder's shape.  Used for offline benchmarks and smoke runs."""

    def __init__(self, text_len: int, text_dim: int, pooled_dim: int):
        self.text_len, self.text_dim, self.pooled_dim = text_len, text_dim, pooled_dim

    def __call__(self, prompts: list[str]):
        embs, pooled = [], []
        for p in prompts:
            seed = int.from_bytes(hashlib.sha256(p.encode()).digest()[:8], "little")
            g = torch.Generator().manual_seed(seed)
            embs.append(torch.randn(self.text_len, self.text_dim, generator=g))
            pooled.append(torch.randn(self.pooled_dim, generator=g))
        return torch.stack(embs), torch.stack(pooled)


@dataclass
class StepTimes:
    device_ms: list


class FluxApplication:
    def __init__(self, transformer: FluxTransformer, vae=None, *, text_encoder=None, text_len: int = 512,
                 use_cuda_graph: bool = True):
        self.dit = transformer
        self.cfg: FluxConfig = transformer.cfg
        self.vae = vae
        self.text_len = text_len
        self.text_encoder = text_encoder or SyntheticTextEncoder(text_len, self.cfg.text_dim, self.cfg.pooled_dim)
        self.use_cuda_graph = use_cuda_graph
        self._graphs = {}
        self.last_step_ms: list[float] = []
        self.teacache = None

    @property
    def device(self):
        return self.dit.device

    # ------------------------------------------------------------------ helpers
    def _sched(self, steps: int, S_img: int):
        return FlowMatchEulerScheduler().set_timesteps(steps, mu=flux_time_shift_mu(S_img))

    def modulation_all(self, timesteps: torch.Tensor, guidance: torch.Tensor, pooled: torch.Tensor) -> torch.Tensor:
        """f32 [steps, B, N_mod]: every step's adaLN vectors from one GEMM."""
        steps, B = timesteps.shape[0], pooled.shape[0]
        t = timesteps.repeat_interleave(B)
        g = guidance.repeat(steps)
        p = pooled.repeat(steps, 1)
        temb = self.dit.temb(t, g, p)  # f32 [steps*B, D]
        w = self.dit.w
        if temb.is_cuda:
            a = torch.nn.functional.silu(temb).to(w["mod.w"].dtype)
            mod = F.linear(a, w["mod.w"], w["mod.b"], out_f32=True)
        else:
            mod = self.dit.modulation(temb)
        return mod.view(steps, B, -1)

    def _step_fn(self, key, x16, txt, pooled, t, g, mod_buf, img_hw):
        """DiT forward on static buffers (captured into a CUDA graph when enabled)."""

        def run():
            return self.dit(x16, txt, pooled, t, g, img_hw=img_hw, mod=mod_buf)

        if not (self.use_cuda_graph and x16.is_cuda):
            return run
        if key in self._graphs:
            graph, out = self._graphs[key]
            return lambda: (graph.replay(), out)[1]
        # warm up on a side stream, then capture
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            run()
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = run()
        self._graphs[key] = (graph, out)
        return lambda: (graph.replay(), out)[1]

    # ------------------------------------------------------------------ generate
    @torch.no_grad()
    def generate(self, *, prompt=None, prompt_embeds=None, pooled_prompt_embeds=None, height: int = 1024,
                 width: int = 1024, num_inference_steps: int = 28, guidance_scale: float = 3.5, seed: int = 0,
                 latents=None, output_type: str = "uint8", time_steps: bool = False, callback=None):
        """Returns images ``[B, H, W, 3]`` uint8 (``output_type='uint8'``), decoded float
        images (``'float'``) or the final latents (``'latent'``)."""
        dev = self.device
        cfg = self.cfg
        if prompt_embeds is None:
            prompts = [prompt] if isinstance(prompt, str) else list(prompt)
            prompt_embeds, pooled_prompt_embeds = self.text_encoder(prompts)
        B = prompt_embeds.shape[0]
        lh, lw = height // cfg.vae_scale, width // cfg.vae_scale
        h_tok, w_tok = lh // cfg.patch, lw // cfg.patch
        S_img = h_tok * w_tok
        par = self.dit.par
        dt = self.dit.dtype
        txt = prompt_embeds.to(dev, dt, non_blocking=True)
        pooled = pooled_prompt_embeds.to(dev, torch.float32, non_blocking=True)
        if latents is None:
            g = torch.Generator().manual_seed(seed)
            latents = torch.randn(B, cfg.latent_channels, lh, lw, generator=g)
        x32 = pack_latents(latents.to(dev, torch.float32, non_blocking=True)).contiguous()
        sched = self._sched(num_inference_steps, S_img)
        ts = torch.tensor(sched.timesteps, device=dev, dtype=torch.float32) / 1000.0
        gvec = torch.full((B,), float(guidance_scale), device=dev, dtype=torch.float32)
        mod_all = self.modulation_all(ts, gvec, pooled)
        # sequence-parallel shard of the tokens (text and image split over ranks)
        if par is not None:
            x_loc, txt_loc = par.shard_tokens(x32), par.shard_tokens(txt)
        else:
            x_loc, txt_loc = x32, txt
        x32_loc = x_loc.contiguous()
        x16 = x32_loc.to(dt)
        txt_loc = txt_loc.contiguous()
        mod_buf = torch.empty_like(mod_all[0])
        t_buf = torch.empty(B, device=dev, dtype=torch.float32)
        key = (B, txt_loc.shape[1], x16.shape[1], h_tok, w_tok)
        step = self._step_fn(key, x16, txt_loc, pooled, t_buf, gvec, mod_buf, (h_tok, w_tok))
        self.last_step_ms = []
        tc = self.teacache
        if tc is not None:
            tc.cal.num_steps = num_inference_steps
            tc.reset()
        for i in range(num_inference_steps):
            ev = None
            if time_steps and x16.is_cuda:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record()
            mod_buf.copy_(mod_all[i])
            t_buf.fill_(float(ts[i]))
            probe = self.dit.teacache_probe(x16, mod_buf) if (tc is not None and tc.needs_probe()) else None
            if tc is not None and tc.should_skip(i, probe):
                v = tc.skip_noise_pred()
            else:
                v = step()
                if tc is not None:
                    tc.record_full_step(i, v)
            F.euler_step(x32_loc, v, sched.dt(i), x16=x16)
            if ev is not None:
                ev[1].record()
                self.last_step_ms.append(ev)
            if callback is not None:
                callback(i, x32_loc)
        if time_steps and x16.is_cuda:
            torch.cuda.synchronize()
            self.last_step_ms = [a.elapsed_time(b) for a, b in self.last_step_ms]
        x_full = par.gather_tokens(x32_loc) if par is not None else x32_loc
        lat = unpack_latents(x_full, lh, lw)
        if output_type == "latent":
            return lat
        if self.vae is None:
            raise RuntimeError("no VAE loaded; use output_type='latent'")
        if par is not None and par.rank != 0 and not par.decode_on_all_ranks:
            return None
        from difflet_b200.utils.host_vae import for_vae

        img = self.vae.decode(for_vae(self.vae, lat))
        if output_type == "float":
            return img
        from difflet_b200.models.vae.autoencoder_kl import to_uint8

        return to_uint8(img)

    __call__ = generate
