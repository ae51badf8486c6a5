"""FLUX MMDiT configuration (reference: ``difflet/models/flux/dit_config.py``)."""

from __future__ import annotations

from dataclasses import dataclass, replace


@dataclass(frozen=True)
class FluxConfig:
    in_channels: int = 64          # 16 latent channels x 2x2 patch
    out_channels: int = 64
    hidden: int = 3072
    heads: int = 24
    head_dim: int = 128
    double_blocks: int = 19
    single_blocks: int = 38
    mlp_ratio: float = 4.0
    text_dim: int = 4096           # T5-XXL hidden states
    pooled_dim: int = 768          # CLIP pooled
    timestep_dim: int = 256        # sinusoidal features
    axes_dim: tuple = (16, 56, 56)
    theta: float = 10000.0
    guidance_embed: bool = True    # FLUX.1-dev is guidance-distilled
    eps: float = 1e-6
    latent_channels: int = 16
    patch: int = 2
    vae_scale: int = 8

    @property
    def mlp_hidden(self) -> int:
        return int(self.hidden * self.mlp_ratio)

    @property
    def mod_rows(self) -> int:
        D = self.hidden
        return self.double_blocks * 12 * D + self.single_blocks * 3 * D + 2 * D

    def double_mod_offset(self, i: int, stream: str) -> int:
        return i * 12 * self.hidden + (0 if stream == "img" else 6 * self.hidden)

    def single_mod_offset(self, j: int) -> int:
        return self.double_blocks * 12 * self.hidden + j * 3 * self.hidden

    def final_mod_offset(self) -> int:
        return self.double_blocks * 12 * self.hidden + self.single_blocks * 3 * self.hidden

    def num_params(self) -> int:
        D, F = self.hidden, self.mlp_hidden
        dbl = 2 * (3 * D * D + D * D + 2 * D * F)
        sgl = (3 * D + F) * D + (D + F) * D
        emb = D * self.in_channels + D * self.text_dim + 2 * (D * self.timestep_dim + D * D) + D * self.pooled_dim + D * D
        return self.double_blocks * dbl + self.single_blocks * sgl + self.mod_rows * D + emb + self.out_channels * D


PRESETS = {
    "flux-dev": FluxConfig(),
    "flux-schnell": FluxConfig(guidance_embed=False),
    # tiny FLUX-style MMDiT for the CPU float64 parity check.
    "tiny": FluxConfig(hidden=256, heads=4, head_dim=64, double_blocks=2, single_blocks=2,
                       text_dim=256, pooled_dim=256, axes_dim=(8, 28, 28), guidance_embed=False),
    # head_dim-128 variant of the tiny model, runnable on the tcgen05 kernels.
    "tiny128": FluxConfig(hidden=256, heads=2, head_dim=128, double_blocks=2, single_blocks=2,
                          text_dim=256, pooled_dim=256, axes_dim=(16, 56, 56), guidance_embed=True),
}


def get_config(name: str, **overrides) -> FluxConfig:
    return replace(PRESETS[name], **overrides)
