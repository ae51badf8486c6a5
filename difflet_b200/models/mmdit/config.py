"""MMDiT configuration shared by FLUX, HunyuanVideo and Qwen-Image.

All three are dual-stream diffusion transformers with joint attention over a
text stream and an image/video stream, adaLN-Zero modulation, per-head RMS q/k
norm and multi-axis RoPE (reference: ``difflet/models/flux/dit_config.py``,
``difflet/models/hunyuan_video/modeling_hunyuan_video.py:74-128``,
``difflet/models/qwen_image/dit_config.py:40-117``).  What differs is data:
stream order in the joint sequence, number of single-stream blocks, which
embedders feed ``temb``, text preprocessing (HunyuanVideo token refiner,
Qwen-Image text RMSNorm) and the RoPE position ids.
"""

from __future__ import annotations

from dataclasses import dataclass, replace


@dataclass(frozen=True)
class MMDiTConfig:
    family: str = "flux"           # flux | hunyuan_video | qwen_image
    in_channels: int = 64          # latent channels x patch volume
    out_channels: int = 64
    hidden: int = 3072
    heads: int = 24
    head_dim: int = 128
    double_blocks: int = 19
    single_blocks: int = 38
    mlp_ratio: float = 4.0
    text_dim: int = 4096
    pooled_dim: int = 768          # 0 = no pooled-text embedder
    timestep_dim: int = 256
    axes_dim: tuple = (16, 56, 56)
    theta: float = 10000.0
    guidance_embed: bool = True
    eps: float = 1e-6
    order: str = "txt_img"         # joint sequence order: "txt_img" or "img_txt"
    refiner_layers: int = 0        # HunyuanVideo token refiner depth
    txt_norm: bool = False         # Qwen-Image: RMSNorm on the raw text states
    latent_channels: int = 16
    patch: int = 2
    patch_t: int = 1
    vae_scale: int = 8
    vae_scale_t: int = 1

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

    @property
    def streams(self) -> tuple[str, str]:
        return ("txt", "img") if self.order == "txt_img" else ("img", "txt")


FluxConfig = MMDiTConfig

PRESETS = {
    "flux-dev": MMDiTConfig(),
    "flux-schnell": MMDiTConfig(guidance_embed=False),
    # The tiny FLUX-style MMDiT of the CPU float64 parity check (2 + 2 blocks, hidden 256, 4 heads of 64).
    "tiny": MMDiTConfig(hidden=256, heads=4, head_dim=64, double_blocks=2, single_blocks=2, text_dim=256,
                        pooled_dim=256, axes_dim=(8, 28, 28), guidance_embed=False),
    # head_dim-128 variant of the tiny model, runnable on the tcgen05 kernels.
    "tiny128": MMDiTConfig(hidden=256, heads=2, head_dim=128, double_blocks=2, single_blocks=2, text_dim=256,
                           pooled_dim=256, axes_dim=(16, 56, 56), guidance_embed=True),
    # HunyuanVideo 13B: 20 double + 40 single blocks, [video ; text], RoPE theta 256
    "hunyuan-video": MMDiTConfig(family="hunyuan_video", double_blocks=20, single_blocks=40, theta=256.0,
                                 order="img_txt", refiner_layers=2, text_dim=4096, pooled_dim=768,
                                 guidance_embed=True, patch_t=1, vae_scale_t=4),
    "tiny-hunyuan": MMDiTConfig(family="hunyuan_video", hidden=256, heads=2, head_dim=128, double_blocks=2,
                                single_blocks=2, theta=256.0, order="img_txt", refiner_layers=2, text_dim=256,
                                pooled_dim=256, guidance_embed=True, vae_scale_t=4),
    # HunyuanVideo 1.5 (480p T2V): 54 dual-stream blocks, 16 heads, 1x1x1 patches of
    # [32 latent | 32 condition | 1 mask] channels, token-refined Qwen2.5-VL text, true CFG
    "hunyuan-video-1.5": MMDiTConfig(family="hunyuan_video", hidden=2048, heads=16, double_blocks=54,
                                     single_blocks=0, theta=256.0, order="img_txt", refiner_layers=2,
                                     text_dim=3584, pooled_dim=0, guidance_embed=False, in_channels=65,
                                     out_channels=32, latent_channels=32, patch=1, vae_scale=16, vae_scale_t=4),
    # Qwen-Image 20B: 60 dual-stream blocks, Qwen2.5-VL text (3584), no pooled / guidance
    "qwen-image": MMDiTConfig(family="qwen_image", double_blocks=60, single_blocks=0, text_dim=3584, pooled_dim=0,
                              guidance_embed=False, txt_norm=True),
    "tiny-qwen": MMDiTConfig(family="qwen_image", hidden=256, heads=2, head_dim=128, double_blocks=3,
                             single_blocks=0, text_dim=192, pooled_dim=0, guidance_embed=False, txt_norm=True),
}


def get_config(name: str, **overrides) -> MMDiTConfig:
    return replace(PRESETS[name], **overrides)
