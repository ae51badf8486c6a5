"""Dual-stream MMDiT shared by FLUX, HunyuanVideo and Qwen-Image."""

from difflet_b200.models.mmdit.config import PRESETS, MMDiTConfig, get_config  # noqa: F401
from difflet_b200.models.mmdit.model import MMDiT, pack_latents, unpack_latents  # noqa: F401
