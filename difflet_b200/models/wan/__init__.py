"""Wan 2.1 / 2.2 text-to-video: DiT, UniPC denoise loop, causal 3-D VAE."""
