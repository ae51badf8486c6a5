"""Diffusion schedulers: flow-matching Euler (FLUX / HunyuanVideo / Qwen-Image) and UniPC (Wan)."""

from difflet_b200.schedulers.flow_match import FlowMatchEulerScheduler, flux_time_shift_mu  # noqa: F401
