"""MiniMax-H3's data-ward rectified-flow Euler scheduler (behaviour of
difflet/models/minimax_h3/scheduling_minimax_h3.py:1-170).

``t = 1 - sigma``; the grid is ``sigma_i = shift b / (1 + (shift - 1) b)`` for
``b = linspace(1, 0, N)`` with consecutive duplicates removed (the terminal 0 is one
of the N points); the model predicts a velocity towards the data, so
``x0 = x + sigma v`` and ``x_next = (sigma_next / sigma) x + (1 - sigma_next / sigma) x0``.
"""

from __future__ import annotations

import torch


class RectifiedFlowScheduler:
    def __init__(self, shift: float = 12.0):
        if shift <= 0:
            raise ValueError(f"shift must be positive, got {shift}")
        self.shift = float(shift)
        self.sigmas = None
        self.timesteps = None

    def set_timesteps(self, num_inference_steps: int | None = None, sigmas=None):
        if sigmas is None:
            if num_inference_steps is None or num_inference_steps < 2:
                raise ValueError("set_timesteps needs explicit sigmas or num_inference_steps >= 2")
            b = torch.linspace(1.0, 0.0, int(num_inference_steps), dtype=torch.float32)
            sig = torch.unique_consecutive(self.shift * b / (1 + (self.shift - 1) * b))
        else:
            sig = torch.as_tensor(sigmas, dtype=torch.float32).flatten()
            if sig.numel() < 2 or not bool((sig[1:] < sig[:-1]).all()) or float(sig[-1]) != 0.0:
                raise ValueError("sigmas must be at least two strictly decreasing values ending at 0.0")
        self.sigmas = sig
        self.timesteps = 1.0 - sig[:-1]
        return self

    def __len__(self):
        return 0 if self.timesteps is None else int(self.timesteps.numel())

    @staticmethod
    def scale_noise(sample, t, noise):
        return t * sample + (1.0 - t) * noise

    def step(self, velocity: torch.Tensor, i: int, sample: torch.Tensor) -> torch.Tensor:
        sigma, sigma_next = float(self.sigmas[i]), float(self.sigmas[i + 1])
        sigma_t = 1.0 - float(self.timesteps[i])
        denoised = sample.float() + sigma_t * velocity.float()
        r = sigma_next / sigma
        return r * sample.float() + (1.0 - r) * denoised


__all__ = ["RectifiedFlowScheduler"]
