"""Flow-matching Euler scheduler.

Same schedule as diffusers' ``FlowMatchEulerDiscreteScheduler`` used by the
reference FLUX / HunyuanVideo / Qwen-Image pipelines
(``difflet/models/flux/pipeline.py:46-460``): sigmas linearly spaced from 1 to
1/N, optionally shifted by ``exp(mu) / (exp(mu) + (1/sigma - 1))`` (dynamic,
resolution-dependent ``mu``) or by a static ``shift``, with a terminal 0.  The
update ``x <- x + (sigma_{i+1} - sigma_i) * v`` runs on the device in fp32
(fused with the CFG combine when there is one).
"""

from __future__ import annotations

import math

import numpy as np


def flux_time_shift_mu(image_seq_len: int, base_seq_len: int = 256, max_seq_len: int = 4096,
                       base_shift: float = 0.5, max_shift: float = 1.15) -> float:
    m = (max_shift - base_shift) / (max_seq_len - base_seq_len)
    b = base_shift - m * base_seq_len
    return image_seq_len * m + b


class FlowMatchEulerScheduler:
    def __init__(self, num_train_timesteps: int = 1000, shift: float = 1.0, use_dynamic_shifting: bool = True):
        self.num_train_timesteps = num_train_timesteps
        self.shift = shift
        self.use_dynamic_shifting = use_dynamic_shifting
        self.sigmas = None
        self.timesteps = None

    def set_timesteps(self, num_inference_steps: int, mu: float | None = None, sigmas=None):
        if sigmas is None:
            sigmas = np.linspace(1.0, 1.0 / num_inference_steps, num_inference_steps)
        sigmas = np.asarray(sigmas, dtype=np.float64)
        if self.use_dynamic_shifting:
            if mu is None:
                raise ValueError("dynamic shifting needs mu")
            sigmas = math.exp(mu) / (math.exp(mu) + (1.0 / sigmas - 1.0))
        elif self.shift != 1.0:
            sigmas = self.shift * sigmas / (1 + (self.shift - 1) * sigmas)
        self.timesteps = (sigmas * self.num_train_timesteps).astype(np.float32)
        self.sigmas = np.concatenate([sigmas, [0.0]]).astype(np.float32)
        return self

    def dt(self, i: int) -> float:
        return float(self.sigmas[i + 1]) - float(self.sigmas[i])

    def __len__(self):
        return 0 if self.timesteps is None else len(self.timesteps)
