"""UniPC multistep scheduler (flow prediction), data-prediction form, B(h) = expm1(h).

UniPC (Zhao et al., "UniPC: A Unified Predictor-Corrector Framework for Fast
Sampling of Diffusion Models", 2023) as configured by the Wan pipelines
(reference ``difflet/models/wan/pipeline.py:525-582``, diffusers
``UniPCMultistepScheduler`` with ``prediction_type='flow_prediction'``,
``use_flow_sigmas``, ``solver_order=2``, ``solver_type='bh2'``,
``lower_order_final``).  For flow matching, alpha_t = 1 - sigma_t and the
model's velocity converts to a data prediction x0 = x - sigma * v.

Each step is: corrector (UniC) on the current sample using the new model
output, then predictor (UniP) to the next sigma.  The per-step scalar
coefficients are computed on the host in float64; the tensor updates are
linear combinations evaluated on the device in fp32 (the reference keeps fp32
latents because the corrector is unstable in bf16).
"""

from __future__ import annotations

import math

import numpy as np
import torch


class UniPCScheduler:
    def __init__(self, num_train_timesteps: int = 1000, shift: float = 5.0, solver_order: int = 2,
                 lower_order_final: bool = True, disable_corrector=()):
        self.T = num_train_timesteps
        self.shift = shift
        self.order = solver_order
        self.lower_order_final = lower_order_final
        self.disable_corrector = set(disable_corrector)

    def set_timesteps(self, num_inference_steps: int):
        n = num_inference_steps
        alphas = np.linspace(1.0, 1.0 / self.T, n + 1)
        sigmas = 1.0 - alphas
        sigmas = np.flip(self.shift * sigmas / (1 + (self.shift - 1) * sigmas))[:-1].copy()
        self.timesteps = (sigmas * self.T).astype(np.float64)
        self.sigmas = np.concatenate([sigmas, [0.0]]).astype(np.float64)
        self.num_steps = n
        self.model_outputs: list = [None] * self.order
        self.last_sample = None
        self.lower_order_nums = 0
        self.step_index = 0
        self.this_order = 1
        return self

    # ---------------------------------------------------------------- helpers
    @staticmethod
    def _lam(sigma: float) -> float:
        alpha = 1.0 - sigma
        if sigma <= 0.0:
            return math.inf
        if alpha <= 0.0:
            return -math.inf
        return math.log(alpha) - math.log(sigma)

    def _coeffs(self, order: int, lam_t: float, lam_s0: float, lam_prev: list):
        """Return (h_phi_1, B_h, rks, b) for the data-prediction UniPC update."""
        h = lam_t - lam_s0
        hh = -h
        h_phi_1 = math.expm1(hh)
        B_h = math.expm1(hh)
        rks = [(lp - lam_s0) / h for lp in lam_prev] + [1.0]
        if math.isinf(h):
            rks = [0.0 for _ in lam_prev] + [1.0]
        b = []
        h_phi_k = (h_phi_1 / hh - 1.0) if not math.isinf(hh) else -1.0
        fact = 1
        for i in range(1, order + 1):
            b.append(h_phi_k * fact / B_h)
            fact *= i + 1
            h_phi_k = (h_phi_k / hh - 1.0 / fact) if not math.isinf(hh) else -1.0 / fact
        return h_phi_1, B_h, rks, b

    def _x0(self, v: torch.Tensor, x: torch.Tensor, sigma: float) -> torch.Tensor:
        return x - sigma * v.float()

    # ---------------------------------------------------------------- step
    def step(self, model_output: torch.Tensor, sample: torch.Tensor) -> torch.Tensor:
        """model_output: predicted velocity (any float dtype); sample: fp32 latents.
        Returns the next fp32 sample."""
        m_t = self._x0(model_output, sample, float(self.sigmas[self.step_index]))
        return self._advance(m_t, sample)

    def fused_coeffs(self):
        """This step's update as weights over the sampler state u = (x, last, m1, m2, m) (x the
        current sample, last the previous corrected sample, m1 / m2 the previous two data
        predictions, m = x - sigma v this step's), for the fused guidance + sampler kernel.

        The corrector and predictor are linear in u, so the weights are what ``_advance`` returns
        when it runs on the basis vectors of u instead of tensors: the same code, the same
        bookkeeping (order warm-up, lower-order final steps).  Returns (k_v, e, g): m = x + k_v v,
        corrected sample xc = e . u, next sample xn = g . u (+ g[5] v, zero here)."""
        bx, blast, bm1, bm2, bm = np.eye(5)
        i = self.step_index
        have = [o is not None for o in self.model_outputs]
        # where step() would hold tensors, hold the matching basis vectors (history newest last)
        basis_hist = [bm2, bm1][-len(have):] if len(have) <= 2 else [None] * (len(have) - 2) + [bm2, bm1]
        self.model_outputs = [b if h else None for b, h in zip(basis_hist, have)]
        had_last = self.last_sample is not None
        self.last_sample = blast if had_last else None
        xn = self._advance(bm, bx)
        xc = self.last_sample
        # back to presence markers: the tensors themselves live in the caller's device buffers
        self.model_outputs = [True if o is not None else None for o in self.model_outputs]
        self.last_sample = True
        return -float(self.sigmas[i]), [float(c) for c in xc], [float(c) for c in xn] + [0.0]

    def _advance(self, m_t, sample):
        """Corrector on ``sample`` with the new data prediction ``m_t``, history shift, predictor."""
        i = self.step_index
        use_corr = i > 0 and (i - 1) not in self.disable_corrector and self.last_sample is not None
        if use_corr:
            sample = self._corrector(m_t, sample)
        for k in range(self.order - 1):
            self.model_outputs[k] = self.model_outputs[k + 1]
        self.model_outputs[-1] = m_t
        if self.lower_order_final:
            this_order = min(self.order, self.num_steps - i)
        else:
            this_order = self.order
        self.this_order = min(this_order, self.lower_order_nums + 1)
        self.last_sample = sample
        out = self._predictor(sample, self.this_order)
        if self.lower_order_nums < self.order:
            self.lower_order_nums += 1
        self.step_index += 1
        return out

    def _predictor(self, x: torch.Tensor, order: int) -> torch.Tensor:
        i = self.step_index
        s_t, s_s0 = float(self.sigmas[i + 1]), float(self.sigmas[i])
        alpha_t = 1.0 - s_t
        lam_t, lam_s0 = self._lam(s_t), self._lam(s_s0)
        m0 = self.model_outputs[-1]
        lam_prev = [self._lam(float(self.sigmas[i - k])) for k in range(1, order)]
        h_phi_1, B_h, rks, b = self._coeffs(order, lam_t, lam_s0, lam_prev)
        ratio = s_t / s_s0 if s_s0 > 0 else 0.0
        x_t = ratio * x - alpha_t * h_phi_1 * m0
        if order >= 2:
            D1s = [(self.model_outputs[-(k + 1)] - m0) / rks[k - 1] for k in range(1, order)]
            if order == 2:
                rhos = [0.5]
            else:
                R = np.array([[rk ** (p) for rk in rks[:-1]] for p in range(order - 1)])
                rhos = list(np.linalg.solve(R, np.array(b[:-1])))
            res = sum(r * d for r, d in zip(rhos, D1s))
            x_t = x_t - alpha_t * B_h * res
        return x_t

    def _corrector(self, m_t: torch.Tensor, x_t: torch.Tensor) -> torch.Tensor:
        i = self.step_index
        order = self.this_order
        x = self.last_sample
        s_t, s_s0 = float(self.sigmas[i]), float(self.sigmas[i - 1])
        alpha_t = 1.0 - s_t
        lam_t, lam_s0 = self._lam(s_t), self._lam(s_s0)
        m0 = self.model_outputs[-1]
        lam_prev = [self._lam(float(self.sigmas[i - (k + 1)])) for k in range(1, order)]
        h_phi_1, B_h, rks, b = self._coeffs(order, lam_t, lam_s0, lam_prev)
        D1s = [(self.model_outputs[-(k + 1)] - m0) / rks[k - 1] for k in range(1, order)]
        if order == 1:
            rhos = [0.5]
        else:
            R = np.array([[rk ** p for rk in rks] for p in range(order)])
            rhos = list(np.linalg.solve(R, np.array(b)))
        ratio = s_t / s_s0 if s_s0 > 0 else 0.0
        x_t_ = ratio * x - alpha_t * h_phi_1 * m0
        corr = sum(r * d for r, d in zip(rhos[:-1], D1s)) if D1s else 0.0
        return x_t_ - alpha_t * B_h * (corr + rhos[-1] * (m_t - m0))
