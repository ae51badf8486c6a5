"""Schedulers: flow-match Euler schedule and UniPC on an exactly solvable flow."""

import math

import numpy as np
import torch

from difflet_b200.schedulers import FlowMatchEulerScheduler, flux_time_shift_mu
from difflet_b200.schedulers.unipc import UniPCScheduler


def test_flux_schedule_shape_and_shift():
    s = FlowMatchEulerScheduler().set_timesteps(28, mu=flux_time_shift_mu(4096))
    assert len(s.timesteps) == 28 and s.sigmas[-1] == 0.0
    assert abs(flux_time_shift_mu(4096) - 1.15) < 1e-9 and abs(flux_time_shift_mu(256) - 0.5) < 1e-9
    assert np.all(np.diff(s.sigmas) < 0) and abs(s.sigmas[0] - 1.0) < 1e-6


def test_unipc_recovers_single_point_data():
    # data = one point x0: the exact flow velocity is v = (x - x0) / sigma, every
    # x0-prediction equals x0, so a consistent solver must land on x0.
    x0 = torch.randn(4, 8, dtype=torch.float64)
    sch = UniPCScheduler(shift=5.0).set_timesteps(20)
    x = torch.randn(4, 8, dtype=torch.float64)
    for i in range(20):
        sigma = float(sch.sigmas[i])
        v = (x - x0) / sigma
        x = sch.step(v, x)
    assert (x - x0).abs().max().item() < 1e-6


def test_unipc_second_order_beats_first_order_on_gaussian_flow():
    # data ~ N(mu, s^2): exact x0-prediction for flow matching is known in closed form
    mu, s = 1.5, 0.3

    def v_exact(x, sigma):
        a = 1 - sigma
        var = (a * s) ** 2 + sigma ** 2
        x0 = mu + a * s * s * (x - a * mu) / var
        return (x - x0) / sigma

    def run(order, n):
        sch = UniPCScheduler(shift=1.0, solver_order=order).set_timesteps(n)
        g = torch.Generator().manual_seed(0)
        z = torch.randn(20000, generator=g, dtype=torch.float64)
        x = z.clone()
        for i in range(n):
            x = sch.step(v_exact(x, float(sch.sigmas[i])), x)
        # exact transport of the noise z (deterministic ODE): x = mu + s * z
        return (x - (mu + s * z)).abs().mean().item()

    e1, e2 = run(1, 8), run(2, 8)
    assert e2 < e1
