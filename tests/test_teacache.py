"""TeaCache controller modes and the FLUX pipeline integration (CPU)."""

import torch

from difflet_b200.models.flux.config import get_config
from difflet_b200.models.flux.model import FluxTransformer
from difflet_b200.models.flux.pipeline import FluxApplication
from difflet_b200.pipeline.teacache import TeaCacheCalibration, TeaCacheController, build_controller
from difflet_b200.pipeline.teacache_gate import decide_method, fit_coefficients


def test_cadence_mode_and_residual_reuse():
    c = TeaCacheController(TeaCacheCalibration(cadence=2, warmup_steps=1, cooldown_steps=1, num_steps=8))
    preds = []
    for i in range(8):
        if c.should_skip(i, None):
            v = c.skip_noise_pred()
        else:
            v = torch.full((4,), float(i))
            c.record_full_step(i, v)
        preds.append(v.clone())
    assert c.skipped_steps > 0 and c.full_steps + c.skipped_steps == 8
    # a skipped step extrapolates by the last residual
    for i, v in enumerate(preds):
        if float(v[0]) != float(i):
            assert float(v[0]) == float(preds[i - 1][0]) + 1.0


def test_adaptive_mode_skips_when_input_static():
    cal = TeaCacheCalibration(coefficients=[1.0, 0.0], threshold=0.5, accumulate=True, warmup_steps=0,
                              cooldown_steps=0, num_steps=10)
    c = TeaCacheController(cal)
    x = torch.ones(64)
    skips = 0
    for i in range(10):
        if c.should_skip(i, x):
            c.skip_noise_pred()
            skips += 1
        else:
            c.record_full_step(i, torch.randn(8))
    assert skips >= 5  # identical inputs -> zero signal -> skip after the cache fills


def test_gate():
    s = [0.1, 0.2, 0.3, 0.4, 0.5]
    assert decide_method(s, [1, 2, 3, 4, 5]) == "adaptive"
    assert len(fit_coefficients(s, [1, 2, 3, 4, 5], degree=2)) == 3


def test_flux_pipeline_with_teacache_runs_fewer_steps():
    cfg = get_config("tiny128")
    dit = FluxTransformer.random_init(cfg, seed=1)
    app = FluxApplication(dit, None, text_len=16)
    app.teacache = build_controller({"teacache_cadence": 2})
    out = app.generate(prompt="x", height=64, width=64, num_inference_steps=8, output_type="latent")
    assert torch.isfinite(out).all() and app.teacache.skipped_steps >= 2


def test_run_gate_picks_a_method_and_calibrates():
    """run_gate on a synthetic trajectory: a probe proportional to the output change -> adaptive
    with a fitted polynomial; no probe and smooth changes -> online-delta."""
    import torch

    from difflet_b200.pipeline.teacache_gate import run_gate

    g = torch.Generator().manual_seed(0)
    scales = [1.0 + 0.5 * i + 0.05 * float(torch.rand(1, generator=g)) for i in range(12)]

    def step(i, lat):
        return lat * scales[i], lat * (scales[i] ** 0.5)

    cal, summ = run_gate(family="flux", num_steps=12, init_latent=lambda: torch.ones(64),
                         step_fn=step, advance_fn=lambda lat, out, i: lat)
    assert summ["method"] == "adaptive" and summ["n_pairs"] == 11
    assert cal.accumulate and len(cal.coefficients) >= 2
    cal2, summ2 = run_gate(family="flux", num_steps=12, init_latent=lambda: torch.ones(64),
                           step_fn=lambda i, lat: (lat * (1 + 0.1 * i), None), advance_fn=lambda lat, out, i: lat)
    assert summ2["probe_pearson"] is None and summ2["method"] in ("online_delta", "cadence")
    assert (cal2.online_delta_alpha > 0) != (cal2.cadence > 0)


def test_probe_free_controller():
    import pytest

    from difflet_b200.pipeline.teacache import build_probe_free_controller

    c = build_probe_free_controller(cadence=2)
    assert c.cal.cadence == 2 and not c.needs_probe()
    with pytest.raises(ValueError):
        build_probe_free_controller()
    with pytest.raises(ValueError):
        build_probe_free_controller(cadence=2, online_delta_alpha=0.3)
