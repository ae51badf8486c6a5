"""Pick a TeaCache mode from a gate trajectory (reference ``difflet/pipeline/teacache_gate.py:44-154``).

Given a short full-step trajectory of (probe signal, true output change)
pairs: if the probe predicts the change well (Pearson r >= ``r_min``) use the
adaptive mode; else if the output changes are smooth (lag-1 autocorrelation
>= ``ac_min``) use online-delta; otherwise a fixed cadence.
"""

from __future__ import annotations

import numpy as np


def pearson(x, y) -> float:
    x, y = np.asarray(x, float), np.asarray(y, float)
    if len(x) < 3 or x.std() == 0 or y.std() == 0:
        return 0.0
    return float(np.corrcoef(x, y)[0, 1])


def lag1_autocorr(y) -> float:
    y = np.asarray(y, float)
    if len(y) < 3 or y.std() == 0:
        return 0.0
    return float(np.corrcoef(y[:-1], y[1:])[0, 1])


def decide_method(signals, deltas, r_min: float = 0.8, ac_min: float = 0.6) -> str:
    if pearson(signals, deltas) >= r_min:
        return "adaptive"
    if lag1_autocorr(deltas) >= ac_min:
        return "online_delta"
    return "cadence"


def fit_coefficients(signals, deltas, degree: int = 4) -> list:
    """Least-squares polynomial (highest degree first) mapping probe signal -> output change."""
    return list(np.polyfit(np.asarray(signals, float), np.asarray(deltas, float), degree))


def _rel_change(cur, prev) -> float:
    """mean |cur - prev| / mean |prev| (f32, on the tensors' device, one host number)."""
    import torch

    c = cur.detach().float() if torch.is_tensor(cur) else torch.as_tensor(cur, dtype=torch.float32)
    p = prev.detach().float() if torch.is_tensor(prev) else torch.as_tensor(prev, dtype=torch.float32)
    return float((c - p).abs().mean() / p.abs().mean().clamp_min(1e-8))


def build_calibration(*, family: str, num_steps: int, signals, deltas, warmup: int = 2, cooldown: int = 2,
                      threshold: float = 0.25, cadence: int = 2, online_alpha: float = 0.25, degree: int = 4):
    """A ``TeaCacheCalibration`` for the method the trajectory supports: adaptive (the probe
    predicts the output change: fitted polynomial + threshold), online-delta (smooth output
    changes), or a fixed cadence."""
    from difflet_b200.pipeline.teacache import DEFAULT_COEFFS, TeaCacheCalibration

    method = decide_method(signals, deltas)
    cal = TeaCacheCalibration(coefficients=list(DEFAULT_COEFFS.get(family, DEFAULT_COEFFS["flux"])),
                              threshold=threshold, warmup_steps=warmup, cooldown_steps=cooldown, num_steps=num_steps)
    if method == "adaptive":
        deg = min(degree, max(1, len(signals) - 1))
        cal.coefficients = fit_coefficients(signals, deltas, deg)
    elif method == "online_delta":
        cal.accumulate, cal.online_delta_alpha = False, float(online_alpha)
    else:
        cal.accumulate, cal.cadence = False, int(cadence)
    return cal, method


def run_gate(*, family: str, num_steps: int, init_latent, step_fn, advance_fn, warmup: int = 2, cooldown: int = 2,
             cadence: int = 2):
    """Run a full denoise trajectory and choose the TeaCache method for this model / shape.

    The model-specific glue is three callables: ``init_latent()``, ``step_fn(i, latent) ->
    (noise_pred, probe_signal or None)`` (the DiT forward with real conditioning and the block-0
    modulated input it saw) and ``advance_fn(latent, noise_pred, i) -> latent`` (one scheduler step).
    Per step the probe signal is the relative change of the probe input and the delta the relative
    change of the noise prediction.  Returns ``(calibration, summary)``; save the calibration with
    ``to_json`` and pass it as ``teacache_calibration``.  Reference behaviour:
    difflet/pipeline/teacache_gate.py:97-154."""
    latent = init_latent()
    prev_out = prev_sig = None
    signals, deltas = [], []
    for i in range(int(num_steps)):
        out, sig = step_fn(i, latent)
        if prev_out is not None:
            deltas.append(_rel_change(out, prev_out))
            if sig is not None and prev_sig is not None:
                signals.append(_rel_change(sig, prev_sig))
        prev_out, prev_sig = out, sig
        latent = advance_fn(latent, out, i)
    if len(signals) != len(deltas):  # no probe: the method comes from the output trajectory alone
        signals = []
    cal, method = build_calibration(family=family, num_steps=num_steps, signals=signals, deltas=deltas,
                                    warmup=warmup, cooldown=cooldown, cadence=cadence)
    summary = {"method": method, "probe_pearson": pearson(signals, deltas) if signals else None,
               "delta_autocorr": lag1_autocorr(deltas), "n_pairs": len(deltas)}
    return cal, summary


__all__ = ["build_calibration", "decide_method", "fit_coefficients", "lag1_autocorr", "pearson", "run_gate"]
