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
