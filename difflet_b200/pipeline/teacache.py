"""TeaCache: skip DiT steps whose input barely changed, reusing the last residual.

Same controller semantics as the reference (``difflet/pipeline/teacache.py:21-405``):
  * adaptive: a calibrated polynomial maps the probe signal (relative L1 change
    of block 0's modulated input since the last full step) to a predicted
    output change; skip when it is below ``threshold`` (or, with
    ``accumulate``, until the accumulated prediction reaches it); committed skip
    runs of ``skip_run_length``
  * cadence: skip every ``cadence``-th step after warm-up (no probe)
  * online-delta: skip when the last full step's relative change of the noise
    prediction is below ``alpha`` x the first measured change; never twice in a row
  * warm-up / cool-down windows always run full steps
  * a skipped step returns ``prev_noise_pred + cached_residual`` where the
    residual is the change between the last two full predictions
On B200 the probe is one fused device reduction (``ops.fused.rel_l1``) that
returns a single scalar.
"""

from __future__ import annotations

import json
from dataclasses import asdict, dataclass, field

import numpy as np
import torch

# Published TeaCache rescale polynomials (highest degree first), per model family.
DEFAULT_COEFFS = {
    "flux": [4.98651651e02, -2.83781631e02, 5.58554382e01, -3.82021401e00, 2.64230861e-01],
    "hunyuan_video": [7.33226126e02, -4.01131952e02, 6.75869174e01, -3.14987800e00, 9.61237896e-02],
    "wan": [-5.21862437e04, 9.23041404e03, -5.28275948e02, 1.36987616e01, -4.99875664e-02],
}


@dataclass
class TeaCacheCalibration:
    coefficients: list = field(default_factory=lambda: list(DEFAULT_COEFFS["flux"]))
    threshold: float = 0.25
    accumulate: bool = True
    warmup_steps: int = 1
    cooldown_steps: int = 1
    num_steps: int = 28
    skip_run_length: int = 1
    cadence: int = 0
    online_delta_alpha: float = 0.0

    def predict_delta(self, signal: float) -> float:
        return float(np.polyval(self.coefficients, signal))

    def to_json(self) -> str:
        return json.dumps(asdict(self))

    @classmethod
    def from_json(cls, s: str) -> "TeaCacheCalibration":
        return cls(**json.loads(s))


# speedup target -> (threshold) for the accumulate mode (reference presets, approximate)
SPEEDUP_THRESHOLDS = {1.5: 0.25, 2.0: 0.4, 2.5: 0.6, 3.0: 0.8}


class TeaCacheController:
    def __init__(self, calibration: TeaCacheCalibration):
        self.cal = calibration
        self.reset()

    def reset(self):
        self.prev_mod_input = None
        self.prev_noise_pred = None
        self.cached_residual = None
        self.full_steps = 0
        self.skipped_steps = 0
        self._accum = 0.0
        self._run = 0
        self._just_skipped = False
        self._last_delta = None
        self._baseline = None
        self.last_signal = None

    def needs_probe(self) -> bool:
        return self.cal.cadence <= 0 and self.cal.online_delta_alpha <= 0 and self._run <= 0

    def should_skip(self, step: int, mod_input, extra=None) -> bool:
        c = self.cal
        if step < c.warmup_steps or step >= c.num_steps - c.cooldown_steps:
            self._run, self._accum = 0, 0.0
            self._update_probe(mod_input)
            return False
        if self.prev_noise_pred is None or self.cached_residual is None:
            self._update_probe(mod_input)
            return False
        if c.cadence > 0:
            pos = step - c.warmup_steps
            return pos % c.cadence == c.cadence - 1
        if c.online_delta_alpha > 0:
            if self._just_skipped:
                self._just_skipped = False
                return False
            if self._last_delta is None or self._baseline is None:
                return False
            return self._last_delta < c.online_delta_alpha * self._baseline
        if self._run > 0:
            self._run -= 1
            return True
        if mod_input is None or self.prev_mod_input is None:
            self._update_probe(mod_input)
            return False
        from difflet_b200.ops import fused as F

        signal = float(F.rel_l1(mod_input, self.prev_mod_input).item())
        self.last_signal = signal
        self._update_probe(mod_input)
        pred = abs(c.predict_delta(signal))
        if c.accumulate:
            self._accum += pred
            if self._accum < c.threshold:
                return True
            self._accum = 0.0
            return False
        skip = pred < c.threshold
        self._run = max(c.skip_run_length - 1, 0) if skip else 0
        return skip

    def _update_probe(self, mod_input):
        if mod_input is not None:
            self.prev_mod_input = mod_input.detach().clone()

    def skip_noise_pred(self):
        if self.prev_noise_pred is None or self.cached_residual is None:
            raise RuntimeError("TeaCache skip before the residual cache was filled")
        self.skipped_steps += 1
        self._just_skipped = True
        v = self.prev_noise_pred + self.cached_residual
        self.prev_noise_pred = v
        return v

    def record_full_step(self, step: int, noise_pred: torch.Tensor):
        self.full_steps += 1
        if self.prev_noise_pred is not None:
            self.cached_residual = (noise_pred - self.prev_noise_pred).detach()
            from difflet_b200.ops import fused as F

            if noise_pred.dtype == torch.bfloat16 and noise_pred.is_cuda:
                d = float(F.rel_l1(noise_pred, self.prev_noise_pred).item())
            else:
                d = float(((noise_pred - self.prev_noise_pred).abs().sum() /
                           self.prev_noise_pred.abs().sum().clamp_min(1e-12)).item())
            self._last_delta = d
            if self._baseline is None:
                self._baseline = d
        self.prev_noise_pred = noise_pred.detach().clone()

    def stats(self) -> dict:
        return {"full_steps": self.full_steps, "skipped_steps": self.skipped_steps}


def build_controller(kw: dict, family: str = "flux", num_steps: int = 28) -> TeaCacheController:
    """From application kwargs: teacache_speedup / teacache_cadence / teacache_online_delta /
    teacache_calibration (JSON path or dict)."""
    cal = TeaCacheCalibration(coefficients=list(DEFAULT_COEFFS.get(family, DEFAULT_COEFFS["flux"])),
                              num_steps=num_steps)
    src = kw.get("teacache_calibration")
    if src:
        if isinstance(src, dict):
            cal = TeaCacheCalibration(**src)
        else:
            cal = TeaCacheCalibration.from_json(open(src).read())
    if kw.get("teacache_speedup"):
        sp = float(kw["teacache_speedup"])
        best = min(SPEEDUP_THRESHOLDS, key=lambda k: abs(k - sp))
        cal.threshold = SPEEDUP_THRESHOLDS[best]
    if kw.get("teacache_cadence"):
        cal.cadence = int(kw["teacache_cadence"])
    if kw.get("teacache_online_delta"):
        cal.online_delta_alpha = float(kw["teacache_online_delta"])
    return TeaCacheController(cal)


def build_probe_free_controller(*, cadence: int | None = None, online_delta_alpha: float | None = None,
                                num_steps: int = 0) -> TeaCacheController:
    """A controller for the modes that need no probe and no calibration file: a fixed cadence
    (skip decisions by step index) or online-delta (from the noise-prediction trajectory the
    pipeline already has).  Exactly one of the two.  ``num_steps`` may stay 0: the pipelines set
    it to the request's step count before denoising, so the cooldown protects the real tail.
    Reference behaviour: difflet/pipeline/teacache.py:365-405."""
    cadence = int(cadence or 0)
    alpha = float(online_delta_alpha or 0.0)
    if cadence <= 0 and alpha <= 0.0:
        raise ValueError(f"a probe-free TeaCache needs cadence > 0 or online_delta_alpha > 0 "
                         f"(got {cadence}, {alpha})")
    if cadence > 0 and alpha > 0.0:
        raise ValueError("cadence and online_delta_alpha exclude each other")
    cal = TeaCacheCalibration(accumulate=False, num_steps=num_steps, cadence=cadence, online_delta_alpha=alpha,
                              coefficients=[0.0], threshold=0.0)
    return TeaCacheController(cal)
