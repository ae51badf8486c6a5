"""Roofline denominators: the measured B200 peaks of this pool (copy bandwidth, cuBLAS bf16)."""

from __future__ import annotations

import json
from pathlib import Path

FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "nvlink_gbs_per_dir": 770.0, "source": "fallback"}


def load_peaks() -> dict:
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    out = dict(FALLBACK)
    if p.exists():
        try:
            d = json.loads(p.read_text())
            out.update({k: d[k] for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained") if k in d})
            out["source"] = "measured"
        except Exception:
            pass
    return out
