"""Decode-free per-step latent telemetry and cross-candidate divergence.

Behaviour of the reference's collector (difflet/pipeline/latent_metrics.py:50-149): per
denoising step and candidate (the leading latent dim), the latent mean / std, the cosine
to candidate 0 and optionally to a reference trajectory; ``shared_prefix_steps`` is the
leading run of steps in which every candidate stays within a cosine threshold of
candidate 0 (how long candidates could share one trajectory).  The JSON schema
(``difflet-latent-metrics-v1``) is kept so existing analysis scripts read these files.

B200 design: ``record`` queues a handful of device reductions and keeps the results on
the device (no host synchronisation inside the denoise loop, so it works inside CUDA
graph-driven loops at no measurable cost); the host sees numbers only when
``to_metrics_dict`` / ``write_json`` is called after the run.  Pass
``collector.callback`` as a pipeline's ``callback``.
"""

from __future__ import annotations

import json
from pathlib import Path
from statistics import mean, pstdev
from typing import Any

import torch

DEFAULT_FORK_COSINE_THRESHOLD = 0.9995
SCHEMA = "difflet-latent-metrics-v1"


def _cos_rows(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """Cosine of every row of x [N, L] with the matching row of y [N, L] (or y [1, L])."""
    dots = (x * y).sum(1)
    return dots / (x.norm(dim=1) * y.norm(dim=1)).clamp_min(1e-30)


class LatentMetricCollector:
    def __init__(self, fork_cosine_threshold: float = DEFAULT_FORK_COSINE_THRESHOLD):
        self.fork_cosine_threshold = float(fork_cosine_threshold)
        self._steps: list[tuple[int, torch.Tensor, torch.Tensor | None]] = []
        self._final: torch.Tensor | None = None
        self._host: list[dict[str, Any]] | None = None

    def record(self, step_index: int, latents: torch.Tensor, *, reference: torch.Tensor | None = None) -> None:
        """latents [N, ...]: N candidates (N = 1 is the single-sample case)."""
        if latents.dim() < 1:
            raise ValueError("latents need a leading candidate dim")
        n = latents.shape[0]
        x = latents.detach().reshape(n, -1).float()
        stats = torch.stack([x.mean(1), x.std(1), _cos_rows(x, x[:1])])  # [3, N] on the device
        ref = None
        if reference is not None:
            r = reference.detach().reshape(reference.shape[0], -1).float()
            ref = _cos_rows(x, r if r.shape[0] == n else r[:1])
        self._steps.append((int(step_index), stats, ref))
        self._final = latents.detach().clone()
        self._host = None

    def callback(self, step_index: int, latents: torch.Tensor) -> None:
        self.record(step_index, latents)

    # ------------------------------------------------------------------ host side
    @property
    def steps(self) -> list[dict[str, Any]]:
        if self._host is None:
            out = []
            for step, stats, ref in self._steps:
                s = stats.cpu().tolist()
                cross = s[2]
                e = {"step": step, "num_candidates": len(cross), "candidate_mean": s[0], "candidate_std": s[1],
                     "cross_candidate_cosine_vs_0": cross, "min_cross_candidate_cosine": min(cross),
                     "candidates_converged": min(cross) >= self.fork_cosine_threshold}
                if ref is not None:
                    e["cosine_vs_reference"] = ref.cpu().tolist()
                out.append(e)
            self._host = out
        return self._host

    @property
    def shared_prefix_steps(self) -> int:
        count = 0
        for e in self.steps:
            if not e["candidates_converged"]:
                break
            count += 1
        return count

    @property
    def shared_prefix_fraction(self) -> float:
        return self.shared_prefix_steps / len(self.steps) if self.steps else 0.0

    def to_metrics_dict(self) -> dict[str, Any]:
        steps = self.steps
        mins = [e["min_cross_candidate_cosine"] for e in steps]
        m: dict[str, Any] = {
            "schema": SCHEMA, "num_steps": len(steps),
            "num_candidates": steps[-1]["num_candidates"] if steps else 0,
            "fork_cosine_threshold": self.fork_cosine_threshold, "per_step": steps,
            "per_step_min_cross_candidate_cosine": mins,
            "min_cross_candidate_cosine_mean": mean(mins) if mins else 1.0,
            "min_cross_candidate_cosine_pstdev": pstdev(mins) if len(mins) > 1 else 0.0,
            "shared_prefix_steps": self.shared_prefix_steps, "shared_prefix_fraction": self.shared_prefix_fraction,
        }
        if self._final is not None:
            f = self._final.float()
            m.update(final_latents_shape=list(f.shape), final_latents_mean=float(f.mean()),
                     final_latents_std=float(f.std()))
        return m

    def write_json(self, path) -> Path:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(json.dumps(self.to_metrics_dict(), indent=2, sort_keys=True) + "\n", encoding="utf-8")
        return path


__all__ = ["DEFAULT_FORK_COSINE_THRESHOLD", "LatentMetricCollector", "SCHEMA"]
