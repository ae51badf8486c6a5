"""``--mode latency | throughput | mixed``: parallel layout presets by model class and GPU count.

Reference behaviour (``difflet/cli/modes.py:20-71``): a model is ``distilled`` (one pass per
step: the cfg lane is free), ``true_cfg`` (two CFG branches, context parallelism available) or
``true_cfg_no_cp``; latency spends the devices on one request, throughput on replicas, mixed on
both; explicitly given flags win over the preset.  The reference's table is fixed to a
four-device host.  Here the preset is computed for the GPUs of this node and the model's head
count (Ulysses needs heads % cp == 0; every registered model fits one B200's 180 GB, so a
throughput replica is one GPU):

  latency     dp 1; true CFG: cfg2 x cp(N / 2); distilled: cp(N)
  throughput  dp N, one GPU per replica
  mixed       dp 2; the remaining N / 2 GPUs of a replica as in latency
"""

from __future__ import annotations

from dataclasses import dataclass

MODES = ("latency", "throughput", "mixed")


def model_class(model_id: str) -> str:
    from difflet_b200.registry import resolve_model

    cap = resolve_model(model_id).capabilities
    if cap.is_distilled:
        return "distilled"
    return "true_cfg" if cap.supports_cp else "true_cfg_no_cp"


@dataclass(frozen=True)
class ModeConfig:
    dp: int
    cfg_parallel: bool
    cp_degree: int
    cp_mode: str


def _largest_cp(n: int, heads: int) -> int:
    """The largest context-parallel degree <= n that divides the head count (Ulysses)."""
    for c in range(max(1, n), 0, -1):
        if heads % c == 0 and n % c == 0:
            return c
    return 1


def preset(model_id: str, mode: str, gpus: int) -> ModeConfig:
    if mode not in MODES:
        raise ValueError(f"unknown mode {mode!r}; choose one of {', '.join(MODES)}")
    from difflet_b200.registry import resolve_model

    klass = model_class(model_id)
    heads = resolve_model(model_id).capabilities.num_attention_heads
    gpus = max(1, gpus)
    if mode == "throughput":
        return ModeConfig(dp=gpus, cfg_parallel=False, cp_degree=1, cp_mode="gather_kv")
    dp = 2 if (mode == "mixed" and gpus >= 2) else 1
    per = gpus // dp
    cfg = klass != "distilled" and per >= 2
    lanes = per // 2 if cfg else per
    cp = 1 if klass == "true_cfg_no_cp" else _largest_cp(lanes, heads)
    return ModeConfig(dp=dp, cfg_parallel=cfg, cp_degree=cp, cp_mode="ulysses" if cp > 1 else "gather_kv")


def apply_mode(a, gpus: int | None = None) -> ModeConfig | None:
    """Fill the parallel flags the user left unset (None) from ``--mode``; then the defaults."""
    mode = getattr(a, "mode", None)
    cfg = None
    if mode is not None:
        if gpus is None:
            try:
                import torch

                gpus = torch.cuda.device_count() or 1
            except Exception:  # noqa: BLE001
                gpus = 1
        cfg = preset(a.model_id, mode, gpus)
        if getattr(a, "dp", None) is None:
            a.dp = cfg.dp
        if hasattr(a, "dp_degree") and a.dp_degree is None:
            a.dp_degree = cfg.dp
        if not a.cfg_parallel:
            a.cfg_parallel = cfg.cfg_parallel
        if a.cp_degree is None:
            a.cp_degree = cfg.cp_degree
            if a.cp_mode is None and cfg.cp_degree > 1:
                a.cp_mode = cfg.cp_mode
    for name in ("dp", "cp_degree", "tp_degree", "dp_degree"):
        if hasattr(a, name) and getattr(a, name) is None:
            setattr(a, name, 1)
    return cfg


__all__ = ["MODES", "ModeConfig", "apply_mode", "model_class", "preset"]
