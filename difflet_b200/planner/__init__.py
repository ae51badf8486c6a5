"""Parallel-configuration planner for B200 / NVSwitch.

Same role as the reference planner (``difflet/planner/feasibility.py:135``,
``cost_model.py:107-202``, ``planner.py:116``): enumerate the legal
``DiffletParallelConfig``s for a model and GPU count (head divisibility, CFG
only for true-CFG models, the model's CP modes), estimate a denoise step as

    T = FLOPs / (world_model * peak * eff(rows per rank)) + comm_bytes / link_bw
        + n_sync * sync_latency

and rank them.  On NVSwitch every GPU pair has the same bandwidth, so the
reference's topology-aware placement stage is trivial (identity placement).
Peaks are the measured ones of this pool; ``calibrate`` fits the efficiency
scale to measured step times.
"""

from __future__ import annotations

import itertools
import math

from difflet_b200.pipeline.parallel_config import DiffletParallelConfig
from difflet_b200.registry import resolve_model

LINK_BW = 770e9          # measured peer copy, bytes/s per direction per GPU
SYNC_S = 6e-6            # one device barrier over NVLink
_EFF_SCALE = [0.85]      # calibrated fraction of the measured GEMM peak


def model_shape(entry, height=None, width=None, num_frames=None) -> dict:
    """Per-step workload: tokens, hidden, layers, heads, and ``params`` = the weights of the linears
    every token passes through (MMDiT dual blocks count one stream; the per-step modulation
    GEMVs are not token work)."""
    s = entry.resolve_shape(height=height, width=width, num_frames=num_frames)
    h, w, f = s.get("height") or 1024, s.get("width") or 1024, s.get("num_frames")
    if entry.name == "wan":
        t = ((f or 81) - 1) // 4 + 1
        return dict(tokens=t * (h // 16) * (w // 16), text=512, hidden=5120, layers=40, heads=40, params=14e9,
                    mlp=13824 / 5120)
    if entry.name.startswith("hunyuan_video"):
        t = ((f or 129) - 1) // 4 + 1
        return dict(tokens=t * (h // 16) * (w // 16), text=256, hidden=3072, layers=60, heads=24, params=13e9, mlp=4)
    if entry.name == "qwen_image":
        return dict(tokens=(h // 16) * (w // 16), text=256, hidden=3072, layers=60, heads=24, params=20e9, mlp=4)
    # FLUX.1: 19 dual blocks (one stream per token: 113 M) + 38 single blocks (113 M)
    return dict(tokens=(h // 16) * (w // 16), text=512, hidden=3072, layers=57, heads=24, params=6.45e9, mlp=4)


def enumerate_candidates(entry, gpus: int, exact: bool = True) -> list[DiffletParallelConfig]:
    caps = entry.capabilities
    out = []
    divs = [d for d in range(1, gpus + 1) if gpus % d == 0]
    for tp, cp, cfg, dp in itertools.product(divs, divs, (False, True), divs):
        world = tp * cp * (2 if cfg else 1) * dp
        if world > gpus or (exact and world != gpus):
            continue
        modes = ["ulysses", "ring", "gather_kv"] if cp > 1 else ["gather_kv"]
        for mode in modes:
            try:
                p = DiffletParallelConfig(tp_degree=tp, cp_degree=cp, cfg_parallel_enabled=cfg, cp_mode=mode,
                                          dp_degree=dp)
                if caps is not None:
                    caps.check_parallel(p)
            except ValueError:
                continue
            out.append(p)
    return out


def _eff(rows: int) -> float:
    # GEMM efficiency falls off once each rank has fewer rows than ~2 waves of 128-row tiles
    return _EFF_SCALE[0] * min(1.0, rows / 2048.0) ** 0.35


ATTN_EFF = 0.80  # flash attention's measured fraction of the sustained GEMM peak (FLUX 24 x 4608)
ATTN_EFF_LONG = 0.89  # ... at video lengths (HunyuanVideo 118,800 tokens: per-tile overheads amortised)


def _attn_eff(seq: int) -> float:
    """Attention efficiency rising with the key length, log-linear from 5,120 to 118,800 keys."""
    x = math.log(max(seq, 5120) / 5120) / math.log(118800 / 5120)
    return ATTN_EFF + (ATTN_EFF_LONG - ATTN_EFF) * min(1.0, x)
KERNEL_TAIL_S = 3e-6  # fill / drain of one launch inside the CUDA graph
KERNELS_PER_LAYER = 8
N_SMS = 148


def _attn_occupancy(heads_per_rank: int, seq: int) -> float:
    """Fraction of the SMs the attention grid keeps busy (256-query CTAs; grids under half the
    SMs split the key range in two)."""
    ctas = max(1, heads_per_rank) * math.ceil(seq / 256)
    if ctas * 2 <= N_SMS:
        ctas *= 2
    return ctas / (math.ceil(ctas / N_SMS) * N_SMS)


def estimate_step_s(entry, p: DiffletParallelConfig, shape: dict, peak_flops: float) -> float:
    S = shape["tokens"] + shape["text"]
    D, L = shape["hidden"], shape["layers"]
    cfg_mult = 1 if (entry.capabilities and entry.capabilities.is_distilled) else 2
    gemm_flops = 2.0 * shape["params"] * S * cfg_mult
    attn_flops = 4.0 * L * S * S * D * cfg_mult
    world_model = p.tp_degree * p.cp_degree * (2 if p.cfg_parallel_enabled else 1)
    rows = S // p.cp_degree
    heads_rank = max(1, shape["heads"] // (p.tp_degree * p.cp_degree))
    t_comp = gemm_flops / (world_model * peak_flops * _eff(rows)) + attn_flops / (
        world_model * peak_flops * _attn_eff(S) * _attn_occupancy(heads_rank, S))
    act = S * D * 2 / max(1, p.cp_degree)  # bytes of one activation shard
    comm = 0.0
    syncs = 0
    if p.cp_degree > 1:
        f = (p.cp_degree - 1) / p.cp_degree
        if p.cp_mode == "ulysses":
            comm += L * 4 * act * f
            syncs += 2 * L
        elif p.cp_mode == "ring":
            comm += L * 2 * act * (p.cp_degree - 1)
            syncs += L * p.cp_degree
        else:
            comm += L * 2 * act * (p.cp_degree - 1)
            syncs += L
    if p.tp_degree > 1:
        comm += L * 2 * 2 * act * (p.tp_degree - 1) / p.tp_degree
        syncs += 4 * L
    if p.cfg_parallel_enabled:
        comm += shape["tokens"] * 64 * 2
        syncs += 2
    t_comm = comm / LINK_BW / max(1.0, 0.5 * (1 + (p.cp_degree > 1)))  # partial overlap with compute
    return t_comp + t_comm + syncs * SYNC_S + L * KERNELS_PER_LAYER * KERNEL_TAIL_S


def plan(model_id: str, *, gpus: int = 8, height=None, width=None, num_frames=None, exact: bool = True) -> list[dict]:
    from difflet_b200.utils.peaks import load_peaks

    entry = resolve_model(model_id)
    shape = model_shape(entry, height, width, num_frames)
    peak = load_peaks()["bf16_tflops_sustained"] * 1e12
    rows = []
    for p in enumerate_candidates(entry, gpus, exact=exact):
        t = estimate_step_s(entry, p, shape, peak)
        rows.append({"parallel": p.to_cache_dict(), "world": p.world_size, "dp": p.dp_degree,
                     "est_step_ms": round(t * 1e3, 2), "est_throughput_steps_per_s": round(p.dp_degree / t, 2)})
    rows.sort(key=lambda r: (r["est_step_ms"], -r["dp"]))
    return rows


def calibrate(measurements: list[tuple[float, float]]) -> float:
    """measurements: (estimated_s, measured_s) pairs -> new efficiency scale (least squares on the ratio)."""
    if not measurements:
        return _EFF_SCALE[0]
    ratio = sum(e / m for e, m in measurements) / len(measurements)
    _EFF_SCALE[0] = max(0.05, min(1.0, _EFF_SCALE[0] * ratio))
    return _EFF_SCALE[0]
