"""Per-(block, linear) bf16 / MXFP8 precision schedules: artefacts, synthesis, calibration, apply.

Artefact behaviour follows the reference (difflet/pipeline/precision_schedule.py:41-121,
135-287): a schedule maps cells ``"<block>:<linear>"`` to ``bf16`` / ``mxfp8_e4m3`` /
``mxfp8_e5m2``; schedules are synthesised from a calibration table (one cosine per cell,
or per-format cosines) with one threshold (E4M3 when cos >= tau) or two (E4M3 when
e4m3_cos >= tau_hi, else E5M2 when e5m2_cos >= tau_lo, else bf16); JSON schema_version 1
is kept so schedules move between the two engines.

B200 additions:
  * ``calibrate``: measures each fused weight's output cosine (bf16 vs MXFP8 weight) on a
    seeded Gaussian probe with this engine's own quantizer, producing the table.
  * ``apply_schedule``: quantizes the fused GEMM weights whose every diffusers linear is
    scheduled E4M3 (the block-scaled tcgen05 GEMM runs them); E5M2 cells run in bf16 here
    (the tensor-core MX path of this build is E4M3) and are reported as such.
Cells: ``block`` is the index in the diffusers block list, ``linear`` the diffusers module
path with the block list's name in front (``transformer_blocks/attn.to_q``), so FLUX's
dual and single blocks do not collide.
"""

from __future__ import annotations

import json
import re
from dataclasses import dataclass
from pathlib import Path
from typing import Iterable

PRECISION_BF16 = "bf16"
PRECISION_MXFP8_E4M3 = "mxfp8_e4m3"
PRECISION_MXFP8_E5M2 = "mxfp8_e5m2"
_MX = (PRECISION_MXFP8_E4M3, PRECISION_MXFP8_E5M2)
SCHEMA_VERSION = 1
_ALIASES = {
    PRECISION_BF16: ("bf16", "bfloat16", "torch.bfloat16"),
    PRECISION_MXFP8_E4M3: ("mx", "mxfp8", "mxfp8_e4m3", "e4m3", "float8_e4m3fn_x4"),
    PRECISION_MXFP8_E5M2: ("mxfp8_e5m2", "e5m2", "float8_e5m2_x4"),
}


def normalize_precision(value: str) -> str:
    v = str(value).lower()
    for canon, names in _ALIASES.items():
        if v in names:
            return canon
    raise ValueError(f"unsupported precision: {value!r}")


def cell_key(block: int, linear: str) -> str:
    return f"{int(block)}:{linear}"


_CELL_RE = re.compile(r"^(?P<list>[A-Za-z_]+)\.(?P<block>\d+)\.(?P<rest>.+)$")


def cell_of(module_name: str) -> str:
    """``transformer_blocks.3.attn.to_q`` -> ``3:transformer_blocks/attn.to_q``."""
    m = _CELL_RE.match(module_name)
    if m is None:
        raise ValueError(f"not a per-block linear: {module_name!r}")
    return cell_key(int(m["block"]), f"{m['list']}/{m['rest']}")


@dataclass(frozen=True)
class PrecisionSchedule:
    model_id: str
    bundle: str
    tau: float | None
    assignments: dict
    metadata: dict | None = None

    def __post_init__(self):
        object.__setattr__(self, "assignments",
                           {str(k): normalize_precision(v) for k, v in self.assignments.items()})
        object.__setattr__(self, "metadata", dict(self.metadata or {}))

    @property
    def mx_coverage(self) -> float:
        """Fraction of cells on a microscaled (E4M3 or E5M2) precision."""
        a = self.assignments
        return sum(v in _MX for v in a.values()) / len(a) if a else 0.0

    @property
    def coverage_by_precision(self) -> dict:
        a = self.assignments
        counts: dict[str, int] = {}
        for v in a.values():
            counts[v] = counts.get(v, 0) + 1
        return {k: c / len(a) for k, c in sorted(counts.items())} if a else {}

    def precision_for(self, block: int, linear: str) -> str:
        return self.assignments[cell_key(block, linear)]

    def precision_of_module(self, module_name: str) -> str | None:
        return self.assignments.get(cell_of(module_name))

    def to_dict(self) -> dict:
        return {"schema_version": SCHEMA_VERSION, "model_id": self.model_id, "bundle": self.bundle, "tau": self.tau,
                "mx_coverage": self.mx_coverage, "coverage_by_precision": self.coverage_by_precision,
                "assignments": dict(sorted(self.assignments.items())), "metadata": self.metadata or {}}

    @classmethod
    def from_dict(cls, d: dict) -> "PrecisionSchedule":
        if d.get("schema_version") != SCHEMA_VERSION:
            raise ValueError(f"unsupported PrecisionSchedule schema_version: {d.get('schema_version')!r}")
        return cls(model_id=str(d["model_id"]), bundle=str(d["bundle"]), tau=d.get("tau"),
                   assignments=dict(d["assignments"]), metadata=dict(d.get("metadata") or {}))

    def write_json(self, path) -> Path:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(json.dumps(self.to_dict(), indent=2, sort_keys=True) + "\n")
        return path

    @classmethod
    def read_json(cls, path) -> "PrecisionSchedule":
        return cls.from_dict(json.loads(Path(path).read_text(encoding="utf-8")))


# ---------------------------------------------------------------------------- synthesis
def _rows(table) -> list:
    if isinstance(table, dict):
        if "rows" not in table:
            raise ValueError("calibration table dict must contain a 'rows' field")
        return list(table["rows"])
    return list(table)


def _cosines(row: dict) -> tuple:
    """(e4m3 cosine, e5m2 cosine or None): per-format ``metrics`` rows, or a plain ``cosine``."""
    m = row.get("metrics")
    if isinstance(m, dict) and "e4m3" in m:
        e5 = m.get("e5m2")
        return float(m["e4m3"]["cosine"]), (float(e5["cosine"]) if e5 is not None else None)
    return float(row["cosine"]), None


def synthesize_schedule(table, tau: float, *, model_id: str, bundle: str, metadata=None) -> PrecisionSchedule:
    """E4M3 for cells whose calibration cosine is at least tau, bf16 otherwise."""
    a = {cell_key(r["block"], r["linear"]): PRECISION_MXFP8_E4M3 if _cosines(r)[0] >= tau else PRECISION_BF16
         for r in _rows(table)}
    return PrecisionSchedule(model_id, bundle, float(tau), a, metadata)


def synthesize_two_threshold_schedule(table, tau_hi: float, tau_lo: float, *, model_id: str, bundle: str,
                                      metadata=None) -> PrecisionSchedule:
    a = {}
    for r in _rows(table):
        e4, e5 = _cosines(r)
        a[cell_key(r["block"], r["linear"])] = (PRECISION_MXFP8_E4M3 if e4 >= tau_hi else
                                                PRECISION_MXFP8_E5M2 if e5 is not None and e5 >= tau_lo else
                                                PRECISION_BF16)
    meta = dict(metadata or {})
    meta.update(tau_hi=float(tau_hi), tau_lo=float(tau_lo))
    return PrecisionSchedule(model_id, bundle, float(tau_hi), a, meta)


def extreme_schedule(table, precision: str, *, model_id: str, bundle: str, metadata=None) -> PrecisionSchedule:
    p = normalize_precision(precision)
    return PrecisionSchedule(model_id, bundle, None, {cell_key(r["block"], r["linear"]): p for r in _rows(table)},
                             metadata)


def schedule_frontier(table, taus: Iterable[float], *, model_id: str, bundle: str) -> list:
    rows = _rows(table)
    out = [extreme_schedule(rows, PRECISION_BF16, model_id=model_id, bundle=bundle),
           extreme_schedule(rows, PRECISION_MXFP8_E4M3, model_id=model_id, bundle=bundle)]
    return out + [synthesize_schedule(rows, t, model_id=model_id, bundle=bundle) for t in taus]


def two_threshold_frontier(table, tau_pairs, *, model_id: str, bundle: str) -> list:
    rows = _rows(table)
    out = [extreme_schedule(rows, p, model_id=model_id, bundle=bundle)
           for p in (PRECISION_BF16, PRECISION_MXFP8_E4M3, PRECISION_MXFP8_E5M2)]
    return out + [synthesize_two_threshold_schedule(rows, hi, lo, model_id=model_id, bundle=bundle)
                  for hi, lo in tau_pairs]


# ---------------------------------------------------------------------------- B200: calibrate / apply
def _fused_parts(model) -> dict:
    from difflet_b200.quant import apply as qa

    cfg = model.cfg
    if hasattr(cfg, "double_blocks"):
        return qa.mmdit_fused_parts(cfg)
    if "blk.0.v_qkv.w" in model.w:
        return qa.ltx2_fused_parts(cfg)
    if "blk.0.qkv.w" in model.w:
        return qa.wan_fused_parts(cfg)
    raise NotImplementedError(f"no fused-weight map for {type(model).__name__}")


def calibrate(model, *, probe_rows: int = 256, seed: int = 0) -> dict:
    """Calibration table of this engine's quantizer: for every fused weight W, the cosine
    between x W^T and x Q(W)^T (Q = MXFP8 E4M3 quantize + dequantize, 32-value blocks
    along K) on a seeded Gaussian probe x; every diffusers linear the fused weight holds
    gets that cosine (they are quantized together)."""
    import torch

    from difflet_b200.ops import fused as F

    rows = []
    gen = torch.Generator().manual_seed(seed)
    for key, names in _fused_parts(model).items():
        w = model.w[key]
        if isinstance(w, F.MXWeight) or w.shape[1] % 128:
            continue
        x = torch.randn(probe_rows, w.shape[1], generator=gen).to(w.device, torch.float32)
        wq = F.MXWeight.quantize(w).dequantize(torch.float32)
        y, yq = x @ w.float().t(), x @ wq.t()
        cos = float(torch.nn.functional.cosine_similarity(y.reshape(1, -1), yq.reshape(1, -1)).item())
        for n in names:
            blk, lin = cell_of(n).split(":", 1)
            rows.append({"block": int(blk), "linear": lin, "cosine": cos, "fused_weight": key})
    return {"rows": rows, "probe_rows": probe_rows, "seed": seed}


class _ScheduleTargets:
    """The ``matches`` / ``compute`` interface ``quant.apply.apply_to_weights`` reads."""

    def __init__(self, schedule: PrecisionSchedule, compute: str):
        self.schedule, self.compute = schedule, compute

    def matches(self, name: str) -> bool:
        return self.schedule.precision_of_module(name) == PRECISION_MXFP8_E4M3


def apply_schedule(model, schedule: PrecisionSchedule, *, compute: str = "mx") -> dict:
    """Quantize the fused weights whose every linear is scheduled E4M3.  Returns
    ``quantized`` / ``partial`` fused keys and the E5M2 cells (run in bf16 in this build)."""
    from difflet_b200.quant.apply import apply_to_weights

    parts = _fused_parts(model)
    res = apply_to_weights(model.w, parts, _ScheduleTargets(schedule, compute))
    res["e5m2_as_bf16"] = sorted(k for k, v in schedule.assignments.items() if v == PRECISION_MXFP8_E5M2)
    model.precision_schedule = schedule
    return res


__all__ = ["PRECISION_BF16", "PRECISION_MXFP8_E4M3", "PRECISION_MXFP8_E5M2", "PrecisionSchedule", "SCHEMA_VERSION",
           "apply_schedule", "calibrate", "cell_key", "cell_of", "extreme_schedule", "normalize_precision",
           "schedule_frontier", "synthesize_schedule", "synthesize_two_threshold_schedule", "two_threshold_frontier"]
