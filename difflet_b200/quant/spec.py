"""What is quantized and how: the MXFP8 recipe every quantized path shares (torch-free).

Behaviour of difflet/quant/spec.py:46-211: a ``QuantSpec`` names the target linears
(regexes full-matched against diffusers module names, a ``transformer.`` prefix
stripped), the compute path, the TP degree the row-parallel weights were quantized
for, the row-parallel targets and the fused linears stored as two column ranges.
It is JSON-serialisable and enters every cache key (``cache_fields``), so a
different spec is a different artefact and no spec changes no key.

Compute paths on B200: ``mx`` runs the block-scaled tcgen05 GEMM on MXFP8
operands (activations quantized on the fly, ``csrc/mx.cu``); ``dequant`` keeps the
FP8 weights in memory and multiplies in bf16 (memory only).  The reference's
name for the tensor-core path, ``nki``, is accepted as an alias of ``mx``.
"""

from __future__ import annotations

import dataclasses
import hashlib
import json
import re
from pathlib import Path
from typing import Any, Iterable

QUANT_SCHEMA = 1
FORMAT = "mxfp8"
COMPUTE_MODES = ("mx", "dequant")
DEFAULT_COMPUTE = "mx"
BLOCK = 32          # values per E8M0 scale, along K
LAYOUT_K = 128      # K granule of the tensor-core scale layout
STRIPPED_PREFIXES = ("transformer.",)


def strip_prefix(name: str) -> str:
    for p in STRIPPED_PREFIXES:
        if name.startswith(p):
            return name[len(p):]
    return name


def _any_full(patterns, name) -> bool:
    return any(re.fullmatch(p, name) for p in patterns)


@dataclasses.dataclass(frozen=True)
class QuantSpec:
    targets: tuple[str, ...]
    compute: str = DEFAULT_COMPUTE
    tp_degree: int = 1
    row_parallel: tuple[str, ...] = ()
    split_linears: tuple[str, ...] = ()
    schema: int = QUANT_SCHEMA

    def __post_init__(self) -> None:
        if self.compute == "nki":
            object.__setattr__(self, "compute", "mx")
        object.__setattr__(self, "targets", tuple(self.targets))
        object.__setattr__(self, "row_parallel", tuple(self.row_parallel))
        object.__setattr__(self, "split_linears", tuple(self.split_linears))
        if int(self.tp_degree) < 1:
            raise ValueError(f"tp_degree must be >= 1, got {self.tp_degree}")
        if self.compute not in COMPUTE_MODES:
            raise ValueError(f"compute must be one of {COMPUTE_MODES}, got {self.compute!r}")
        if not self.targets or any(not t for t in self.targets):
            raise ValueError("a QuantSpec needs at least one non-empty target pattern")
        for p in (*self.targets, *self.row_parallel, *self.split_linears):
            re.compile(p)

    @property
    def format(self) -> str:
        return FORMAT

    # ------------------------------------------------------------ matching
    def matches(self, name: str) -> bool:
        return _any_full(self.targets, strip_prefix(name))

    def unmatched_targets(self, names: Iterable[str]) -> list[str]:
        bare = [strip_prefix(n) for n in names]
        return [p for p in self.targets if not any(re.fullmatch(p, n) for n in bare)]

    def is_row_parallel(self, name: str) -> bool:
        return _any_full(self.row_parallel, strip_prefix(name))

    def k_shards(self, name: str) -> int:
        return int(self.tp_degree) if self.is_row_parallel(name) else 1

    def is_split(self, name: str) -> bool:
        return _any_full(self.split_linears, strip_prefix(name))

    def unmatched_splits(self, names: Iterable[str]) -> list[str]:
        bare = [strip_prefix(n) for n in names]
        return [p for p in self.split_linears if not any(re.fullmatch(p, n) for n in bare)]

    # ------------------------------------------------------------ serialisation
    def to_dict(self) -> dict[str, Any]:
        body = dataclasses.asdict(self)
        body["targets"] = list(self.targets)
        body["row_parallel"] = list(self.row_parallel)
        if self.split_linears:
            body["split_linears"] = list(self.split_linears)
        else:
            del body["split_linears"]
        body["format"] = FORMAT
        return body

    @classmethod
    def from_dict(cls, body: dict[str, Any]) -> "QuantSpec":
        body = dict(body)
        fmt = body.pop("format", FORMAT)
        if fmt != FORMAT:
            raise ValueError(f"quant format must be {FORMAT!r}, got {fmt!r}")
        return cls(targets=tuple(body["targets"]), compute=body.get("compute", DEFAULT_COMPUTE),
                   tp_degree=int(body.get("tp_degree", 1)), row_parallel=tuple(body.get("row_parallel", ())),
                   split_linears=tuple(body.get("split_linears", ())), schema=int(body.get("schema", QUANT_SCHEMA)))

    def targets_sha256(self) -> str:
        return hashlib.sha256(json.dumps(list(self.targets)).encode()).hexdigest()[:16]

    def cache_fields(self) -> dict[str, Any]:
        return {"quant": FORMAT, "quant_schema": self.schema, "quant_compute": self.compute,
                "quant_targets_sha256": self.targets_sha256(), "quant_tp_degree": int(self.tp_degree)}

    def weights_identity(self) -> dict[str, Any]:
        ident = {"quant": FORMAT, "quant_schema": self.schema, "quant_targets": list(self.targets),
                 "quant_row_parallel": list(self.row_parallel), "quant_tp_degree": int(self.tp_degree)}
        if self.split_linears:
            ident["quant_split_linears"] = list(self.split_linears)
        return ident


def quant_cache_fields(spec: QuantSpec | None) -> dict[str, Any]:
    return {} if spec is None else spec.cache_fields()


def file_sha256(path: str | Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


__all__ = ["BLOCK", "COMPUTE_MODES", "DEFAULT_COMPUTE", "FORMAT", "LAYOUT_K", "QUANT_SCHEMA", "QuantSpec",
           "file_sha256", "quant_cache_fields", "strip_prefix"]
