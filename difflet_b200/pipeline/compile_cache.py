"""Content-addressed artefact cache: ``<root>/<model>/<sha256[:16]>/manifest.json``.

Same scheme as the reference (``difflet/pipeline/compile_cache.py:39-327``):
the key hashes only what changes the built artefact -- model id / name /
revision, the parallel config's cache dict, dtype, the canonical shape set,
application kwargs minus runtime-only ones, and toolchain versions -- while the
resolved local path and similar details are recorded unhashed.  On B200 the
toolchain part includes the native-kernel source hash, the CUDA / NCCL
versions and the GPU SKU, and the manifest also stores kernel tuning results
(e.g. chosen GEMM tiles per shape) written by ``compile()``.
"""

from __future__ import annotations

import hashlib
import json
import os
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

from difflet_b200 import envs
from difflet_b200.pipeline.parallel_config import CandidateConfig, DiffletParallelConfig

MANIFEST_FILENAME = "manifest.json"
MANIFEST_SCHEMA_VERSION = 1

# kwargs that only affect a run, never the built artefact
RUNTIME_ONLY_APP_KWARGS = frozenset({
    "prompt", "negative_prompt", "seed", "num_inference_steps", "guidance_scale", "true_cfg_scale",
    "output", "output_type", "teacache_speedup", "teacache_calibration", "teacache_calibration_path",
    "teacache_cadence", "teacache_online_delta", "requests", "random_init",
})


def normalize_dtype(dtype: Any) -> str:
    s = str(dtype)
    s = s.replace("torch.", "")
    aliases = {"bf16": "bfloat16", "fp16": "float16", "half": "float16", "fp32": "float32", "float": "float32"}
    return aliases.get(s, s)


def _normalize(v: Any) -> Any:
    if isinstance(v, dict):
        return {str(k): _normalize(v[k]) for k in sorted(v, key=str)}
    if isinstance(v, (list, tuple)):
        return [_normalize(x) for x in v]
    if isinstance(v, (str, int, float, bool)) or v is None:
        return v
    return str(v)


def canonicalize_shapes(shapes) -> list[tuple]:
    out = []
    for s in shapes:
        t = tuple(s) + (None,) * (3 - len(tuple(s)))
        if t not in out:
            out.append(t)
    out.sort(key=lambda t: tuple(-(x or 0) for x in t))
    return out


def toolchain_versions(backend: str | None) -> dict[str, str]:
    try:
        from difflet_b200.platforms import get_platform

        return get_platform(backend).toolchain_versions()
    except Exception:
        return {}


@dataclass(frozen=True)
class CacheSpec:
    model_id: str
    model_path: str
    model_name: str
    parallel: DiffletParallelConfig
    dtype: Any
    height: int | None = None
    width: int | None = None
    num_frames: int | None = None
    revision: str | None = None
    application_kwargs: dict | None = None
    shapes: tuple | None = None
    backend: str | None = None
    candidate: CandidateConfig | None = None
    toolchain: dict = field(default=None)

    def canonical_shapes(self):
        if self.shapes:
            return [list(s) for s in canonicalize_shapes(self.shapes)]
        return [[self.height, self.width, self.num_frames]]

    def cache_inputs(self) -> dict[str, Any]:
        d = {
            "schema": MANIFEST_SCHEMA_VERSION,
            "model_id": self.model_id,
            "model_name": self.model_name,
            "revision": self.revision,
            "parallel": self.parallel.to_cache_dict(),
            "dtype": normalize_dtype(self.dtype),
            "shapes": self.canonical_shapes(),
            "application_kwargs": _normalize({k: v for k, v in (self.application_kwargs or {}).items()
                                              if k not in RUNTIME_ONLY_APP_KWARGS}),
            "backend": self.backend,
            "toolchain": self.toolchain if self.toolchain is not None else toolchain_versions(self.backend),
        }
        if self.candidate is not None and not self.candidate.is_trivial:
            d["candidate"] = self.candidate.to_cache_dict()
        if (self.application_kwargs or {}).get("quant"):
            from difflet_b200.quant.apply import spec_from_kwargs

            d.update(spec_from_kwargs(self.model_name, self.application_kwargs).cache_fields())
        return d

    def manifest_metadata(self) -> dict[str, Any]:
        return {"model_path": self.model_path}


def cache_key(spec: CacheSpec) -> str:
    blob = json.dumps(spec.cache_inputs(), sort_keys=True, separators=(",", ":"))
    return hashlib.sha256(blob.encode()).hexdigest()[:16]


def cache_path(root: str | None, spec: CacheSpec) -> Path:
    base = Path(root or envs.DIFFLET_COMPILE_CACHE).expanduser()
    return base / spec.model_name / cache_key(spec)


def read_manifest(path: Path) -> dict | None:
    p = Path(path) / MANIFEST_FILENAME
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text())
    except (OSError, json.JSONDecodeError):
        return None


def has_valid_manifest(path: Path, spec: CacheSpec) -> bool:
    m = read_manifest(path)
    return bool(m) and m.get("key") == cache_key(spec) and m.get("inputs") == _normalize(spec.cache_inputs())


def write_manifest(path: Path, spec: CacheSpec, extra: dict | None = None) -> Path:
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    doc = {"key": cache_key(spec), "inputs": _normalize(spec.cache_inputs()),
           "metadata": spec.manifest_metadata(), **(extra or {})}
    tmp = path / f"{MANIFEST_FILENAME}.{os.getpid()}.tmp"  # unique per writer; rename is atomic
    tmp.write_text(json.dumps(doc, indent=2, sort_keys=True))
    os.replace(tmp, path / MANIFEST_FILENAME)
    return path / MANIFEST_FILENAME
