"""The offline MXFP8 checkpoint: a diffusers-layout directory with FP8 target weights.

Layout (the reference's, difflet/quant/checkpoint.py:1-60, so quantized directories
carry over): ``<cache>/quantized/<source label>/<component>/mxfp8-<digest>/`` holds
``diffusion_pytorch_model-0000i-of-0000n.safetensors`` + ``.index.json`` with every
tensor of the source; a target ``<prefix>.weight`` is stored as ``float8_e4m3fn``
``[N, K]`` with its uint8 E8M0 scales ``<prefix>.weight_scale`` ``[N, K/32]``; a
linear the spec splits (the single-stream ``proj_out`` over ``cat([attn, mlp])``)
is stored as ``<prefix>_attn.weight`` (input columns ``[0, N)``) and
``<prefix>_mlp.weight`` (the rest), each a target of its own; everything else is
copied.  ``config.json`` is copied and ``difflet_quant.json`` records the spec, the
source fingerprint and the tensor counts; ``check_quantized_dir`` refuses a
directory whose manifest does not match.

Block membership is OCP's (32 consecutive K values), so a row-parallel weight
quantized whole equals the concatenation of its per-rank K ranges whenever a
rank's range is a multiple of 32; the writer checks the stricter tensor-core
granule (K / tp a multiple of 128) for row-parallel targets and refuses otherwise.
"""

from __future__ import annotations

import hashlib
import json
import os
import shutil
import time
from pathlib import Path
from typing import Any, Iterator

import torch

from difflet_b200.quant.spec import LAYOUT_K, QuantSpec, strip_prefix

MANIFEST = "difflet_quant.json"
SHARD_BYTES = 4 * 1024 ** 3
_SHARD = "diffusion_pytorch_model-{i:05d}-of-{n:05d}.safetensors"
_INDEX = "diffusion_pytorch_model.safetensors.index.json"


def is_fp8(t: torch.Tensor) -> bool:
    return t.dtype in (torch.float8_e4m3fn, torch.float8_e5m2)


def source_fingerprint(model_dir: str | Path) -> list[list[Any]]:
    """Names, sizes and resolved blob names of the safetensors files, sha256 of index files."""
    d = Path(model_dir)
    out = []
    for f in sorted(d.glob("*.safetensors")):
        out.append([f.name, f.stat().st_size, os.path.basename(os.path.realpath(f))])
    for f in sorted(d.glob("*.index.json")):
        out.append([f.name, hashlib.sha256(f.read_bytes()).hexdigest()])
    return out


def quantized_digest(spec: QuantSpec, fingerprint) -> str:
    body = json.dumps({"spec": spec.weights_identity(), "source": fingerprint}, sort_keys=True)
    return hashlib.sha256(body.encode()).hexdigest()[:16]


def quantized_dir(cache_root: str | Path, model_dir: str | Path, spec: QuantSpec) -> Path:
    md = Path(model_dir)
    label = "".join(c if c.isalnum() or c in "._-" else "_" for c in f"{md.parent.name}--{md.name}")
    return Path(cache_root) / "quantized" / label / f"mxfp8-{quantized_digest(spec, source_fingerprint(md))}"


def _iter_source(sd_or_dir) -> Iterator[tuple[str, torch.Tensor]]:
    if isinstance(sd_or_dir, dict):
        yield from sd_or_dir.items()
        return
    from safetensors import safe_open

    from difflet_b200.utils.checkpoint import component_files

    d = Path(sd_or_dir)
    for f in component_files(str(d.parent), d.name):
        with safe_open(str(f), framework="pt", device="cpu") as h:
            for k in h.keys():
                yield k, h.get_tensor(k)


def _shapes(sd_or_dir) -> dict[str, tuple]:
    if isinstance(sd_or_dir, dict):
        return {k: tuple(v.shape) for k, v in sd_or_dir.items()}
    from safetensors import safe_open

    from difflet_b200.utils.checkpoint import component_files

    d = Path(sd_or_dir)
    out = {}
    for f in component_files(str(d.parent), d.name):
        with safe_open(str(f), framework="pt", device="cpu") as h:
            for k in h.keys():
                out[k] = tuple(h.get_slice(k).get_shape())
    return out


def _weight_prefixes(shapes) -> list[str]:
    return [k[: -len(".weight")] for k, s in shapes.items() if k.endswith(".weight") and len(s) == 2]


def _split_names(prefix: str) -> tuple[str, str]:
    return prefix + "_attn", prefix + "_mlp"


def plan(sd_or_dir, spec: QuantSpec) -> dict[str, Any]:
    """Which linears the spec quantizes / splits; refuses dead patterns and bad K granules."""
    shapes = _shapes(sd_or_dir)
    prefixes = _weight_prefixes(shapes)
    splits = [p for p in prefixes if spec.is_split(p)]
    dead_splits = spec.unmatched_splits(prefixes)
    if dead_splits:
        raise ValueError(f"split patterns match no linear: {dead_splits}")
    k_of = {p: shapes[p + ".weight"][1] for p in prefixes if p not in splits}
    for p in splits:
        N, Kfull = shapes[p + ".weight"]
        a, m = _split_names(p)
        k_of[a], k_of[m] = N, Kfull - N
    names = list(k_of)
    fused_targets = [p for p in splits if spec.matches(p)]
    if fused_targets:
        raise ValueError(f"targets name the fused split linears {fused_targets}; name their _attn / _mlp halves")
    dead = spec.unmatched_targets(names)
    if dead:
        raise ValueError(f"target patterns match no linear (a split linear counts as its _attn / _mlp "
                         f"halves): {dead}")
    targets = [n for n in names if spec.matches(n)]
    for n in targets:
        shards = spec.k_shards(n)
        if k_of[n] % (LAYOUT_K * shards):
            raise ValueError(f"{n}: K {k_of[n]} over {shards} row-parallel rank(s) is not a multiple of {LAYOUT_K}")
    return {"targets": targets, "splits": splits}


def quantize_tensors(sd_or_dir, spec: QuantSpec) -> Iterator[tuple[str, torch.Tensor]]:
    from difflet_b200.ops.mx import quantize_mx

    p = plan(sd_or_dir, spec)
    targets, splits = set(p["targets"]), set(p["splits"])

    def emit(name, w):
        if name in targets:
            q, s = quantize_mx(w.to(torch.bfloat16))
            yield name + ".weight", q
            yield name + ".weight_scale", s
        else:
            yield name + ".weight", w

    for k, t in _iter_source(sd_or_dir):
        if k.endswith(".weight") and k[:-7] in splits:
            base = k[:-7]
            N = t.shape[0]
            a, m = _split_names(base)
            yield from emit(a, t[:, :N].contiguous())
            yield from emit(m, t[:, N:].contiguous())
        elif k.endswith(".weight") and t.dim() == 2:
            yield from emit(k[:-7], t)
        else:
            yield k, t


def write_quantized_dir(sd_or_dir, out_dir: str | Path, spec: QuantSpec, *, config: dict | None = None) -> Path:
    """Write the quantized directory (atomically: a temporary sibling renamed at the end)."""
    from safetensors.torch import save_file

    out = Path(out_dir)
    if out.is_symlink() or (out.exists() and not out.is_dir()):
        raise ValueError(f"{out} exists and is not a directory this writer may replace")
    if out.is_dir() and any(out.iterdir()) and not (out / MANIFEST).is_file():
        # only an earlier quantized checkpoint (or an empty directory) is replaced
        raise ValueError(f"{out} holds files that are not a quantized checkpoint; choose another --out")
    tmp = out.parent / f".{out.name}.tmp{os.getpid()}"
    if tmp.exists():
        shutil.rmtree(tmp)
    tmp.mkdir(parents=True)
    shards, cur, size, counts = [], {}, 0, {"fp8": 0, "copied": 0}
    for k, t in quantize_tensors(sd_or_dir, spec):
        if is_fp8(t):
            counts["fp8"] += 1
        elif not k.endswith(".weight_scale"):
            counts["copied"] += 1
        nb = t.numel() * t.element_size()
        if cur and size + nb > SHARD_BYTES:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = t.contiguous()
        size += nb
    if cur:
        shards.append(cur)
    weight_map = {}
    for i, sh in enumerate(shards, 1):
        name = _SHARD.format(i=i, n=len(shards))
        save_file(sh, str(tmp / name))
        weight_map.update({k: name for k in sh})
    (tmp / _INDEX).write_text(json.dumps({"metadata": {}, "weight_map": weight_map}, indent=1))
    if not isinstance(sd_or_dir, dict):
        src = Path(sd_or_dir)
        for f in src.iterdir():
            if f.is_file() and not f.name.endswith((".safetensors", ".index.json")) and f.name != MANIFEST:
                shutil.copy2(f, tmp / f.name)
    if config is not None:
        (tmp / "config.json").write_text(json.dumps(config, indent=2))
    fp = source_fingerprint(sd_or_dir) if not isinstance(sd_or_dir, dict) else []
    manifest = {"format": "mxfp8", "spec": spec.to_dict(), "source": fp, "counts": counts,
                "digest": quantized_digest(spec, fp), "created": time.time()}
    (tmp / MANIFEST).write_text(json.dumps(manifest, indent=2))
    if out.exists():
        shutil.rmtree(out)
    tmp.rename(out)
    return out


def read_manifest(quantized: str | Path) -> dict[str, Any]:
    return json.loads((Path(quantized) / MANIFEST).read_text())


def check_quantized_dir(quantized: str | Path, model_dir: str | Path | None, spec: QuantSpec) -> None:
    m = read_manifest(quantized)
    got = QuantSpec.from_dict(m["spec"])
    if got.weights_identity() != spec.weights_identity():
        raise ValueError(f"{quantized} was quantized with another spec: {got.weights_identity()} != "
                         f"{spec.weights_identity()}")
    if model_dir is not None and m.get("source") and m["source"] != source_fingerprint(model_dir):
        raise ValueError(f"{quantized} was quantized from another checkpoint than {model_dir}")


def ensure_quantized_dir(cache_root, model_dir, spec: QuantSpec, *, create: bool = True) -> Path:
    out = quantized_dir(cache_root, model_dir, spec)
    if (out / MANIFEST).exists():
        check_quantized_dir(out, model_dir, spec)
        return out
    if not create:
        raise FileNotFoundError(f"no quantized checkpoint at {out} (run `difflet compile` with --quant mxfp8)")
    return write_quantized_dir(model_dir, out, spec)


def quantized_linear_names(quantized: str | Path) -> list[str]:
    idx = json.loads((Path(quantized) / _INDEX).read_text())["weight_map"]
    return sorted(k[: -len(".weight_scale")] for k in idx if k.endswith(".weight_scale"))


def load_quantized(quantized: str | Path, device="cpu") -> dict[str, torch.Tensor]:
    """The quantized directory's tensors (FP8 weights, uint8 scales, everything else as stored)."""
    from safetensors import safe_open

    d = Path(quantized)
    idx = json.loads((d / _INDEX).read_text())["weight_map"]
    out = {}
    for f in sorted(set(idx.values())):
        with safe_open(str(d / f), framework="pt", device="cpu") as h:
            for k in h.keys():
                out[strip_prefix(k)] = h.get_tensor(k).to(device)
    return out


__all__ = ["MANIFEST", "check_quantized_dir", "ensure_quantized_dir", "is_fp8", "load_quantized", "plan",
           "quantize_tensors", "quantized_digest", "quantized_dir", "quantized_linear_names", "read_manifest",
           "source_fingerprint", "write_quantized_dir"]
