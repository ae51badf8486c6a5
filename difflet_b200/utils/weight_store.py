"""Pre-sharded weight store: this rank's converted, sharded (and quantized) weights, written by
the first load and read straight back by later ones.

Behaviour of the reference's store (difflet/backends/neuron/core/weight_store.py:1-60): without
it every launch reads the diffusers safetensors, converts them to the engine layout (here: the
fused q|k|v / [q|mlp|k|v] matrices, the modulation stack) and shards them for its tensor-
parallel rank.  With ``DIFFLET_WEIGHT_STORE`` set to a directory, the first load saves exactly
the tensors the engine keeps on the device, per tensor-parallel rank, and later loads of the
same checkpoint / layout read those bytes instead.

Layout: ``<store>/<label>__<digest>/tp<r>-of-<n>.safetensors`` plus ``<file>.manifest.json``
(format, digest, tensors with dtype and shape, byte size, sha256 of the safetensors header).
The digest hashes the store format, the checkpoint's content fingerprint (name, size, mtime of
every ``*.safetensors`` / index file), the load dtype, the tp degree and the caller's layout
fields (preset, quantization spec), so any change of those is another entry.  A manifest that
does not match the file (a partial write) makes the entry a miss; files are written to a
temporary name and renamed, so readers never see half a file.  MXFP8 weights (``MXWeight``) are
stored as their FP8 data and scales (``<name>.__mxq`` / ``<name>.__mxsf``).
"""

from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path
from typing import Callable

import torch

FORMAT = 1
_OFF = {"", "0", "off", "false", "none"}


def store_root() -> Path | None:
    from difflet_b200 import envs

    v = envs.DIFFLET_WEIGHT_STORE
    return None if v is None or str(v).strip().lower() in _OFF else Path(v)


def checkpoint_fingerprint(path) -> list:
    """(relative name, size, mtime) of every safetensors / index file under ``path``."""
    if path is None:
        return []
    root = Path(path)
    out = []
    for p in sorted(root.rglob("*")):
        if p.is_file() and (p.suffix == ".safetensors" or p.name.endswith(".index.json")):
            st = p.stat()
            out.append((str(p.relative_to(root)), st.st_size, int(st.st_mtime)))
    return out


def entry_dir(label: str, model_path, dtype: torch.dtype, tp: int, layout: dict) -> Path | None:
    root = store_root()
    if root is None:
        return None
    blob = json.dumps({"format": FORMAT, "ckpt": checkpoint_fingerprint(model_path), "dtype": str(dtype), "tp": tp,
                       "layout": layout}, sort_keys=True, default=str)
    digest = hashlib.sha256(blob.encode()).hexdigest()[:16]
    return root / f"{label}__{digest}"


def _flatten(w: dict) -> dict:
    from difflet_b200.ops.fused import MXWeight

    out = {}
    for k, t in w.items():
        if isinstance(t, MXWeight):
            out[k + ".__mxq"] = t.q.contiguous()
            out[k + ".__mxsf"] = t.sf.contiguous()
        else:
            out[k] = t.contiguous()
    return out


def _unflatten(flat: dict, compute: str) -> dict:
    from difflet_b200.ops.fused import MXWeight

    out = {}
    for k, t in flat.items():
        if k.endswith(".__mxq"):
            base = k[: -len(".__mxq")]
            out[base] = MXWeight(t, flat[base + ".__mxsf"], compute)
        elif not k.endswith(".__mxsf"):
            out[k] = t
    return out


def _header_sha(path: Path) -> str:
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        return hashlib.sha256(f.read(n)).hexdigest()


def save(entry: Path, rank: int, tp: int, w: dict) -> Path:
    from safetensors.torch import save_file

    entry.mkdir(parents=True, exist_ok=True)
    flat = {k: v.detach().to("cpu") for k, v in _flatten(w).items()}
    final = entry / f"tp{rank}-of-{tp}.safetensors"
    tmp = final.with_suffix(f".tmp{os.getpid()}")
    save_file(flat, str(tmp))
    os.replace(tmp, final)
    man = {"format": FORMAT, "entry": entry.name, "bytes": final.stat().st_size, "header_sha256": _header_sha(final),
           "tensors": [[k, str(v.dtype), list(v.shape)] for k, v in flat.items()]}
    mtmp = final.with_suffix(f".mtmp{os.getpid()}")
    mtmp.write_text(json.dumps(man, indent=1))
    os.replace(mtmp, Path(str(final) + ".manifest.json"))
    return final


def load(entry: Path, rank: int, tp: int, device, compute: str = "mx") -> dict | None:
    """This rank's tensors, or None on a miss (absent file or a manifest that does not match)."""
    from safetensors.torch import load_file

    f = entry / f"tp{rank}-of-{tp}.safetensors"
    mf = Path(str(f) + ".manifest.json")
    if not f.exists() or not mf.exists():
        return None
    try:
        man = json.loads(mf.read_text())
        if man.get("format") != FORMAT or man.get("bytes") != f.stat().st_size or \
                man.get("header_sha256") != _header_sha(f):
            return None
        flat = load_file(str(f), device=str(device))
    except Exception:  # noqa: BLE001 - a damaged entry is a miss, the checkpoint is still there
        return None
    return _unflatten(flat, compute)


def load_or_build(label: str, model_path, dtype: torch.dtype, tp: int, rank: int, layout: dict, device,
                  build: Callable[[], dict], compute: str = "mx") -> tuple[dict, str]:
    """(weights, "hit" | "miss" | "off"): the stored shard, or ``build()`` (saved on a miss)."""
    entry = entry_dir(label, model_path, dtype, tp, layout)
    if entry is None:
        return build(), "off"
    w = load(entry, rank, tp, device, compute)
    if w is not None:
        return w, "hit"
    w = build()
    save(entry, rank, tp, w)
    return w, "miss"


__all__ = ["FORMAT", "checkpoint_fingerprint", "entry_dir", "load", "load_or_build", "save", "store_root"]
