"""Safetensors loading for diffusers-layout component directories.

Reads ``<model>/<component>/diffusion_pytorch_model*.safetensors`` (sharded via
``*.safetensors.index.json`` or a single file) lazily with the safetensors
slice API, so a rank can read only the rows it owns (reference lazy sharded
loader, ``difflet/backends/_torch_megatron/checkpoint.py:34-195``).
"""

from __future__ import annotations

import json
from pathlib import Path

import torch


def component_files(model_path: str, component: str) -> list[Path]:
    d = Path(model_path) / component
    idx = sorted(d.glob("*.safetensors.index.json"))
    if idx:
        m = json.loads(idx[0].read_text())["weight_map"]
        return sorted({d / f for f in m.values()})
    files = sorted(d.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no safetensors under {d}")
    return files


def load_component(model_path: str, component: str, *, dtype=None, device="cpu", keys=None,
                   row_slices: dict | None = None) -> dict[str, torch.Tensor]:
    """Load a component's state dict.  ``row_slices[name] = (start, stop)`` reads only
    those rows of a tensor (tensor-parallel shards)."""
    from safetensors import safe_open

    out = {}
    for f in component_files(model_path, component):
        with safe_open(str(f), framework="pt", device="cpu") as h:
            for k in h.keys():
                if keys is not None and k not in keys:
                    continue
                if row_slices and k in row_slices:
                    a, b = row_slices[k]
                    t = h.get_slice(k)[a:b]
                else:
                    t = h.get_tensor(k)
                if dtype is not None and t.is_floating_point() and t.element_size() > 1:  # FP8 stays FP8
                    t = t.to(dtype)
                out[k] = t.to(device)
    return out


def save_component(sd: dict[str, torch.Tensor], model_path: str, component: str, config: dict | None = None):
    from safetensors.torch import save_file

    d = Path(model_path) / component
    d.mkdir(parents=True, exist_ok=True)
    save_file({k: v.contiguous().cpu() for k, v in sd.items()}, str(d / "diffusion_pytorch_model.safetensors"))
    if config is not None:
        (d / "config.json").write_text(json.dumps(config, indent=2))
