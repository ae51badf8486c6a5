"""Provenance of a bench result (reference: difflet/bench/provenance.py:79-147): the source
revision, the package versions, the DIFFLET_* environment, the GPU and driver, and the peak
device memory of the run, attached to every result line so numbers stay traceable."""

from __future__ import annotations

import os
import platform
import subprocess
from pathlib import Path


def git_revision(root: Path | None = None) -> dict:
    root = root or Path(__file__).resolve().parents[2]
    out = {}
    for key, args in (("sha", ["rev-parse", "HEAD"]), ("dirty", ["status", "--porcelain", "--untracked-files=no"])):
        try:
            r = subprocess.run(["git", "-C", str(root), *args], capture_output=True, text=True, timeout=10)
            v = r.stdout.strip()
            out[key] = bool(v) if key == "dirty" else (v or None)
        except Exception:  # noqa: BLE001 - a tarball without .git
            out[key] = None
    return out


def packages() -> dict:
    import torch

    d = {"python": platform.python_version(), "torch": torch.__version__, "cuda": torch.version.cuda}
    try:
        d["nccl"] = ".".join(str(x) for x in torch.cuda.nccl.version())
    except Exception:  # noqa: BLE001
        d["nccl"] = None
    return d


def device() -> dict:
    import torch

    if not torch.cuda.is_available():
        return {"gpu": None}
    p = torch.cuda.get_device_properties(torch.cuda.current_device())
    d = {"gpu": p.name, "sms": p.multi_processor_count, "hbm_gb": round(p.total_memory / 1e9, 1),
         "capability": f"{p.major}.{p.minor}"}
    try:
        import pynvml

        pynvml.nvmlInit()
        d["driver"] = pynvml.nvmlSystemGetDriverVersion()
    except Exception:  # noqa: BLE001
        d["driver"] = None
    return d


def memory() -> dict:
    import torch

    if not torch.cuda.is_available():
        return {}
    return {"max_allocated_gb": round(torch.cuda.max_memory_allocated() / 1e9, 2),
            "max_reserved_gb": round(torch.cuda.max_memory_reserved() / 1e9, 2)}


def collect() -> dict:
    return {"git": git_revision(), "packages": packages(), "device": device(),
            "env": {k: v for k, v in sorted(os.environ.items()) if k.startswith("DIFFLET_")}, "host": platform.node()}


__all__ = ["collect", "device", "git_revision", "memory", "packages"]
