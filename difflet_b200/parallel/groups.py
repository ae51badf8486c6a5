"""Process-group bootstrap and per-axis groups of the {dp, cfg, cp, tp} mesh.

NCCL (GPU) or gloo (CPU tests) through ``torch.distributed``, env rendezvous
under torchrun (reference ``difflet/platforms/gpu.py:87-97`` and
``difflet/backends/cuda/ops_impl/parallel_mesh.py:80-118``).  Every rank
creates every group in the same order (a torch.distributed requirement).
"""

from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist

from difflet_b200 import envs
from difflet_b200.parallel.mesh import AXES, MeshSpec

_GROUPS: dict = {}
_MESH: MeshSpec | None = None


def init_distributed(backend: str | None = None, timeout_s: int | None = None) -> None:
    if dist.is_initialized():
        return
    backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29500")
    kw = {}
    if backend == "nccl":
        kw["device_id"] = torch.device("cuda", envs.LOCAL_RANK % max(1, torch.cuda.device_count()))
    dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s or envs.DIFFLET_PG_TIMEOUT_S), **kw)


def world_size() -> int:
    return dist.get_world_size() if dist.is_initialized() else 1


def rank() -> int:
    return dist.get_rank() if dist.is_initialized() else 0


def init_mesh(mesh: MeshSpec):
    """Create one group per axis coordinate slice; returns {axis: (group, ranks)} for this rank."""
    global _MESH
    _MESH = mesh
    _GROUPS.clear()
    me = rank()
    for axis in AXES:
        for ranks in mesh.axis_groups(axis):
            if len(ranks) == 1:
                if me in ranks:
                    _GROUPS[axis] = (None, ranks)
                continue
            g = dist.new_group(ranks)
            if me in ranks:
                _GROUPS[axis] = (g, ranks)
    return dict(_GROUPS)


def get_group(axis: str):
    return _GROUPS.get(axis, (None, [rank()]))[0]


def get_group_ranks(axis: str) -> list[int]:
    return _GROUPS.get(axis, (None, [rank()]))[1]


def mesh() -> MeshSpec | None:
    return _MESH
