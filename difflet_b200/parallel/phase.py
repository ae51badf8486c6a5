"""Status-synced host phases: every rank leaves a fallible host step together.

Behaviour of the reference's neuron runtime (difflet/backends/neuron/core/distributed.py:68-117):
one process per device issues the same collectives in the same order, so a rank that raises
before a collective would leave its peers blocked in it until the process-group timeout.
Fallible, collective-free host work (a checkpoint read, an HBM fit check, input parsing, an
output write on rank 0) therefore runs inside ``collective_phase``, which ends with one int32
all-reduce(MAX) of a status code: every rank raises when any rank failed (the failing rank its
own error, the others ``RankFailureError`` naming it).  A phase body must not issue collectives
(a failing rank's status all-reduce would pair with its peers' body collective), so a model
forward never runs inside one: a rank failing mid-forward exits and the launcher tears the
others down (the device-side waits are bounded, so they return an error instead of hanging).
"""

from __future__ import annotations

from contextlib import contextmanager
from typing import Any, Callable, Iterator, TypeVar

import torch
import torch.distributed as dist

T = TypeVar("T")


class RankFailureError(RuntimeError):
    """Another rank failed in a collective phase; this rank stops at the same point."""


def world_info() -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def _status_device(device=None) -> torch.device:
    if device is not None:
        return torch.device(device)
    if dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def sync_status(ok: bool, *, what: str, device=None) -> None:
    """All-reduce(MAX) of 0 (ok) / rank + 1 (failed); healthy ranks raise when any failed."""
    rank, world = world_info()
    if world == 1:
        return
    flag = torch.tensor([0 if ok else rank + 1], dtype=torch.int32, device=_status_device(device))
    dist.all_reduce(flag, op=dist.ReduceOp.MAX)
    failed = int(flag.cpu()[0])
    if ok and failed:
        raise RankFailureError(f"{what}: failed on rank {failed - 1}; rank {rank} stops too")


@contextmanager
def collective_phase(what: str, *, device=None) -> Iterator[None]:
    """Run a collective-free body, then agree on its outcome (exactly one all-reduce on every
    exit path, including a nested phase's ``RankFailureError``)."""
    try:
        yield
    except Exception:
        sync_status(False, what=what, device=device)
        raise
    sync_status(True, what=what, device=device)


def rank0_call(fn: Callable[..., T], *args: Any, what: str, device=None, **kwargs: Any) -> T | None:
    """``fn(*args, **kwargs)`` on rank 0 inside a phase; None on the other ranks."""
    rank, _ = world_info()
    with collective_phase(what, device=device):
        return fn(*args, **kwargs) if rank == 0 else None


def broadcast_object(obj: Any, *, src: int = 0, device=None) -> Any:
    """A picklable host object from rank ``src`` to every rank (identity on one rank)."""
    rank, world = world_info()
    if world == 1:
        return obj
    box = [obj if rank == src else None]
    dist.broadcast_object_list(box, src=src, device=_status_device(device))
    return box[0]


__all__ = ["RankFailureError", "broadcast_object", "collective_phase", "rank0_call", "sync_status", "world_info"]
