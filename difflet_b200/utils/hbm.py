"""HBM fit check before any weight is materialised.

Behaviour of the reference's budget check (difflet/backends/neuron/hbm.py:1-58): a rank whose
weights cannot fit fails in seconds with a message saying what would fit, instead of deep
inside the load.  On B200 the budget is ``FIT_FRACTION`` of the device's free memory (another
process may hold part of the 180 GB), the estimate is the model's weight bytes (materialised
whole before tensor-parallel sharding) plus a per-token activation allowance, and the message
says whether the weights alone fit.  The check runs inside a status-synced phase so every rank
stops together.
"""

from __future__ import annotations

import math

import torch

GIB = 1024**3
FIT_FRACTION = 0.92


class HbmBudgetError(ValueError):
    """The model does not fit in this device's free HBM."""


def weight_bytes(shapes: dict, dtype: torch.dtype) -> int:
    elem = torch.empty((), dtype=dtype).element_size()
    return sum(math.prod(s) for s in shapes.values()) * elem


def free_bytes(device) -> int:
    free, _ = torch.cuda.mem_get_info(device)
    return int(free)


def check_fit(need_bytes: int, device, *, what: str, free: int | None = None, tp: int = 1,
              weights: int | None = None) -> None:
    """Raise ``HbmBudgetError`` when ``need_bytes`` exceed ``FIT_FRACTION`` of the free HBM."""
    dev = torch.device(device)
    if dev.type != "cuda":
        return
    avail = free if free is not None else free_bytes(dev)
    budget = FIT_FRACTION * avail
    if need_bytes <= budget:
        return
    hint = ""
    if weights and weights <= budget:
        hint = "; the weights fit, so fewer tokens per rank (more context-parallel ranks) would"
    raise HbmBudgetError(f"{what}: needs {need_bytes / GIB:.1f} GiB but {avail / GIB:.1f} GiB are free on {dev} "
                         f"(budget {FIT_FRACTION:.0%}){hint}")


def check_model_fit(shapes: dict, dtype: torch.dtype, device, *, what: str, tokens: int = 0, hidden: int = 0,
                    tp: int = 1, free: int | None = None) -> int:
    """Weights (whole, as loaded) + about 48 bytes per token and hidden unit of activations
    (residual, norm, q/k/v, MLP and workspaces in bf16).  Returns the estimate in bytes."""
    w = weight_bytes(shapes, dtype)
    need = w + 48 * tokens * hidden
    check_fit(need, device, what=what, free=free, tp=tp, weights=w)
    return need


__all__ = ["FIT_FRACTION", "GIB", "HbmBudgetError", "check_fit", "check_model_fit", "free_bytes", "preload_check",
           "weight_bytes"]


def preload_check(shapes: dict, dtype: torch.dtype, device, *, what: str, copies: int = 1, tokens: int = 0,
                  hidden: int = 0) -> None:
    """The engines' pre-load check: ``copies`` models of ``shapes`` (Wan's two experts) on
    ``device``, every rank agreeing on the outcome (a status-synced phase)."""
    from difflet_b200.parallel.phase import collective_phase

    with collective_phase(f"HBM fit check ({what})"):
        if torch.device(device).type == "cuda":
            w = weight_bytes(shapes, dtype) * copies
            check_fit(w + 48 * tokens * hidden, device, what=what, weights=w)
