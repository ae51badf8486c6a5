"""Bring the GPU runtime up on a background thread while the host loads weights.

Reference behaviour (``difflet/cli/prewarm.py:29-80``): the first device operation of a process
pays the runtime's start-up, serially in front of the first weight upload; firing it early on a
daemon thread overlaps it with host-side loading.  Best effort: every failure is swallowed, and
``DIFFLET_DISABLE_PREWARM`` (non-empty) turns it off.

On B200 the start-up is the CUDA context of each local GPU (driver initialisation, context and
memory-pool creation), loading this engine's kernel module onto the device, and the cuBLAS
handle a library GEMM would create on first use.
"""

from __future__ import annotations

import os
import threading


def prewarm_cuda(devices: list[int] | None = None) -> threading.Thread | None:
    """Start the warm-up thread (None when disabled or there is no GPU)."""
    if os.environ.get("DIFFLET_DISABLE_PREWARM"):
        return None
    try:
        import torch

        if not torch.cuda.is_available():
            return None
    except Exception:  # noqa: BLE001
        return None

    def touch() -> None:
        try:
            import torch

            devs = devices if devices is not None else [torch.cuda.current_device()]
            for d in devs:
                with torch.cuda.device(d):
                    x = torch.empty(1 << 20, device=f"cuda:{d}", dtype=torch.bfloat16)
                    torch.cuda.synchronize(d)
                    del x
            from difflet_b200 import _native

            _native.load()  # dlopen + module registration of the sm_100a kernels
        except Exception:  # noqa: BLE001 - the main thread pays the start-up instead
            pass

    t = threading.Thread(target=touch, name="difflet-prewarm", daemon=True)
    t.start()
    return t


__all__ = ["prewarm_cuda"]
