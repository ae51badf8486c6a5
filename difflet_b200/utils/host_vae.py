"""``--host-vae``: run a pipeline's VAE decode on the host CPU in fp32.

The decoder's weights move to host memory once at load, freeing their device memory (and the
decode's activations) for the DiT; the final latents are copied to the host and decoded there
by the same decoder code on its CPU path (the PyTorch oracle of the native kernels).  Much
slower than the device decode (``--device-vae``, the default); meant for memory-bound setups.
"""

from __future__ import annotations

import torch


def move_to_host(vae) -> None:
    """Move a decoder's weight dict (``vae.w``) to host memory in fp32 (in place)."""
    vae.w = {k: (v.to("cpu", torch.float32) if v.is_floating_point() else v.to("cpu")) for k, v in vae.w.items()}
    if hasattr(vae, "_convs"):
        vae._convs = None  # kernel-layout copies are rebuilt from the host weights
    if hasattr(vae, "slabs"):
        vae.slabs = None


def vae_device(vae):
    w = getattr(vae, "w", None)
    if not w:
        return None
    return next(iter(w.values())).device


def for_vae(vae, z: torch.Tensor) -> torch.Tensor:
    """``z`` on the decoder's device and in its weights' dtype."""
    dev = vae_device(vae)
    if dev is None:
        return z
    dt = next(iter(vae.w.values())).dtype
    return z.to(dev, dt)
