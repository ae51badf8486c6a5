"""Device state of the fused guidance + sampler step (one kernel per denoise step).

``GuidedSampler`` owns a latent tensor's sampler state on the device -- the f32 sample, its
bf16 mirror the DiT reads, and for UniPC the previous corrected sample and the last two data
predictions -- and advances it with ``ops.fused.guided_step``: the CFG combine of the two
branch predictions, the UniPC corrector + predictor (or the flow-matching Euler update) and the
bf16 mirror in one pass over the latents.  The history buffers rotate on the host; nothing is
copied between steps.  Under CFG parallelism (``parallel/cfg.py``) the other branch's
prediction is read from the partner rank's memory by the same kernel.

Reference: the CFG combine and UniPC steps of difflet/models/wan/pipeline.py:403-405,525-582,
the Euler step of difflet/models/flux/pipeline.py:414-420.
"""

from __future__ import annotations

import torch

from difflet_b200.ops import fused as F
from difflet_b200.schedulers.flow_match import FlowMatchEulerScheduler
from difflet_b200.schedulers.unipc import UniPCScheduler


class GuidedSampler:
    def __init__(self, scheduler, x32: torch.Tensor, x16: torch.Tensor | None = None):
        if not x32.is_contiguous():
            raise ValueError("the sampler's latents must be contiguous")
        self.sched = scheduler
        self.x = x32
        self.x16 = x16
        self.i = 0
        self.multistep = isinstance(scheduler, UniPCScheduler)
        if self.multistep:
            self.last = torch.zeros_like(x32)
            self.m1 = torch.zeros_like(x32)
            self.m2 = torch.zeros_like(x32)

    def coeffs(self):
        """(k_v, e, g, store_last) of the next step."""
        if self.multistep:
            k_v, e, g = self.sched.fused_coeffs()
            return k_v, e, g, True
        if isinstance(self.sched, FlowMatchEulerScheduler):
            dt = self.sched.dt(self.i)
            return 0.0, (1.0, 0.0, 0.0, 0.0, 0.0), (1.0, 0.0, 0.0, 0.0, 0.0, dt), False
        raise TypeError(f"no fused update for {type(self.sched).__name__}")

    def step(self, a: torch.Tensor, b: torch.Tensor | None = None, scale: float = 1.0, *, b_ptr=None,
             swap: bool = False):
        """One step from the prediction ``a`` (uncond) and ``b`` (cond, or None without CFG);
        ``b_ptr`` gives ``b`` as a device pointer instead (a peer rank's buffer); ``swap``: ``a``
        is the cond branch and ``b`` the uncond one (the combine is evaluated the same way)."""
        k_v, e, g, store_last = self.coeffs()
        if self.multistep:
            F.guided_step(a, b, scale=scale, x=self.x, x16=self.x16, last=self.last, m1=self.m1, m2=self.m2,
                          m_out=self.m2, k_v=k_v, e=e, g=g, store_last=store_last, b_ptr=b_ptr, swap=swap)
            self.m1, self.m2 = self.m2, self.m1  # this step's m is next step's m1
        else:
            F.guided_step(a, b, scale=scale, x=self.x, x16=self.x16, k_v=k_v, e=e, g=g, b_ptr=b_ptr, swap=swap)
        self.i += 1
        return self.x


__all__ = ["GuidedSampler"]
