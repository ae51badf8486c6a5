"""CFG parallelism: the two guidance branches on two ranks, exchanged through peer memory.

Reference semantics (``difflet/models/wan/pipeline.py:389-407``,
``difflet/models/wan/modeling_wan.py:941-963,1063-1066``): the batch
``[uncond, cond]`` is split over a cfg axis of 2; after the DiT forward the two
predictions are gathered and combined as ``u + s (c - u)``.  Here each rank
keeps its branch's prediction in a symmetric buffer and one kernel reads the
partner's prediction over NVLink and writes the combined fp32 velocity (no
NCCL all-gather, no staging copy); both ranks then take the same scheduler step
and stay bit-identical.  ``CollectiveCfg`` is the NCCL / gloo baseline.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from difflet_b200.ops import fused as F


class PeerCfg:
    def __init__(self, group, ranks, device):
        from difflet_b200.parallel.symm import SymmetricHeap

        self.heap = SymmetricHeap(group, ranks, device)
        self.rank = self.heap.rank          # 0 = uncond branch, 1 = cond branch
        self.is_cond = self.rank == 1
        self._pred = {}
        self._turn = 0

    def pred_buffer(self, shape, dtype=torch.bfloat16, parity: int = 0):
        """The symmetric prediction buffer of one parity (two alternate between steps)."""
        key = (tuple(shape), dtype, parity)
        if key not in self._pred:
            self._pred[key] = self.heap.empty(shape, dtype)
        return self._pred[key]

    def next_pred_buffer(self, shape, dtype=torch.bfloat16):
        """Where this step's prediction should be written (the DiT's final projection stores
        straight into it).  Buffers alternate by step, so one barrier per step suffices: a rank
        writes a buffer again only after the next step's barrier, which its partner passes
        only after its read of that buffer was issued on its stream."""
        return self.pred_buffer(shape, dtype, self._turn)

    def step(self, pred: torch.Tensor, scale: float, sampler) -> None:
        """CFG exchange + guidance combine + sampler update (``GuidedSampler``) in one kernel:
        this rank's prediction and the partner's, read over NVLink, form u + s (c - u); both
        ranks apply the identical update to their copy of the latents."""
        buf = self.pred_buffer(pred.shape, pred.dtype, self._turn)
        if buf.data_ptr() != pred.data_ptr():
            buf.copy_(pred)
        self.heap.barrier()  # the partner's prediction of this step is complete
        peer = self.heap.peer_ptrs(buf)[1 - self.rank]
        sampler.step(buf, None, scale, b_ptr=peer, swap=self.is_cond)
        self._turn ^= 1

    def combine(self, pred: torch.Tensor, scale: float, out: torch.Tensor | None = None) -> torch.Tensor:
        buf = self.pred_buffer(pred.shape, pred.dtype)
        if buf.data_ptr() != pred.data_ptr():
            buf.copy_(pred)
        out = out if out is not None else torch.empty(pred.shape, device=pred.device, dtype=torch.float32)
        self.heap.barrier()  # partner's prediction is complete
        peer = self.heap.peer_ptrs(buf)[1 - self.rank]
        F.native().cfg_combine(buf, peer, out, float(scale), self.is_cond)
        self.heap.barrier()  # partner finished reading mine before either overwrites
        return out

    def close(self):
        self.heap.close()


class CollectiveCfg:
    def __init__(self, group, ranks, device):
        self.group = group
        self.ranks = list(ranks)
        self.rank = self.ranks.index(dist.get_rank())
        self.is_cond = self.rank == 1

    def next_pred_buffer(self, shape, dtype=torch.bfloat16):
        return None  # the DiT allocates its own output

    def step(self, pred, scale, sampler) -> None:
        """All-gather of both branches (NCCL / gloo), then the fused combine + update."""
        parts = [torch.empty_like(pred) for _ in range(2)]
        dist.all_gather(parts, pred.contiguous(), group=self.group)
        sampler.step(parts[0].contiguous(), parts[1].contiguous(), scale)

    def combine(self, pred, scale, out=None):
        parts = [torch.empty_like(pred) for _ in range(2)]
        dist.all_gather(parts, pred.contiguous(), group=self.group)
        u, c = parts[0].float(), parts[1].float()
        r = u + scale * (c - u)
        if out is not None:
            out.copy_(r)
            return out
        return r

    def close(self):
        pass
