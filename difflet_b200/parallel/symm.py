"""Symmetric peer memory over CUDA IPC (NVLink / NVSwitch).

Every rank of a group allocates the same buffers in the same order
(``cudaMalloc`` in the native runtime), exports IPC handles, all-gathers them
and opens the peers', so each buffer has a table of peer device pointers that
the fused kernels store to / load from directly.  A device epoch barrier
(``barrier()``) orders those accesses; its counter lives on the GPU, so it is
valid inside CUDA graphs.  No NVLS object is created: plain P2P
loads and stores only.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from difflet_b200 import envs


class SymmetricHeap:
    def __init__(self, group, ranks: list[int], device: torch.device):
        from difflet_b200 import _native

        self.nat = _native.require()
        self.group = group
        self.ranks = list(ranks)
        self.world = len(ranks)
        self.rank = self.ranks.index(dist.get_rank())
        self.device = device
        self._local: list[torch.Tensor] = []
        self._opened: list[int] = []
        self._peers: dict[int, list[int]] = {}  # local data_ptr -> peer base pointers (index = group rank)
        self._retired: list[torch.Tensor] = []
        self._nbytes: dict[int, int] = {}
        # barrier flags: world int32 slots; counter: local epoch
        self.flags, self.flag_ptrs = self._alloc_raw(max(self.world, 4) * 4)
        self.counter = torch.zeros(1, dtype=torch.int32, device=device)
        self.timeout = int(envs.DIFFLET_COMM_TIMEOUT_CYCLES)
        dist.barrier(group=group)

    def _alloc_raw(self, nbytes: int):
        nbytes = int(math.ceil(nbytes / 256) * 256)
        t = self.nat.symm_alloc(nbytes, self.device.index)
        h = self.nat.ipc_handle(t)
        handles = [None] * self.world
        dist.all_gather_object(handles, h, group=self.group)
        ptrs = []
        for r, hr in enumerate(handles):
            if r == self.rank:
                ptrs.append(t.data_ptr())
            else:
                p = self.nat.ipc_open(hr, self.device.index)
                self._opened.append(p)
                ptrs.append(p)
        self._local.append(t)
        self._peers[t.data_ptr()] = ptrs
        self._nbytes[t.data_ptr()] = nbytes
        return t, ptrs

    CANARY_BYTES = 256
    CANARY_BYTE = 0xA5

    def empty(self, shape, dtype) -> torch.Tensor:
        """A symmetric buffer.  With DIFFLET_BOUNDS_CHECK=1 it is followed by a 256-byte canary
        region that ``check_canaries`` verifies (a peer store past the end shows up there)."""
        n = int(math.prod(shape)) * torch.empty((), dtype=dtype).element_size()
        guard = self.CANARY_BYTES if envs.DIFFLET_BOUNDS_CHECK else 0
        raw, _ = self._alloc_raw(n + guard)
        # _alloc_raw returns a buffer zeroed (cudaMemset + device synchronise) before the handle
        # exchange, so no rank can see a peer's buffer before it is zero
        if guard:
            if not hasattr(self, "_canaries"):
                self._canaries = []
            c = raw[n:n + guard]
            c.fill_(self.CANARY_BYTE)
            self._canaries.append(c)
        return raw[:n].view(dtype).view(shape)

    def check_canaries(self) -> None:
        """Raise when any canary region after a symmetric buffer was overwritten."""
        for i, c in enumerate(getattr(self, "_canaries", [])):
            if not bool((c == self.CANARY_BYTE).all()):
                from difflet_b200.utils.errors import DeviceError

                raise DeviceError(code=3, kernel=0, detail=(i, int((c != self.CANARY_BYTE).sum())))

    def peer_ptrs(self, t: torch.Tensor) -> list[int]:
        """Peer pointers of the same element as ``t`` (which may be a view) on every rank."""
        p = t.data_ptr()
        for base, ptrs in self._peers.items():
            if base <= p < base + self._nbytes[base]:
                off = p - base
                return [q + off for q in ptrs]
        raise KeyError("tensor is not in the symmetric heap")

    def barrier(self) -> None:
        self.nat.peer_barrier(self.flag_ptrs, self.counter, self.rank, self.timeout)

    def retire(self, t: torch.Tensor) -> None:
        """Keep a symmetric buffer that is being replaced alive until ``close``: peers have it
        mapped, and freeing an exported allocation before every importer has closed it is
        undefined behaviour."""
        self._retired.append(t)

    def close(self) -> None:
        """Unmap the peers' buffers, wait until every rank has unmapped ours, then free ours."""
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            self.nat.ipc_close(p)
        self._opened.clear()
        self._peers.clear()
        try:
            dist.barrier(group=self.group)
        except Exception:  # noqa: BLE001 - a broken group: the process is going down anyway
            pass
        self._local.clear()
        self._retired.clear()
