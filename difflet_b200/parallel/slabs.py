"""Spatial slabs of a multi-GPU video decode: the picture's rows split over ranks, with one row
of halo context above and below each rank's rows for the 3x3 convolutions.

Three transports with one interface (``empty`` zero-filled buffers, ``neighbours`` for the
producer kernels' halo stores, ``sync`` after a producer, ``gather_rows`` / ``gather_video``):

``PeerSlabs`` (B200 path)
    Buffers live in symmetric peer memory.  The producer of a convolution's input (the channel
    RMS norm + SiLU, the nearest upsampler) stores its first and last rows straight into the
    neighbouring ranks' halo rows over NVLink (``csrc/vae.cu``); ``sync`` is one device barrier.
``CollectiveSlabs`` (CPU / NCCL baseline)
    The producer writes only its own rows; ``sync`` all-gathers every rank's boundary rows and
    fills the halos.
``LocalSlabs``: one device, whole frames (halo rows stay zero: the picture's own border).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class _Slabs:
    def __init__(self, world: int, rank: int, rows: int):
        self.world, self.rank, self.rows = world, rank, rows

    def bounds(self, r: int, rows: int | None = None) -> tuple[int, int]:
        """Rows [r0, r1) of rank r in a picture of ``rows`` rows (default: the latent's)."""
        rows = self.rows if rows is None else rows
        scale = rows // self.rows
        return (r * self.rows // self.world) * scale, ((r + 1) * self.rows // self.world) * scale

    def local_rows(self, rows: int | None = None) -> int:
        r0, r1 = self.bounds(self.rank, rows)
        return r1 - r0

    @property
    def halo(self) -> int:
        return 1 if self.world > 1 else 0

    def neighbours(self, buf: torch.Tensor, frame_off: int, rows: int) -> dict:
        """Keyword arguments of the producer kernels: peer pointers of the slabs above / below
        (their frame ``frame_off`` of the same buffer) and their row counts."""
        return {}

    def sync(self, buf: torch.Tensor, frames: slice, rows: int) -> None:
        pass

    def close(self) -> None:
        pass


class LocalSlabs(_Slabs):
    def __init__(self, rows: int, device):
        super().__init__(1, 0, rows)
        self.device = device
        self.distributed = False

    def empty(self, shape, dtype) -> torch.Tensor:
        return torch.zeros(shape, dtype=dtype, device=self.device)

    def gather_rows(self, t: torch.Tensor, rows: int) -> torch.Tensor:
        return t

    def gather_video(self, t: torch.Tensor, rows: int):
        return t


class CollectiveSlabs(_Slabs):
    distributed = True

    def __init__(self, group, ranks, device, rows: int):
        super().__init__(len(ranks), list(ranks).index(dist.get_rank()), rows)
        self.group, self.device = group, device

    def empty(self, shape, dtype) -> torch.Tensor:
        return torch.zeros(shape, dtype=dtype, device=self.device)

    def sync(self, buf: torch.Tensor, frames: slice, rows: int) -> None:
        """buf [F, rows + 2, W, C]: fill the halo rows of ``frames`` from the neighbours."""
        own = buf[frames, 1:rows + 1]
        edge = torch.stack([own[:, 0], own[:, -1]], 1).contiguous()  # [F, 2, W, C]
        parts = [torch.empty_like(edge) for _ in range(self.world)]
        dist.all_gather(parts, edge, group=self.group)
        if self.rank > 0:
            buf[frames, 0] = parts[self.rank - 1][:, 1]
        if self.rank < self.world - 1:
            buf[frames, rows + 1] = parts[self.rank + 1][:, 0]

    def _gather(self, t: torch.Tensor, rows: int, dim: int) -> list:
        """Every rank's slab of ``t`` (rows along ``dim``), padded to the largest slab for the
        collective and trimmed again."""
        rmax = max(self.bounds(r, rows)[1] - self.bounds(r, rows)[0] for r in range(self.world))
        pad = list(t.shape)
        pad[dim] = rmax
        buf = torch.zeros(pad, dtype=t.dtype, device=t.device)
        buf.narrow(dim, 0, t.shape[dim]).copy_(t)
        parts = [torch.empty_like(buf) for _ in range(self.world)]
        dist.all_gather(parts, buf, group=self.group)
        out = []
        for r, p in enumerate(parts):
            r0, r1 = self.bounds(r, rows)
            out.append(p.narrow(dim, 0, r1 - r0))
        return out

    def gather_rows(self, t: torch.Tensor, rows: int) -> torch.Tensor:
        """[F, rows_local, ...] on every rank -> [F, rows, ...] on every rank."""
        return torch.cat(self._gather(t, rows, 1), 1)

    def gather_video(self, t: torch.Tensor, rows: int):
        """[F, rows_local, W, 3] -> the whole video on rank 0 (None elsewhere)."""
        full = torch.cat(self._gather(t, rows, 1), 1)
        return full if self.rank == 0 else None


class PeerSlabs(CollectiveSlabs):
    """Symmetric-heap buffers; halo rows arrive by the producers' peer stores."""

    def __init__(self, group, ranks, device, rows: int):
        super().__init__(group, ranks, device, rows)
        from difflet_b200.parallel.symm import SymmetricHeap

        self.heap = SymmetricHeap(group, ranks, device)

    def empty(self, shape, dtype) -> torch.Tensor:
        # zero-filled and synchronised by the allocation itself: a zero_() queued here could run
        # after a neighbour's producer kernel has already stored halo rows into this buffer
        return self.heap.empty(shape, dtype)

    def neighbours(self, buf: torch.Tensor, frame_off: int, rows: int) -> dict:
        # buf is this rank's [F, rows + 2, W, C] view from the base of its symmetric allocation;
        # a neighbour's view has its own row count, so its frame stride differs
        W, C = buf.shape[2], buf.shape[3]
        esz = buf.element_size()
        ptrs = self.heap.peer_ptrs(buf)
        out = {}
        scale = rows // self.local_rows() if self.local_rows() else 1
        for side, r in (("up", self.rank - 1), ("down", self.rank + 1)):
            if 0 <= r < self.world:
                b0, b1 = self.bounds(r)
                nr = (b1 - b0) * scale
                out[side] = ptrs[r] + frame_off * (nr + 2) * W * C * esz
                out[side + "_rows"] = nr
        return out

    def sync(self, buf: torch.Tensor, frames: slice, rows: int) -> None:
        self.heap.barrier()

    def close(self) -> None:
        self.heap.close()


def make_slabs(rows: int, device, group=None, ranks=None, transport: str | None = None):
    """Slabs over ``ranks`` (default: every rank of an initialised process group)."""
    from difflet_b200 import envs

    if not dist.is_initialized() or (ranks is not None and len(ranks) == 1) or dist.get_world_size() == 1:
        return LocalSlabs(rows, device)
    if ranks is None:
        ranks = list(range(dist.get_world_size()))
        group = dist.group.WORLD
    transport = transport or envs.DIFFLET_KERNEL_COMM
    if device.type == "cuda" and transport == "fused":
        return PeerSlabs(group, ranks, device, rows)
    return CollectiveSlabs(group, ranks, device, rows)


__all__ = ["CollectiveSlabs", "LocalSlabs", "PeerSlabs", "make_slabs"]
