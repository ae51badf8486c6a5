"""Ring and gather-KV context parallelism (joint MMDiT and plain self-attention).

Every rank owns ``n0`` rows of the first stream and ``n1`` rows of the second
(for MMDiT ``[text ; image]`` or ``[image ; text]``; Wan has one stream) and
computes the queries of exactly those rows for all heads, so no query, text or
image row is computed twice.  What differs is how each rank sees the keys:

ring (``cp_mode="ring"``, memory O(S / cp) per rank)
    The K/V of a rank's own rows are written by the fused q/k/v kernel into a
    symmetric buffer.  Hop 0 attends to them; hop ``j`` attends to the block of
    rank ``(rank + j) % cp``, which a copy engine pulls over NVLink into a local
    double buffer on a side stream while the previous hop computes.  The
    attention kernel merges each hop's partial by log-sum-exp into an fp32
    running output in its epilogue and the last hop writes the bf16 rows.
    Semantics of ``ring_attention`` / ``joint_ring_attention``
    (difflet/backends/neuron/ops_impl/attention.py:435-456, :518-583, merge
    :607-619); the text block here is sharded like the image block instead of
    being replicated, which is the same softmax over the same keys.

gather-KV (``cp_mode="gather_kv"``, K/V O(S) per rank)
    The fused q/k/v kernel stores each K/V row into every rank's full K/V
    buffer (the all-gather is its store pattern); one attention call over all
    keys follows (difflet/models/flux/modeling_flux.py:1330-1357).

Key windows: a per-batch prefix window ``[0, kv_hi)`` over the global joint
sequence (a padded text stream placed last) maps to one prefix window per ring
block, computed once per forward.

``CollectiveRing`` / ``CollectiveGatherKV`` run the same math with
``torch.distributed`` point-to-point / all-gather (gloo on CPU, NCCL on GPU):
the multi-rank oracle of the tests and the baseline of the fused path.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from difflet_b200.ops import fused as F
from difflet_b200.parallel.ulysses import PeerBase, _Base


def block_windows(kv_hi: torch.Tensor, n0: int, n1: int, world: int) -> torch.Tensor:
    """[world, B] int32: the prefix window of each rank's ``[seg0_j ; seg1_j]`` key block
    for a global prefix window ``[0, kv_hi[b])`` over ``[seg0_all ; seg1_all]``."""
    j = torch.arange(world, device=kv_hi.device, dtype=torch.int64)[:, None]
    hi = kv_hi.to(torch.int64)[None, :]
    a = (hi - j * n0).clamp(0, n0)
    b = (hi - n0 * world - j * n1).clamp(0, n1)
    return (a + b).to(torch.int32).contiguous()


class _LocalKV:
    """Shared by ring / gather-KV: local queries for all heads, output rows written locally."""

    def heads_local(self, H: int) -> int:
        return H

    def check_heads(self, H: int) -> None:
        pass

    @staticmethod
    def out_view(target, B, H, S_loc, dh, ld):
        return target.as_strided((B, H, S_loc, dh), (S_loc * ld, dh, ld, 1))


# ---------------------------------------------------------------------------- ring
class _RingWindows:
    def _windows(self, kv_lo, kv_hi, n0, n1):
        if kv_hi is None:
            return None
        if getattr(self, "_win_src", None) is not kv_hi:
            self._win_src = kv_hi
            self._win = block_windows(kv_hi, n0, n1, self.world)
        return self._win


class PeerRing(_LocalKV, _RingWindows, PeerBase):
    kind = "ring"

    def __init__(self, group, ranks, device):
        super().__init__(group, ranks, device)
        self._kv = {}
        self._bufs = {}
        self._acc = {}
        self._side = torch.cuda.Stream(device=device)
        self._events = None

    def layout(self, B, H, dh, S_loc, S, dtype):
        q = torch.empty(B, H, S_loc, dh, device=self.device, dtype=dtype)
        kv = self.heap.empty((2, B, H, S_loc, dh), dtype)
        self._kv[kv[0].data_ptr()] = kv
        return q, kv[0], kv[1]

    def scatter_kwargs(self, q, k, v, row, pos, S_loc, S, H):
        return dict(q_dst=[q], k_dst=[k], v_dst=[v], S_dst=S_loc, seq_off=row, heads_per_rank=H)

    def _buffers(self, kv):
        key = kv.data_ptr()
        if key not in self._bufs:
            self._bufs[key] = [torch.empty_like(kv) for _ in range(2)]
        return self._bufs[key]

    def _accumulators(self, B, H, S_loc):
        key = (B, H, S_loc)
        if key not in self._acc:
            self._acc[key] = (torch.empty(B, H, S_loc, 128, device=self.device, dtype=torch.float32),
                              torch.empty(B, H, S_loc, device=self.device, dtype=torch.float32))
        return self._acc[key]

    def attention(self, q, k, v, scale, target, B, n0, n1, ld, kv_lo=None, kv_hi=None):
        H, S_loc, dh = q.shape[1], q.shape[2], q.shape[3]
        W, r = self.world, self.rank
        kv = self._kv[k.data_ptr()]
        bufs = self._buffers(kv)
        acc_o, acc_lse = self._accumulators(B, H, S_loc)
        wins = self._windows(kv_lo, kv_hi, n0, n1)
        win = (lambda j: None) if wins is None else (lambda j: wins[j])  # noqa: E731
        o = self.out_view(target, B, H, S_loc, dh, ld)
        nat = F.native()
        peers = self.heap.peer_ptrs(kv)
        nbytes = kv.numel() * kv.element_size()
        if self._events is None or len(self._events[0]) < W + 1:
            self._events = ([torch.cuda.Event() for _ in range(W + 1)], [torch.cuda.Event() for _ in range(W + 1)])
        copied, attended = self._events
        main, side = torch.cuda.current_stream(self.device), self._side

        self.heap.barrier()  # every rank's K/V block of this layer is written
        attended[0].record(main)
        side.wait_event(attended[0])

        def pull(j):  # block of rank (r + j) % W into bufs[(j - 1) % 2]
            with torch.cuda.stream(side):
                if j >= 3:  # hop j - 2 read this buffer
                    side.wait_event(attended[j - 2])
                nat.memcpy_async(bufs[(j - 1) % 2].data_ptr(), peers[(r + j) % W], nbytes)
                copied[j].record(side)

        pull(1)
        F.attention_partial(q, kv[0], kv[1], scale, acc_o, acc_lse, F.MERGE_FIRST, kv_hi=win(r))
        for j in range(1, W):
            if j + 1 < W:
                pull(j + 1)
            main.wait_event(copied[j])
            buf = bufs[(j - 1) % 2]
            mode = F.MERGE_LAST if j == W - 1 else F.MERGE_MID
            F.attention_partial(q, buf[0], buf[1], scale, acc_o, acc_lse, mode, out=o, kv_hi=win((r + j) % W))
            attended[j].record(main)
        self.heap.barrier()  # every peer finished pulling this rank's block


class CollectiveRing(_LocalKV, _RingWindows, _Base):
    """Ring shift with point-to-point send / recv (gloo or NCCL)."""

    kind = "ring"

    def empty(self, shape, dtype):
        return torch.zeros(shape, dtype=dtype, device=self.device)

    def peer_views(self, t):
        return [t]

    def layout(self, B, H, dh, S_loc, S, dtype):
        return tuple(self.empty((B, H, S_loc, dh), dtype) for _ in range(3))

    def scatter_kwargs(self, q, k, v, row, pos, S_loc, S, H):
        return dict(q_dst=[q], k_dst=[k], v_dst=[v], S_dst=S_loc, seq_off=row, heads_per_rank=H)

    def attention(self, q, k, v, scale, target, B, n0, n1, ld, kv_lo=None, kv_hi=None):
        H, S_loc, dh = q.shape[1], q.shape[2], q.shape[3]
        W, r = self.world, self.rank
        wins = self._windows(kv_lo, kv_hi, n0, n1)
        acc_o = torch.empty(B, H, S_loc, dh, device=q.device, dtype=torch.float64 if q.dtype == torch.float64
                            else torch.float32)
        acc_lse = torch.empty(B, H, S_loc, device=q.device, dtype=acc_o.dtype)
        o = self.out_view(target, B, H, S_loc, dh, ld)
        cur = torch.stack([k, v]).contiguous()
        nxt = torch.empty_like(cur)
        dst_rank, src_rank = self.ranks[(r - 1) % W], self.ranks[(r + 1) % W]
        for j in range(W):
            mode = F.MERGE_FIRST if j == 0 else (F.MERGE_LAST if j == W - 1 else F.MERGE_MID)
            reqs = []
            if j + 1 < W:  # block (r + j) goes to rank r - 1; block (r + j + 1) arrives from r + 1
                reqs = [dist.isend(cur, dst_rank, group=self.group), dist.irecv(nxt, src_rank, group=self.group)]
            F.attention_partial(q, cur[0], cur[1], scale, acc_o, acc_lse, mode, out=o,
                                kv_hi=None if wins is None else wins[(r + j) % W])
            for rq in reqs:
                rq.wait()
            cur, nxt = nxt, cur


# ---------------------------------------------------------------------------- gather-KV
class PeerGatherKV(_LocalKV, PeerBase):
    kind = "gather_kv"

    def layout(self, B, H, dh, S_loc, S, dtype):
        q = torch.empty(B, H, S_loc, dh, device=self.device, dtype=dtype)
        kv = self.heap.empty((2, B, H, S, dh), dtype)
        return q, kv[0], kv[1]

    def scatter_kwargs(self, q, k, v, row, pos, S_loc, S, H):
        pad = [None] * (self.world - 1)
        return dict(q_dst=[q] + pad, k_dst=self.peer_views(k), v_dst=self.peer_views(v), S_dst=S, seq_off=pos,
                    heads_per_rank=H, kv_replicate=True, q_S_dst=S_loc, q_seq_off=row)

    def attention(self, q, k, v, scale, target, B, n0, n1, ld, kv_lo=None, kv_hi=None):
        H, S_loc, dh = q.shape[1], q.shape[2], q.shape[3]
        self.heap.barrier()  # every rank's K/V rows have landed here
        F.attention(q, k, v, scale, out=self.out_view(target, B, H, S_loc, dh, ld), kv_lo=kv_lo, kv_hi=kv_hi)
        self.heap.barrier()  # every rank finished reading before the next layer's stores


class CollectiveGatherKV(_LocalKV, _Base):
    """All-gather of the K/V rows with ``torch.distributed`` (gloo or NCCL)."""

    kind = "gather_kv"

    def empty(self, shape, dtype):
        return torch.zeros(shape, dtype=dtype, device=self.device)

    def peer_views(self, t):
        return [t]

    def layout(self, B, H, dh, S_loc, S, dtype):
        q = self.empty((B, H, S_loc, dh), dtype)
        return q, self.empty((B, H, S, dh), dtype), self.empty((B, H, S, dh), dtype)

    def scatter_kwargs(self, q, k, v, row, pos, S_loc, S, H):
        return dict(q_dst=[q], k_dst=[k], v_dst=[v], S_dst=S, seq_off=pos, heads_per_rank=H, kv_replicate=True,
                    q_S_dst=S_loc, q_seq_off=row)

    def _rows(self, n0, n1, r, device):
        S0 = n0 * self.world
        return torch.cat([torch.arange(r * n0, (r + 1) * n0), S0 + torch.arange(r * n1, (r + 1) * n1)]).to(device)

    def attention(self, q, k, v, scale, target, B, n0, n1, ld, kv_lo=None, kv_hi=None):
        H, S_loc, dh = q.shape[1], q.shape[2], q.shape[3]
        for t in (k, v):
            mine = t[:, :, self._rows(n0, n1, self.rank, t.device)].contiguous()
            parts = [torch.empty_like(mine) for _ in range(self.world)]
            dist.all_gather(parts, mine, group=self.group)
            for src in range(self.world):
                t[:, :, self._rows(n0, n1, src, t.device)] = parts[src]
        F.attention(q, k, v, scale, out=self.out_view(target, B, H, S_loc, dh, ld), kv_lo=kv_lo, kv_hi=kv_hi)
