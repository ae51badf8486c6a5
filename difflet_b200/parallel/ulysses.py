"""Ulysses sequence parallelism for MMDiT models (joint ``[text ; image]`` attention).

Semantics of the reference's ``ulysses_attention`` / joint variants
(``difflet/backends/neuron/ops_impl/attention.py:622-713``,
``difflet/backends/neuron/ops_impl/collectives.py:276-348``): every rank holds
``1/N`` of the text rows and ``1/N`` of the image rows; attention needs all
rows for ``H/N`` heads, so q/k/v go sequence->heads and the output goes
heads->sequence.  ``heads % N == 0`` is required.

Two transports with one interface:

``PeerUlysses`` (B200 path)
    q/k/v and attention-output buffers live in symmetric peer memory.  The
    fused q/k-norm + RoPE kernel stores each head block straight into the
    owning rank's q/k/v buffer (the seq->heads all-to-all is its store
    pattern), and the attention kernel's epilogue stores each output row into
    the owning rank's buffer (heads->seq).  Two device barriers per attention
    order the traffic.  No separate collective kernels, no staging copies.

``CollectiveUlysses`` (baseline / CPU)
    The same math with ``torch.distributed.all_to_all`` (NCCL on GPU, gloo on
    CPU) plus pack / unpack copies: the measured NCCL baseline of the fused
    path, and the multi-rank oracle that runs on CPU gloo ranks in the tests.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from difflet_b200 import envs
from difflet_b200.ops import fused as F


def all_to_all(recv: list, send: list, group) -> None:
    """``dist.all_to_all`` (NCCL), or point-to-point pairs where the backend lacks it (gloo)."""
    if dist.get_backend(group) != "gloo":
        dist.all_to_all(recv, send, group=group)
        return
    ranks = dist.get_process_group_ranks(group) if group is not None else list(range(dist.get_world_size()))
    me = dist.get_rank()
    reqs = []
    for i, r in enumerate(ranks):
        if r == me:
            recv[i].copy_(send[i])
            continue
        reqs.append(dist.isend(send[i].contiguous(), r, group=group))
        reqs.append(dist.irecv(recv[i], r, group=group))
    for q in reqs:
        q.wait()


class _Base:
    """Context-parallel state shared by every CP mode.  The model asks it for its
    q/k/v buffers (``layout``), for the destinations of the fused q/k/v scatter
    (``scatter_kwargs``) and runs ``attention``; the three modes differ only there."""

    kind = "ulysses"

    def __init__(self, group, ranks, device):
        self.group = group
        self.ranks = list(ranks)
        self.world = len(ranks)
        self.rank = self.ranks.index(dist.get_rank())
        self.device = device
        self.decode_on_all_ranks = False

    def heads_local(self, H: int) -> int:
        return H // self.world

    def layout(self, B, H, dh, S_loc, S, dtype):
        """q, k, v buffers: this rank's heads over the full joint sequence."""
        Hl = self.heads_local(H)
        return tuple(self.empty((B, Hl, S, dh), dtype) for _ in range(3))

    def scatter_kwargs(self, q, k, v, row, pos, S_loc, S, H):
        """qkv_scatter destinations for rows at local offset ``row`` / global position ``pos``."""
        return dict(q_dst=self.peer_views(q), k_dst=self.peer_views(k), v_dst=self.peer_views(v), S_dst=S,
                    seq_off=pos, heads_per_rank=self.heads_local(H))

    def close(self):
        pass

    # token sharding of the model inputs / outputs
    def shard_tokens(self, x: torch.Tensor) -> torch.Tensor:
        n = x.shape[1] // self.world
        return x[:, self.rank * n:(self.rank + 1) * n]

    def gather_tokens(self, x_loc: torch.Tensor) -> torch.Tensor:
        parts = [torch.empty_like(x_loc) for _ in range(self.world)]
        dist.all_gather(parts, x_loc.contiguous(), group=self.group)
        return torch.cat(parts, 1)

    def check_heads(self, H: int) -> None:
        if H % self.world:
            raise ValueError(f"Ulysses needs heads % world == 0, got {H} heads on {self.world} ranks")


class PeerBase(_Base):
    """Symmetric-heap transport shared by the fused (peer-memory) CP modes."""

    def __init__(self, group, ranks, device):
        super().__init__(group, ranks, device)
        from difflet_b200.parallel.symm import SymmetricHeap

        self.heap = SymmetricHeap(group, ranks, device)

    def empty(self, shape, dtype):
        return self.heap.empty(shape, dtype)

    def peer_views(self, t: torch.Tensor):
        return self.heap.peer_ptrs(t)

    def shard_gemv(self, W, x, bias, *, silu_in=False, silu_out=False):
        """Row-sharded GEMV + all-gather by peer stores: each rank reads 1/N of W
        (the adaLN modulation matrix is 6.5 GB for FLUX) and writes its slice of
        the f32 result into every rank's symmetric copy.  Returns None when the
        shape does not shard (the caller then runs the full GEMV)."""
        N = W.shape[0]
        if x.shape[0] != 1 or N % self.world or (N // self.world) % 4:
            return None
        if not hasattr(self, "_gemv_out"):
            self._gemv_out = {}
        out = self._gemv_out.get(N)
        if out is None:
            out = self._gemv_out[N] = self.heap.empty((1, N), torch.float32)
        n = N // self.world
        r0 = self.rank * n
        F.gemv(W[r0:r0 + n], x, None if bias is None else bias[r0:r0 + n], silu_in=silu_in, silu_out=silu_out,
               out=out[:, r0:r0 + n])
        self.heap.barrier()  # every rank is done reading its copy from the previous step
        F.native().peer_put_f32(out[0, r0:r0 + n], self.heap.peer_ptrs(out), r0)
        self.heap.barrier()  # every slice has landed everywhere
        return out

    def before_attention(self):
        self.heap.barrier()

    def close(self):
        self.heap.close()


class PeerUlysses(PeerBase):
    def attention(self, q, k, v, scale, target, B, n0, n1, ld, kv_lo=None, kv_hi=None):
        """q/k/v: this rank's heads over the full sequence ``[seg0 ; seg1]``; each rank
        owns ``n0`` rows of seg0 and ``n1`` rows of seg1.  ``target``: local
        [B*(n0+n1), ld] buffer whose columns [rank*Hl*dh, (rank+1)*Hl*dh) receive this
        rank's heads for the rows it owns (written by the peers' epilogues)."""
        Hl, dh = q.shape[1], q.shape[3]
        S_loc = n0 + n1
        self.heap.barrier()  # every rank's q/k/v stores have landed
        col = self.rank * Hl * dh * target.element_size()
        peers = [p + col for p in self.heap.peer_ptrs(target)]
        F.native().attention(q, k, v, float(scale), None, None, kv_lo, kv_hi, peers, n0 * self.world, n0, n1,
                             [S_loc * ld, dh, ld], kv_split=F.kv_split_mode())
        self.heap.barrier()  # every output row has landed at its owner


class CollectiveUlysses(_Base):
    """All-to-all transport (NCCL / gloo).  ``peer_views`` returns per-destination
    staging buffers of the full sequence; the exchange packs this rank's rows."""

    def __init__(self, group, ranks, device):
        super().__init__(group, ranks, device)
        self._stage = {}
        self._row_cache = {}

    def empty(self, shape, dtype):
        return torch.zeros(shape, dtype=dtype, device=self.device)

    def peer_views(self, t: torch.Tensor):
        key = (t.data_ptr(), tuple(t.shape), tuple(t.stride()))
        if key not in self._stage:
            self._stage[key] = (t, [torch.zeros_like(t) for _ in range(self.world)])
        return self._stage[key][1]

    def before_attention(self):
        pass

    def _rows(self, S_txt, S_img, r):
        """Global row indices owned by rank r: its text rows then its image rows (cached on
        the device, so the first, eager call fills the cache before any graph capture)."""
        key = (S_txt, S_img, r)
        if key not in self._row_cache:
            Tg = S_txt * self.world
            txt = torch.arange(r * S_txt, (r + 1) * S_txt)
            img = Tg + torch.arange(r * S_img, (r + 1) * S_img)
            self._row_cache[key] = torch.cat([txt, img]).to(self.device)
        return self._row_cache[key]

    def _exchange_qkv(self, S_txt, S_img):
        for t, stages in list(self._stage.values()):
            # staging[r] holds this rank's rows for destination r's heads
            mine = self._rows(S_txt, S_img, self.rank)
            send = [s[:, :, mine].contiguous() for s in stages]
            recv = [torch.empty_like(send[0]) for _ in range(self.world)]
            all_to_all(recv, send, self.group)
            for src in range(self.world):
                t[:, :, self._rows(S_txt, S_img, src)] = recv[src]
            for s in stages:
                s.zero_()

    def attention(self, q, k, v, scale, target, B, S_txt, S_img, ld, kv_lo=None, kv_hi=None):
        # S_txt / S_img here are the per-rank row counts of seg0 / seg1
        Hl, S, dh = q.shape[1], q.shape[2], q.shape[3]
        self._exchange_qkv(S_txt, S_img)
        o = torch.empty(B, S, Hl * dh, dtype=q.dtype, device=q.device)
        F.attention(q, k, v, scale, out=o.view(B, S, Hl, dh).permute(0, 2, 1, 3), kv_lo=kv_lo, kv_hi=kv_hi)
        send = [o[:, self._rows(S_txt, S_img, r)].contiguous() for r in range(self.world)]
        recv = [torch.empty_like(send[0]) for _ in range(self.world)]
        all_to_all(recv, send, self.group)
        S_loc = S_txt + S_img
        tv = target.view(B, S_loc, ld)
        for src in range(self.world):
            tv[:, :, src * Hl * dh:(src + 1) * Hl * dh] = recv[src]

    def close(self):
        self._stage.clear()


def make_sequence_parallel(parallel, device, transport: str | None = None):
    """Context-parallel state over the cp axis of ``parallel`` (None when cp_degree == 1):
    Ulysses, ring or gather-KV after ``parallel.cp_mode``, over peer memory
    (``transport`` "fused", CUDA) or collectives ("nccl" / CPU gloo)."""
    from difflet_b200.parallel import groups

    if parallel.cp_degree == 1:
        return None
    if not dist.is_initialized():
        raise RuntimeError("sequence parallelism needs an initialised process group (run under torchrun)")
    if parallel.dp_degree != 1:
        raise NotImplementedError("data-parallel replicas are separate processes groups (cli/dp.py); "
                                  "build one model replica per dp coordinate")
    if groups.mesh() != parallel.mesh_spec:
        groups.init_mesh(parallel.mesh_spec)
    group, ranks = groups.get_group("cp"), groups.get_group_ranks("cp")
    transport = transport or envs.DIFFLET_KERNEL_COMM
    fused = device.type == "cuda" and transport == "fused"
    mode = getattr(parallel, "cp_mode", "ulysses")
    if mode == "ring" or mode == "gather_kv":
        from difflet_b200.parallel import ring

        if mode == "ring":
            if not fused and device.type == "cuda" and parallel.tp_degree > 1:
                # The NCCL ring baseline inside tensor parallelism (send / recv on the cp subgroup
                # interleaved with the tp all-reduces) raised an illegal-address fault on 4 B200s,
                # twice; its cause is not found, so it stays off the GPU.  The peer-memory ring
                # inside TP is the product path and matched the single-GPU model.
                raise NotImplementedError("cp_mode='ring' with the NCCL transport inside tensor parallelism is "
                                          "disabled on CUDA; use the fused (peer-memory) transport")
            return (ring.PeerRing if fused else ring.CollectiveRing)(group, ranks, device)
        return (ring.PeerGatherKV if fused else ring.CollectiveGatherKV)(group, ranks, device)
    return (PeerUlysses if fused else CollectiveUlysses)(group, ranks, device)


def make_cfg_parallel(parallel, device, transport: str | None = None):
    """CFG-parallel context over the cfg axis (None when cfg-parallel is off)."""
    from difflet_b200.parallel import groups
    from difflet_b200.parallel.cfg import CollectiveCfg, PeerCfg

    if not parallel.cfg_parallel_enabled:
        return None
    if groups.mesh() != parallel.mesh_spec:
        groups.init_mesh(parallel.mesh_spec)
    group, ranks = groups.get_group("cfg"), groups.get_group_ranks("cfg")
    transport = transport or envs.DIFFLET_KERNEL_COMM
    if device.type == "cuda" and transport == "fused":
        return PeerCfg(group, ranks, device)
    return CollectiveCfg(group, ranks, device)
