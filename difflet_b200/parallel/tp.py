"""Tensor parallelism for the MMDiT families and Wan (Megatron column / row split).

Column-parallel linears (q/k/v, MLP up, FLUX's single-block [q|mlp|k|v]) hold this
rank's heads / MLP columns and need no communication; attention runs on the local
heads over the whole sequence.  Row-parallel linears (attention output, MLP down,
single-block ``proj_out`` over [attn|mlp]) produce partial sums that must be
reduced; the B200 path fuses that reduction with the GEMM:

``PeerTP.row_linear`` (peer memory)
    1. the tcgen05 GEMM's epilogue stores each partial row straight into the
       symmetric slot buffer of the rank that owns the row (row scatter over
       NVLink, overlapped with the GEMM's remaining tiles);
    2. device barrier;
    3. ``tp_reduce`` on the owner sums the tp partials in a fixed order (fp32,
       deterministic), adds the bias and the gated residual, and stores the
       finished rows into every rank's residual stream (the all-gather half of
       the all-reduce is its store pattern);
    4. device barrier.
``CollectiveTP.row_linear``: GEMM, ``all_reduce`` (NCCL / gloo), epilogue in
torch -- the baseline and the CPU multi-rank oracle.

Reference semantics: ColumnParallelLinear / RowParallelLinear and the TP
collectives (difflet/backends/neuron/ops_impl/collectives.py:115-200), FLUX's
merged single-block all-reduce (difflet/models/flux/modeling_flux.py:723-727),
TP-aware q/k norms; the TPU collective-matmul design precedent
(difflet/backends/tpu/ops_impl/collective_matmul.py:14-17).
"""

from __future__ import annotations


import torch
import torch.distributed as dist

from difflet_b200.ops import fused as F
from difflet_b200.parallel.ulysses import PeerBase, _Base


def _cols(t, lo, hi):
    return t[:, lo:hi]


def shard_mmdit_weights(cfg, w: dict, tp: int, rank: int) -> dict:
    """This rank's slices of an MMDiT's fused weights (heads, MLP columns, K ranges)."""
    if tp == 1:
        return dict(w)
    D, F_, H = cfg.hidden, cfg.mlp_hidden, cfg.heads
    if H % tp or F_ % tp:
        raise ValueError(f"tensor parallelism needs heads ({H}) and MLP width ({F_}) divisible by tp={tp}")
    Dl, Fl = D // tp, F_ // tp
    d0, d1, f0, f1 = rank * Dl, (rank + 1) * Dl, rank * Fl, (rank + 1) * Fl
    out = {}
    for k, t in w.items():
        if k.startswith("ref."):
            out[k] = t  # the token refiner runs replicated
        elif k.endswith("_qkv.w") or k.endswith("_qkv.b"):
            parts = t.split(D, 0)
            out[k] = torch.cat([p[d0:d1] for p in parts], 0).contiguous()
        elif k.endswith("_out.w"):
            out[k] = t[:, d0:d1].contiguous()
        elif k.endswith("_up.w") or k.endswith("_up.b"):
            out[k] = t[f0:f1].contiguous()
        elif k.endswith("_down.w"):
            out[k] = t[:, f0:f1].contiguous()
        elif k.endswith("fused.w") or k.endswith("fused.b"):
            q, m, kk, v = t.split([D, F_, D, D], 0)
            out[k] = torch.cat([q[d0:d1], m[f0:f1], kk[d0:d1], v[d0:d1]], 0).contiguous()
        elif k.endswith("proj.w") and k.startswith("single."):
            out[k] = torch.cat([t[:, d0:d1], t[:, D + f0:D + f1]], 1).contiguous()
        else:
            out[k] = t  # replicated: embedders, norms, modulation, final layer, refiner
    return out


def shard_wan_weights(cfg, w: dict, tp: int, rank: int) -> dict:
    """This rank's slices of a Wan transformer's weights: q/k/v, cross-attention q and k/v,
    the MLP up projection and the across-heads q/k norm weights by heads / columns
    (column-parallel); the attention / cross-attention outputs and MLP down by K
    (row-parallel, bias added once by the reducer); everything else replicated."""
    if tp == 1:
        return dict(w)
    D, Fh, H = cfg.hidden, cfg.ffn, cfg.heads
    if H % tp or Fh % tp:
        raise ValueError(f"tensor parallelism needs heads ({H}) and FFN width ({Fh}) divisible by tp={tp}")
    Dl, Fl = D // tp, Fh // tp
    d0, d1, f0, f1 = rank * Dl, (rank + 1) * Dl, rank * Fl, (rank + 1) * Fl
    out = {}
    for k, t in w.items():
        name = k.rsplit(".", 2)[-2:] if k.startswith("blk.") else None
        leaf = ".".join(name) if name else k
        if not k.startswith("blk."):
            out[k] = t
        elif leaf in ("qkv.w", "qkv.b", "ckv.w", "ckv.b"):
            out[k] = torch.cat([p[d0:d1] for p in t.split(D, 0)], 0).contiguous()
        elif leaf in ("cq.w", "cq.b") or k.endswith((".qn", ".kn", ".cqn", ".ckn")):
            out[k] = t[d0:d1].contiguous()
        elif leaf in ("up.w", "up.b"):
            out[k] = t[f0:f1].contiguous()
        elif leaf in ("o.w", "co.w"):
            out[k] = t[:, d0:d1].contiguous()
        elif leaf == "down.w":
            out[k] = t[:, f0:f1].contiguous()
        else:
            out[k] = t  # output biases (added once by the reducer), norm affine
    return out


class _TPBase(_Base):
    kind = "tp"
    sp = False  # Megatron sequence parallelism: residual rows sharded, AG in the norm, RS in the reducer

    def heads_local(self, H):
        return H // self.world

    def row_range(self, M: int):
        rpr = -(-M // self.world)
        r0 = self.rank * rpr
        return r0, max(0, min(rpr, M - r0))


class PeerTP(_TPBase, PeerBase):
    def __init__(self, group, ranks, device):
        super().__init__(group, ranks, device)
        self._slots = {}

    def slots(self, rpr: int, N: int, dtype) -> torch.Tensor:
        key = (N, dtype)
        cur = self._slots.get(key)
        if cur is None or cur.shape[0] < self.world * rpr:
            if cur is not None:
                self.heap.retire(cur)  # the peers still map the smaller buffer
            cur = self.heap.empty((self.world * rpr, N), dtype)
            self._slots[key] = cur
        return cur

    def row_linear(self, x, w, b=None, *, out, gate=None, resid=None, rows_per_batch=0):
        """out[rows] = (resid + gate *) (sum over tp of x_r W_r^T + b); ``out`` / ``resid``
        are replicated (symmetric-heap) row buffers of the same rows as ``x``."""
        M, N = x.shape[0], w.shape[0]
        W, r = self.world, self.rank
        rpr = -(-M // W)
        slots = self.slots(rpr, N, torch.bfloat16)
        nat = F.native()
        peers = self.heap.peer_ptrs(slots)
        if isinstance(w, F.MXWeight):
            xq, xs = F.mx_quantize(x, blocked=True)
            nat.gemm_mx(xq, xs, w.q, w.sf, None, None, 0, out_peer=peers, rows_per_rank=rpr, peer_row_off=r * rpr,
                        ldd=N)
        else:
            nat.gemm(x, w, None, None, 0, out_peer=peers, rows_per_rank=rpr, peer_row_off=r * rpr, ldd=N)
        self.heap.barrier()  # every partial of this rank's rows has landed
        rows = max(0, min(rpr, M - r * rpr))
        # all-reduce: the finished rows go to every rank; sequence parallel: only to this rank (reduce-scatter)
        dst = [out.data_ptr()] if self.sp else self.heap.peer_ptrs(out)
        nat.tp_reduce(slots, rpr, W, rows, N, r * rpr, b, gate, rows_per_batch if gate is not None else 0,
                      resid if gate is not None else None, dst, out.stride(0), r * rpr)
        self.heap.barrier()  # the slots are free again (and, all-reduce, every row is everywhere)

    def allreduce_rows(self, t: torch.Tensor) -> torch.Tensor:
        """In-place sum over the tp ranks of a small f32 tensor (per-row partial statistics):
        each rank stores its copy into slot ``rank`` of every rank's symmetric buffer, one
        device barrier, then every rank adds the slots in rank order (identical results).
        Two alternating buffers make one barrier per call enough."""
        n = t.numel()
        key = ("ar", n)
        bufs = self._slots.get(key)
        if bufs is None:
            bufs = self._slots[key] = [self.heap.empty((self.world, n), torch.float32) for _ in range(2)]
            self._ar_turn = 0
        buf = bufs[self._ar_turn]
        self._ar_turn ^= 1
        F.native().peer_put_f32(t.reshape(-1), self.heap.peer_ptrs(buf), self.rank * n)
        self.heap.barrier()
        torch.sum(buf, 0, out=t.view(-1))
        return t

    def ln_gather(self, x, out, **kw):
        """Sequence-parallel norm: this rank normalises its own rows of ``x`` and stores them
        into every rank's ``out`` (the all-gather is the kernel's store pattern)."""
        r0, n = self.row_range(x.shape[0])
        F.ln_modulate(x, out=out, y_peer=self.heap.peer_ptrs(out), row0=r0, rows=n, **kw)
        self.heap.barrier()
        return out

    def sync_rows(self, x):
        """Copy this rank's own rows of ``x`` (a symmetric buffer) into every rank's copy."""
        r0, n = self.row_range(x.shape[0])
        if n:
            src = x[r0:r0 + n]
            nb = n * x.stride(0) * x.element_size()
            for r, p in enumerate(self.heap.peer_ptrs(src)):
                if r != self.rank:
                    F.native().memcpy_async(p, src.data_ptr(), nb)
        self.heap.barrier()


class CollectiveTP(_TPBase):
    """Row-parallel reduction by ``all_reduce`` (NCCL on GPU, gloo on CPU)."""

    def empty(self, shape, dtype):
        return torch.zeros(shape, dtype=dtype, device=self.device)

    def peer_views(self, t):
        return [t]

    def ln_gather(self, x, out, **kw):
        r0, n = self.row_range(x.shape[0])
        y = F.ln_modulate(x, **kw)
        parts = [torch.empty_like(y) for _ in range(self.world)]
        dist.all_gather(parts, y.contiguous(), group=self.group)
        for r in range(self.world):  # rank r's rows come from its copy (the rows it owns)
            rr0 = r * -(-x.shape[0] // self.world)
            rn = max(0, min(-(-x.shape[0] // self.world), x.shape[0] - rr0))
            out[rr0:rr0 + rn] = parts[r][rr0:rr0 + rn]
        return out

    def sync_rows(self, x):
        r0, n = self.row_range(x.shape[0])
        parts = [torch.empty_like(x) for _ in range(self.world)]
        dist.all_gather(parts, x.contiguous(), group=self.group)
        M = x.shape[0]
        rpr = -(-M // self.world)
        for r in range(self.world):
            x[r * rpr:min(M, (r + 1) * rpr)] = parts[r][r * rpr:min(M, (r + 1) * rpr)]

    def allreduce_rows(self, t: torch.Tensor) -> torch.Tensor:
        dist.all_reduce(t, group=self.group)
        return t

    def row_linear(self, x, w, b=None, *, out, gate=None, resid=None, rows_per_batch=0):
        if isinstance(w, F.MXWeight):
            w = w.dequantize()
        ct = torch.float64 if x.dtype == torch.float64 else torch.float32
        y = x.to(ct) @ w.to(ct).t()
        dist.all_reduce(y, group=self.group)
        if b is not None:
            y = y + b.to(ct)
        if gate is not None:
            M = y.shape[0]
            rpb = rows_per_batch if rows_per_batch > 0 else M
            y = resid.to(ct) + gate[:, : y.shape[1]].to(ct).repeat_interleave(rpb, 0)[:M] * y
        out.copy_(y.to(out.dtype))
        return out


def make_tensor_parallel(parallel, device, transport: str | None = None):
    ctx = _make_tp(parallel, device, transport)
    if ctx is not None:
        ctx.sp = bool(getattr(parallel, "sp_enabled", False))
    return ctx


def _make_tp(parallel, device, transport):
    """TP context over the tp axis (None when tp_degree == 1)."""
    from difflet_b200 import envs
    from difflet_b200.parallel import groups

    if parallel.tp_degree == 1:
        return None
    if not dist.is_initialized():
        raise RuntimeError("tensor parallelism needs an initialised process group (run under torchrun)")
    if groups.mesh() != parallel.mesh_spec:
        groups.init_mesh(parallel.mesh_spec)
    group, ranks = groups.get_group("tp"), groups.get_group_ranks("tp")
    transport = transport or envs.DIFFLET_KERNEL_COMM
    if device.type == "cuda" and transport == "fused":
        return PeerTP(group, ranks, device)
    return CollectiveTP(group, ranks, device)


__all__ = ["CollectiveTP", "PeerTP", "make_tensor_parallel", "shard_mmdit_weights", "shard_wan_weights"]
