"""Mesh accessors and tensor- / sequence-parallel collectives of the public op surface.

Names and semantics of difflet/ops/collectives.py:4-80 and the per-backend
implementations (difflet/backends/neuron/ops_impl/collectives.py:115-368): every op
is the identity when its axis has one rank, so model code runs unchanged on one
GPU and on the CPU oracle.  Transfers go through ``torch.distributed`` (NCCL on
GPU, gloo on CPU); the built-in models' fused TP path (``parallel.tp``) moves the
same data inside its GEMM epilogues and norm kernels instead.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from difflet_b200.parallel import groups


class ParallelMeshNotInitializedError(RuntimeError):
    """A multi-rank op was called before ``init_parallel_mesh``."""


def init_parallel_mesh(spec=None, *, tp=1, cp=1, cfg=1, dp=1):
    """Create the {dp, cfg, cp, tp} groups (``spec``: a ``MeshSpec`` or a parallel config)."""
    from difflet_b200.parallel.mesh import MeshSpec

    if spec is None:
        spec = MeshSpec(dp=dp, cfg=cfg, cp=cp, tp=tp)
    elif hasattr(spec, "mesh_spec"):
        spec = spec.mesh_spec
    if spec.world_size > 1:
        groups.init_distributed()
    return groups.init_mesh(spec)


def _axis(axis):
    ranks = groups.get_group_ranks(axis)
    if len(ranks) == 1 or not dist.is_initialized():
        return None, 1, 0
    return groups.get_group(axis), len(ranks), ranks.index(dist.get_rank())


def get_tp_size() -> int:
    return _axis("tp")[1]


def get_tp_rank() -> int:
    return _axis("tp")[2]


get_tensor_model_parallel_size = get_tp_size
get_tensor_model_parallel_rank = get_tp_rank


def get_cp_group():
    return _axis("cp")[0]


def get_cfg_group():
    return _axis("cfg")[0]


def get_world_group():
    return dist.group.WORLD if dist.is_initialized() else None


def get_cp_rank_spmd() -> int:
    return _axis("cp")[2]


def get_cfg_rank_spmd() -> int:
    return _axis("cfg")[2]


class SPMDRank:
    """This rank's coordinates in the mesh (``.tp``, ``.cp``, ``.cfg``, ``.dp``, ``.rank``)."""

    def __init__(self):
        self.rank = groups.rank()
        m = groups.mesh()
        c = m.coords_of(self.rank) if m is not None else None
        for axis in ("dp", "cfg", "cp", "tp"):
            setattr(self, axis, getattr(c, axis) if c is not None else 0)

    def __repr__(self):
        return f"SPMDRank(rank={self.rank}, dp={self.dp}, cfg={self.cfg}, cp={self.cp}, tp={self.tp})"


def safe_tensor_parallel_size(get_size=get_tp_size) -> int:
    try:
        return int(get_size())
    except ParallelMeshNotInitializedError:
        return 1


# ----------------------------------------------------------------------------- TP collectives
def reduce_tp(tensor: torch.Tensor) -> torch.Tensor:
    """All-reduce (sum) over the tp group (row-parallel output)."""
    group, n, _ = _axis("tp")
    if n == 1:
        return tensor
    out = tensor.contiguous().clone()
    dist.all_reduce(out, group=group)
    return out


reduce_from_tensor_model_parallel_region = reduce_tp


def gather_tp_dim(tensor: torch.Tensor, *, dim: int) -> torch.Tensor:
    """All-gather the tp shards along ``dim``."""
    group, n, _ = _axis("tp")
    if n == 1:
        return tensor
    t = tensor.contiguous()
    parts = [torch.empty_like(t) for _ in range(n)]
    dist.all_gather(parts, t, group=group)
    return torch.cat(parts, dim)


def gather_from_tensor_model_parallel_region_with_dim(tensor, dim: int):
    return gather_tp_dim(tensor, dim=dim)


def scatter_tp_dim(tensor: torch.Tensor, *, dim: int) -> torch.Tensor:
    """This rank's slice along ``dim`` (no transfer: every rank holds the full tensor)."""
    _, n, r = _axis("tp")
    if n == 1:
        return tensor
    size = tensor.shape[dim]
    if size % n:
        raise ValueError(f"dim {dim} of size {size} does not split over tp={n}")
    return tensor.narrow(dim, r * (size // n), size // n).contiguous()


def scatter_to_tensor_model_parallel_region(tensor, dim: int = -1):
    return scatter_tp_dim(tensor, dim=dim)


def scatter_to_process_group_spmd(tensor, *, dim: int, group=None, rank=None, size=None):
    """Slice ``dim`` for ``rank`` of a group of ``size`` (defaults: the tp group)."""
    if size is None:
        _, size, rank = _axis("tp")
    if size == 1:
        return tensor
    n = tensor.shape[dim] // size
    return tensor.narrow(dim, rank * n, n).contiguous()


# ----------------------------------------------------------------------------- Megatron-SP
def scatter_to_sequence_parallel_region(tensor, *, dim: int):
    """Full sequence -> this rank's ``S/tp`` shard along ``dim``."""
    return scatter_tp_dim(tensor, dim=dim)


def gather_from_sequence_parallel_region(tensor, *, dim: int):
    """The SP ``g`` operator: all-gather the sequence shards along ``dim``."""
    return gather_tp_dim(tensor, dim=dim)


def reduce_scatter_to_sequence_parallel_region(tensor, *, dim: int):
    """The SP ``g-bar`` operator: reduce the row-parallel partial and keep this rank's shard."""
    group, n, _ = _axis("tp")
    if n == 1:
        return tensor
    t = tensor.movedim(dim, 0).contiguous()
    if t.shape[0] % n:
        raise ValueError(f"dim {dim} of size {t.shape[0]} does not split over tp={n}")
    parts = list(t.chunk(n, 0))
    out = torch.empty_like(parts[0])
    if dist.get_backend(group) == "gloo":  # gloo has no reduce_scatter
        full = t.clone()
        dist.all_reduce(full, group=group)
        out = full.chunk(n, 0)[_axis("tp")[2]].contiguous()
    else:
        dist.reduce_scatter(out, [p.contiguous() for p in parts], group=group)
    return out.movedim(0, dim)


__all__ = [
    "ParallelMeshNotInitializedError", "SPMDRank", "gather_from_sequence_parallel_region",
    "gather_from_tensor_model_parallel_region_with_dim", "gather_tp_dim", "get_cfg_group", "get_cfg_rank_spmd",
    "get_cp_group", "get_cp_rank_spmd", "get_tensor_model_parallel_rank", "get_tensor_model_parallel_size",
    "get_tp_rank", "get_tp_size", "get_world_group", "init_parallel_mesh", "reduce_from_tensor_model_parallel_region",
    "reduce_scatter_to_sequence_parallel_region", "reduce_tp", "safe_tensor_parallel_size", "scatter_to_process_group_spmd",
    "scatter_to_sequence_parallel_region", "scatter_to_tensor_model_parallel_region", "scatter_tp_dim",
]
