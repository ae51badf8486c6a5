"""Tensor-parallel linear layers of the public op surface (difflet/ops/linear.py; the NxD /
Megatron contracts of difflet/backends/cpu/ops_impl/linear.py and
difflet/backends/_torch_megatron/linear.py).

``ColumnParallelLinear``: this rank holds ``output_size / tp`` rows of W (and of b);
``gather_output=True`` all-gathers the output columns.  With
``sequence_parallel_enabled`` the input arrives sequence-sharded (dim
``sequence_dimension``) and is all-gathered first (SP ``g``).

``RowParallelLinear``: this rank holds ``input_size / tp`` columns of W; the partial
products are all-reduced (or reduce-scattered along the sequence with SP, ``g-bar``);
``skip_bias_add=True`` returns ``(y, bias)``.

At tp = 1 both are plain linears.  bf16 CUDA inputs run the tcgen05 GEMM.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as TF

from difflet_b200.ops import collectives as C
from difflet_b200.ops import fused as F


def _linear(x, w, b):
    if x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0:
        y = F.linear(x.reshape(-1, x.shape[-1]).contiguous(), w, b)
        return y.view(*x.shape[:-1], w.shape[0])
    return TF.linear(x, w, b)


class ColumnParallelLinear(nn.Module):
    def __init__(self, input_size, output_size, bias=True, gather_output=True, dtype=None, device=None,
                 sequence_parallel_enabled=False, sequence_dimension=0, **kwargs):
        super().__init__()
        del kwargs
        tp = C.safe_tensor_parallel_size()
        if output_size % tp:
            raise ValueError(f"output_size {output_size} does not split over tp={tp}")
        self.input_size, self.output_size, self.tp = input_size, output_size, tp
        self.gather_output = gather_output
        self.sequence_parallel_enabled = sequence_parallel_enabled
        self.sequence_dimension = sequence_dimension
        self.weight = nn.Parameter(torch.empty(output_size // tp, input_size, dtype=dtype, device=device))
        self.bias = nn.Parameter(torch.zeros(output_size // tp, dtype=dtype, device=device)) if bias else None
        nn.init.kaiming_uniform_(self.weight, a=5 ** 0.5)

    def forward(self, x):
        if self.sequence_parallel_enabled:
            x = C.gather_from_sequence_parallel_region(x, dim=self.sequence_dimension)
        y = _linear(x, self.weight, self.bias)
        return C.gather_tp_dim(y, dim=-1) if self.gather_output else y


class RowParallelLinear(nn.Module):
    def __init__(self, input_size, output_size, bias=True, input_is_parallel=False, reduce_output=True,
                 skip_bias_add=False, dtype=None, device=None, sequence_parallel_enabled=False,
                 sequence_dimension=0, **kwargs):
        super().__init__()
        del kwargs
        tp = C.safe_tensor_parallel_size()
        if input_size % tp:
            raise ValueError(f"input_size {input_size} does not split over tp={tp}")
        self.input_size, self.output_size, self.tp = input_size, output_size, tp
        self.input_is_parallel = input_is_parallel
        self.reduce_output = reduce_output
        self.skip_bias_add = skip_bias_add
        self.sequence_parallel_enabled = sequence_parallel_enabled
        self.sequence_dimension = sequence_dimension
        self.tensor_parallel_group = C._axis("tp")[0]
        self.weight = nn.Parameter(torch.empty(output_size, input_size // tp, dtype=dtype, device=device))
        self.bias = nn.Parameter(torch.zeros(output_size, dtype=dtype, device=device)) if bias else None
        nn.init.kaiming_uniform_(self.weight, a=5 ** 0.5)

    def forward(self, x):
        if not self.input_is_parallel:
            x = C.scatter_tp_dim(x, dim=-1)
        y = _linear(x, self.weight, None)
        if self.reduce_output:
            if self.sequence_parallel_enabled:
                y = C.reduce_scatter_to_sequence_parallel_region(y, dim=self.sequence_dimension)
            else:
                y = C.reduce_tp(y)
        if self.skip_bias_add:
            return y, self.bias
        return y + self.bias.to(y.dtype) if self.bias is not None else y


class ParallelEmbedding(nn.Module):
    """Embedding table sharded over tp along the vocabulary (default) or, with
    ``shard_across_embedding``, along the embedding dim; the lookup is completed by an
    all-reduce (vocab shards) or an all-gather (dim shards)."""

    def __init__(self, num_embeddings, embedding_dim, shard_across_embedding=False, pad=False, dtype=None,
                 device=None, **kwargs):
        super().__init__()
        del kwargs
        tp = C.safe_tensor_parallel_size()
        self.tp, self.rank = tp, C.get_tp_rank()
        self.shard_across_embedding = shard_across_embedding
        self.num_embeddings, self.embedding_dim = num_embeddings, embedding_dim
        if shard_across_embedding:
            if embedding_dim % tp:
                raise ValueError(f"embedding_dim {embedding_dim} does not split over tp={tp}")
            shape = (num_embeddings, embedding_dim // tp)
        else:
            per = -(-num_embeddings // tp) if pad else num_embeddings // tp
            if not pad and num_embeddings % tp:
                raise ValueError(f"num_embeddings {num_embeddings} does not split over tp={tp} (use pad=True)")
            self.vocab_start = self.rank * per
            shape = (per, embedding_dim)
        self.weight = nn.Parameter(torch.empty(*shape, dtype=dtype, device=device))
        nn.init.normal_(self.weight)

    def forward(self, ids):
        if self.shard_across_embedding:
            return C.gather_tp_dim(TF.embedding(ids, self.weight), dim=-1)
        if self.tp == 1:
            return TF.embedding(ids, self.weight)
        local = ids - self.vocab_start
        valid = (local >= 0) & (local < self.weight.shape[0])
        out = TF.embedding(local.clamp(0, self.weight.shape[0] - 1), self.weight) * valid[..., None].to(
            self.weight.dtype)
        return C.reduce_tp(out)


__all__ = ["ColumnParallelLinear", "ParallelEmbedding", "RowParallelLinear"]
