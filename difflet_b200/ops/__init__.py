"""The public op surface model code is written against (names of difflet/ops/__init__.py:3-69).

One implementation per op for B200 (sm_100a kernels in ``csrc/`` through
``ops.fused``) plus the PyTorch oracle that CPU tensors take; no backend dispatch.
Attributes load lazily so ``import difflet_b200.ops`` stays light.
"""

_EXPORTS = {
    "ColumnParallelLinear": "linear",
    "RowParallelLinear": "linear",
    "ParallelEmbedding": "linear",
    "LayerNorm": "norm",
    "RMSNorm": "norm",
    "CustomRMSNorm": "norm",
    "rms_norm_fp32": "norm",
    "attention": "attn",
    "cross_attention": "attn",
    "ring_attention": "attn",
    "joint_ring_attention": "attn",
    "ulysses_attention": "attn",
    "joint_ulysses_attention": "attn",
    "apply_rotary_emb": "embeddings",
    "apply_rotary_emb_fp32": "embeddings",
    "apply_rotary_emb_slices": "embeddings",
    "ModuleMarkerStartWrapper": "markers",
    "ModuleMarkerEndWrapper": "markers",
    "quantize_mx": "mx",
    "dequantize_mx": "mx",
    "matmul_mx": "mx",
    "linear_mx": "mx",
    "SPMDRank": "collectives",
    "init_parallel_mesh": "collectives",
    "get_cfg_group": "collectives",
    "get_cp_group": "collectives",
    "get_world_group": "collectives",
    "get_cfg_rank_spmd": "collectives",
    "get_cp_rank_spmd": "collectives",
    "get_tp_rank": "collectives",
    "get_tp_size": "collectives",
    "get_tensor_model_parallel_rank": "collectives",
    "get_tensor_model_parallel_size": "collectives",
    "gather_tp_dim": "collectives",
    "reduce_tp": "collectives",
    "scatter_tp_dim": "collectives",
    "gather_from_tensor_model_parallel_region_with_dim": "collectives",
    "reduce_from_tensor_model_parallel_region": "collectives",
    "scatter_to_tensor_model_parallel_region": "collectives",
    "scatter_to_process_group_spmd": "collectives",
    "scatter_to_sequence_parallel_region": "collectives",
    "gather_from_sequence_parallel_region": "collectives",
    "reduce_scatter_to_sequence_parallel_region": "collectives",
    "get_platform_target": "platform",
    "hardware": "platform",
}

__all__ = sorted(_EXPORTS)


def __getattr__(name: str):
    mod = _EXPORTS.get(name)
    if mod is None:
        raise AttributeError(f"module 'difflet_b200.ops' has no attribute {name!r}")
    import importlib

    return getattr(importlib.import_module(f"difflet_b200.ops.{mod}"), name)


def __dir__():
    return __all__
