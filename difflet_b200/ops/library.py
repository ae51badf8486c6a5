"""The op surface as PyTorch dispatcher ops (``torch.ops.difflet.*``).

The reference exposes its ops as backend-neutral Python names (difflet/ops/__init__.py:3-69)
whose CUDA backend lowers to SDPA / NCCL (difflet/backends/cuda/ops_impl/attention.py:41-86).
Here the same contracts are registered once as ``torch.library`` custom ops in the
``difflet`` namespace, so that code holding only ``torch.ops`` (TorchScript-free graph
capture, FX passes, ``torch.compile`` fullgraph tracing, other frameworks' op tables) reaches
the sm_100a kernels: CUDA tensors run the native kernels through ``ops.fused``, CPU tensors
the PyTorch oracle of the same op.  Every op has a fake (meta) implementation for shape
propagation, and all are functional (outputs are new tensors).

Ops: ``attention``, ``linear`` (bias + optional GELU / SiLU on a column window),
``linear_gate_resid`` (``resid + gate * (x W^T + b)``), ``ln_modulate`` (LayerNorm / RMSNorm
with affine and per-batch shift / scale), ``rms_norm``, ``quantize_mx`` (OCP-MX E4M3 +
E8M0 per 32), ``linear_mx`` (block-scaled GEMM on quantized operands), ``gemv``.
"""

from __future__ import annotations

from typing import Optional

import torch

from difflet_b200.ops import fused as F

_NS = "difflet"


@torch.library.custom_op(f"{_NS}::attention", mutates_args=())
def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
              bound_min: Optional[torch.Tensor] = None, bound_max: Optional[torch.Tensor] = None) -> torch.Tensor:
    """softmax(scale q k^T) v over [B, H, S, D] (or folded [H, S, D]); optional per-batch key
    window [bound_min, bound_max)."""
    from difflet_b200.ops.attn import attention as _attention

    return _attention(q, k, v, scale=scale, bound_min=bound_min, bound_max=bound_max)


@attention.register_fake
def _(q, k, v, scale, bound_min=None, bound_max=None):
    return q.new_empty(q.shape[:-1] + (v.shape[-1],))


@torch.library.custom_op(f"{_NS}::linear", mutates_args=())
def linear(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor] = None, act: str = "none",
           act_lo: int = 0, act_hi: int = -1) -> torch.Tensor:
    """act(x W^T + b) with ``act`` in {none, gelu (tanh), silu} on columns [act_lo, act_hi)."""
    N = w.shape[0]
    y = F.linear(x.reshape(-1, x.shape[-1]), w, b, act=None if act == "none" else act, act_lo=act_lo,
                 act_hi=N if act_hi < 0 else act_hi)
    return y.reshape(x.shape[:-1] + (N,))


@linear.register_fake
def _(x, w, b=None, act="none", act_lo=0, act_hi=-1):
    return x.new_empty(x.shape[:-1] + (w.shape[0],))


@torch.library.custom_op(f"{_NS}::linear_gate_resid", mutates_args=())
def linear_gate_resid(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor], gate: torch.Tensor,
                      resid: torch.Tensor, rows_per_batch: int = 0) -> torch.Tensor:
    """resid + gate[batch] * (x W^T + b); gate f32 [B, N], rows_per_batch rows per batch."""
    N = w.shape[0]
    out = resid.reshape(-1, N).clone()
    F.linear(x.reshape(-1, x.shape[-1]), w, b, out=out, gate=gate.float().contiguous(), resid=out,
             rows_per_batch=rows_per_batch)
    return out.reshape(resid.shape)


@linear_gate_resid.register_fake
def _(x, w, b, gate, resid, rows_per_batch=0):
    return torch.empty_like(resid)


@torch.library.custom_op(f"{_NS}::ln_modulate", mutates_args=())
def ln_modulate(x: torch.Tensor, shift: Optional[torch.Tensor] = None, scale: Optional[torch.Tensor] = None,
                w: Optional[torch.Tensor] = None, b: Optional[torch.Tensor] = None, eps: float = 1e-6,
                rms: bool = False, rows_per_batch: int = 0) -> torch.Tensor:
    """norm(x) * w + b, then * (1 + scale[batch]) + shift[batch] (f32 statistics)."""
    d = x.shape[-1]
    y = F.ln_modulate(x.reshape(-1, d), shift=shift, scale=scale, w=w, b=b, eps=eps, rms=rms,
                      rows_per_batch=rows_per_batch)
    return y.reshape(x.shape)


@ln_modulate.register_fake
def _(x, shift=None, scale=None, w=None, b=None, eps=1e-6, rms=False, rows_per_batch=0):
    return torch.empty_like(x)


@torch.library.custom_op(f"{_NS}::rms_norm", mutates_args=())
def rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    """RMSNorm over the last dim with fp32 statistics and affine."""
    from difflet_b200.ops.norm import rms_norm_fp32

    return rms_norm_fp32(x, weight, eps)


@rms_norm.register_fake
def _(x, weight, eps):
    return torch.empty_like(x)


@torch.library.custom_op(f"{_NS}::quantize_mx", mutates_args=())
def quantize_mx(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[M, K] -> (E4M3 data [M, K], E8M0 scales [M, K / 32], plain layout)."""
    q, s = F.mx_quantize(x, blocked=False)
    return q, s


@quantize_mx.register_fake
def _(x):
    M, K = x.shape
    return x.new_empty((M, K), dtype=torch.float8_e4m3fn), x.new_empty((M, K // 32), dtype=torch.uint8)


@torch.library.custom_op(f"{_NS}::linear_mx", mutates_args=())
def linear_mx(aq: torch.Tensor, a_sf: torch.Tensor, bq: torch.Tensor, b_sf: torch.Tensor,
              bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16 (A_q * 2^a_sf) (B_q * 2^b_sf)^T + bias on OCP-MX operands (plain scale layout)."""
    M, K = aq.shape
    if aq.is_cuda:
        return F.linear_mx(aq, F.block_scales(a_sf), bq, F.block_scales(b_sf), bias)
    from difflet_b200.ops.mx import dequantize_mx

    a = dequantize_mx(aq, a_sf, output_dtype=torch.float32)
    b = dequantize_mx(bq, b_sf, output_dtype=torch.float32)
    y = a @ b.t()
    if bias is not None:
        y = y + bias.float()
    return y.to(torch.bfloat16)


@linear_mx.register_fake
def _(aq, a_sf, bq, b_sf, bias=None):
    return aq.new_empty((aq.shape[0], bq.shape[0]), dtype=torch.bfloat16)


@torch.library.custom_op(f"{_NS}::gemv", mutates_args=())
def gemv(W: torch.Tensor, x: torch.Tensor, bias: Optional[torch.Tensor] = None, silu_in: bool = False,
         silu_out: bool = False) -> torch.Tensor:
    """[B, K] x W[N, K]^T (+ bias), optional SiLU on the input and / or output (adaLN vectors)."""
    return F.gemv(W, x, bias, silu_in=silu_in, silu_out=silu_out)


@gemv.register_fake
def _(W, x, bias=None, silu_in=False, silu_out=False):
    return x.new_empty((x.shape[0], W.shape[0]), dtype=torch.float64 if x.dtype == torch.float64 else torch.float32)


OPS = ("attention", "linear", "linear_gate_resid", "ln_modulate", "rms_norm", "quantize_mx", "linear_mx", "gemv")

__all__ = list(OPS)
