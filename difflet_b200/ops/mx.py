"""Microscaling (MXFP8) ops of the public op surface (difflet/ops/mx.py:10-87).

Format (OCP Microscaling Formats v1.0, the published spec): elements FP8 E4M3
(or E5M2), one shared E8M0 scale per ``group_size`` = 32 consecutive values along
the last (reduction) dimension.  For a block with largest magnitude ``amax`` the
scale exponent is ``floor(log2(amax)) - emax_elem`` (emax 8 for E4M3, 15 for
E5M2), stored biased by 127; elements are ``x / 2^e`` rounded to the FP8 type with
saturation at its largest normal (448 / 57344).  An all-zero block takes the
smallest exponent.  The block law (largest binade minus the element format's)
is the reference's (difflet/backends/cpu/ops_impl/mx.py:15-88); the block
membership is B200's: 32 contiguous K values, the unit of the block-scaled
tensor-core MMA, where the reference uses Trainium's 8 x 4 swizzled blocks.
The reference packs four FP8 values per ``uint32`` ("_x4"); here data stays
``torch.float8_*`` and the "_x4" names are accepted as aliases.

Layouts: ``data [..., K]`` FP8, ``scale [..., K / 32]`` uint8 (biased exponent).
``matmul_mx(a, sa, b, sb)`` = ``A @ B^T`` with both operands K-major (``b`` is a
Linear weight ``[N, K]``); ``linear_mx(x, w_k_n, bias)`` keeps the reference's
``[K, N]`` weight argument.
"""

from __future__ import annotations

import torch

GROUP = 32
BIAS = 127
# name -> (emax of the element format, largest finite value, torch dtype)
_FORMATS = {
    "float8_e4m3fn": (8, 448.0, torch.float8_e4m3fn),
    "float8_e5m2": (15, 57344.0, torch.float8_e5m2),
}


def _fmt(dtype: str):
    name = dtype[:-3] if dtype.endswith("_x4") else dtype
    if name not in _FORMATS:
        raise NotImplementedError(f"MX element type {dtype!r}: one of {sorted(_FORMATS)} (or their _x4 names)")
    return _FORMATS[name]


def _check_group(group_size: int):
    if group_size != GROUP:
        raise NotImplementedError(f"MX group size is {GROUP} (the tensor-core block), got {group_size}")


def _floor_log2(a: torch.Tensor) -> torch.Tensor:
    """floor(log2(a)) for a > 0 read from the fp32 exponent field (exact; subnormals -> -127)."""
    bits = a.to(torch.float32).view(torch.int32)
    return ((bits >> 23) & 0xFF) - BIAS


def quantize_mx(x: torch.Tensor, *, dtype: str = "float8_e4m3fn", group_size: int = GROUP):
    """bf16 / fp16 / fp32 ``[..., K]`` -> (FP8 data ``[..., K]``, uint8 E8M0 scales ``[..., K/32]``)."""
    emax, vmax, fp8 = _fmt(dtype)
    _check_group(group_size)
    K = x.shape[-1]
    if K % GROUP:
        raise ValueError(f"quantize_mx needs the last dim to be a multiple of {GROUP}, got {K}")
    if x.is_cuda and x.dtype == torch.bfloat16 and fp8 == torch.float8_e4m3fn and x.is_contiguous():
        return _native_quant(x)
    blocks = x.to(torch.float32).reshape(*x.shape[:-1], K // GROUP, GROUP)
    amax = blocks.abs().amax(-1)
    e = torch.where(amax > 0, _floor_log2(amax) - emax, torch.full_like(amax, -BIAS, dtype=torch.int32))
    e = e.clamp(-BIAS, BIAS)
    scale = (e + BIAS).to(torch.uint8)
    q = torch.clamp(blocks * torch.pow(2.0, -e.to(torch.float32))[..., None], -vmax, vmax)
    return q.reshape(x.shape).to(fp8), scale


def _native_quant(x: torch.Tensor):
    from difflet_b200.ops import fused as F

    K = x.shape[-1]
    data, scale = F.native().mx_quantize(x.reshape(-1, K))
    return data.view(*x.shape), scale.view(*x.shape[:-1], K // GROUP)


def dequantize_mx(data, scale, *, dtype: str = "float8_e4m3fn", output_dtype=torch.bfloat16,
                  group_size: int = GROUP):
    _fmt(dtype)
    _check_group(group_size)
    K = data.shape[-1]
    if scale.dtype != torch.uint8 or scale.shape != (*data.shape[:-1], K // GROUP):
        raise ValueError(f"scale must be uint8 {(*data.shape[:-1], K // GROUP)}, got {scale.dtype} "
                         f"{tuple(scale.shape)}")
    s = torch.pow(2.0, scale.to(torch.float32) - BIAS)
    v = data.to(torch.float32).reshape(*data.shape[:-1], K // GROUP, GROUP) * s[..., None]
    return v.reshape(data.shape).to(output_dtype)


def matmul_mx(a_mx, a_scale, b_mx, b_scale, *, dtype: str = "float8_e4m3fn", out_dtype=torch.bfloat16,
              accumulate: bool = False, group_size: int = GROUP, out=None, bias=None):
    """``A @ B^T`` from MX operands (A ``[M, K]``, B ``[N, K]``); ``accumulate`` adds into ``out``."""
    _fmt(dtype)
    _check_group(group_size)
    if (a_mx.is_cuda and a_mx.dtype == torch.float8_e4m3fn and b_mx.dtype == torch.float8_e4m3fn
            and a_mx.shape[-1] % 128 == 0):
        from difflet_b200.ops import fused as F

        M, N = a_mx.shape[0], b_mx.shape[0]
        if accumulate and out is None:
            raise ValueError("accumulate=True needs out")
        return F.linear_mx(a_mx, F.block_scales(a_scale), b_mx, F.block_scales(b_scale), bias=bias, out=out,
                           accumulate=accumulate, out_dtype=out_dtype if out is None else out.dtype)
    a = dequantize_mx(a_mx, a_scale, dtype=dtype, output_dtype=torch.float32)
    b = dequantize_mx(b_mx, b_scale, dtype=dtype, output_dtype=torch.float32)
    y = a @ b.t()
    if bias is not None:
        y = y + bias.to(y.dtype)
    if accumulate:
        if out is None:
            raise ValueError("accumulate=True needs out")
        y = y + out.to(y.dtype)
    if out is not None:
        out.copy_(y.to(out.dtype))
        return out
    return y.to(out_dtype)


def linear_mx(input_bf16, weight_k_n_bf16, bias_bf16=None, *, dtype: str = "float8_e4m3fn",
              out_dtype=torch.bfloat16, group_size: int = GROUP):
    """A Linear evaluated in MXFP8: both operands quantized along K, fp32 accumulation."""
    x = input_bf16.reshape(-1, input_bf16.shape[-1])
    xq, xs = quantize_mx(x, dtype=dtype, group_size=group_size)
    wq, ws = quantize_mx(weight_k_n_bf16.t().contiguous(), dtype=dtype, group_size=group_size)
    y = matmul_mx(xq, xs, wq, ws, dtype=dtype, out_dtype=out_dtype, bias=bias_bf16)
    return y.view(*input_bf16.shape[:-1], y.shape[-1])


__all__ = ["dequantize_mx", "linear_mx", "matmul_mx", "quantize_mx"]
