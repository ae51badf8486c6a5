"""CPU fake-quant oracle: an ``nn.Linear`` whose weight and input go through MXFP8
quantize -> dequantize (difflet/quant/fake_linear.py:28-130), so quality gates run on
CPU against the same law the tensor-core path uses."""

from __future__ import annotations

import re

import torch
import torch.nn as nn

from difflet_b200.ops.mx import dequantize_mx, quantize_mx


def fake_quant(x: torch.Tensor) -> torch.Tensor:
    q, s = quantize_mx(x.to(torch.bfloat16))
    return dequantize_mx(q, s, output_dtype=x.dtype)


class FakeQuantMXLinear(nn.Module):
    def __init__(self, linear: nn.Linear, quantize_input: bool = True):
        super().__init__()
        self.in_features, self.out_features = linear.in_features, linear.out_features
        self.weight = nn.Parameter(fake_quant(linear.weight.detach()), requires_grad=False)
        self.bias = linear.bias
        self.quantize_input = quantize_input

    def forward(self, x):
        if self.quantize_input:
            x = fake_quant(x.reshape(-1, x.shape[-1])).view(x.shape)
        return nn.functional.linear(x, self.weight.to(x.dtype), None if self.bias is None else self.bias.to(x.dtype))


def fake_quantize_model_(model: nn.Module, spec) -> list[str]:
    """Swap every ``nn.Linear`` the spec targets for its fake-quant twin; returns the names."""
    done = []
    for name, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            full = f"{name}.{cname}" if name else cname
            if isinstance(child, nn.Linear) and spec.matches(full):
                setattr(mod, cname, FakeQuantMXLinear(child))
                done.append(full)
    if not done:
        raise ValueError(f"no linear matches {list(spec.targets)}")
    return done


def split_pattern_names(names, patterns) -> list[str]:
    return [n for n in names if any(re.fullmatch(p, n) for p in patterns)]


__all__ = ["FakeQuantMXLinear", "fake_quant", "fake_quantize_model_"]
