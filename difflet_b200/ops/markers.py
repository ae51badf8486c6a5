"""Layer-boundary markers: identity modules (one tensor in -> that tensor; several -> the tuple).

Other hardware's ahead-of-time compilers read them as layer boundaries
(difflet/backends/cpu/ops_impl/markers.py); on B200 CUDA graphs need no hints."""

from torch import nn


class _Passthrough(nn.Module):
    def forward(self, *tensors):
        return tensors[0] if len(tensors) == 1 else tensors


class ModuleMarkerStartWrapper(_Passthrough):
    pass


class ModuleMarkerEndWrapper(_Passthrough):
    pass


__all__ = ["ModuleMarkerEndWrapper", "ModuleMarkerStartWrapper"]
