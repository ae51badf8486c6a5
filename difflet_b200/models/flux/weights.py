"""FLUX checkpoint conversion (diffusers ``FluxTransformer2DModel`` <-> fused layout).

Thin names over the shared MMDiT converter in ``difflet_b200/models/mmdit/weights.py``.
"""

from difflet_b200.models.mmdit.weights import convert_diffusers, to_diffusers


def convert_diffusers_flux(cfg, sd):
    return convert_diffusers(cfg, sd)


def to_diffusers_state_dict(cfg, w):
    return to_diffusers(cfg, w)
