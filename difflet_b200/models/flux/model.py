"""FLUX transformer = the shared sm_100a MMDiT with the FLUX config.

See ``difflet_b200/models/mmdit/model.py`` for the fused layout and kernels.
"""

from difflet_b200.models.mmdit.model import MMDiT, pack_latents, unpack_latents  # noqa: F401

FluxTransformer = MMDiT
