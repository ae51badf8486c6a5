"""FLUX MMDiT configuration (reference: ``difflet/models/flux/dit_config.py``).

FLUX is one family of the shared MMDiT: see ``difflet_b200/models/mmdit/config.py``.
"""

from difflet_b200.models.mmdit.config import PRESETS, MMDiTConfig, get_config  # noqa: F401

FluxConfig = MMDiTConfig
