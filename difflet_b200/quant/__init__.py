"""MXFP8 quantization: recipe (``spec``), per-model targets, offline checkpoint,
fake-quant oracle and the application of a spec to a loaded model (``apply``)."""

from difflet_b200.quant.spec import QuantSpec, quant_cache_fields  # noqa: F401
from difflet_b200.quant.targets import default_spec  # noqa: F401
