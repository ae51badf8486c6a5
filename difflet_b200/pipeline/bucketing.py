"""Shape-set canonicalisation for multi-shape applications (reference ``difflet/pipeline/bucketing.py:52-65``)."""

from difflet_b200.pipeline.compile_cache import canonicalize_shapes  # noqa: F401


def parse_shapes(spec: str) -> list[tuple]:
    """``"1024x1024,768x1344"`` or ``"720x1280x81"`` -> [(h, w, frames|None), ...]."""
    out = []
    for part in spec.split(","):
        nums = [int(x) for x in part.lower().split("x") if x]
        if len(nums) not in (2, 3):
            raise ValueError(f"bad shape {part!r}")
        out.append(tuple(nums) + ((None,) if len(nums) == 2 else ()))
    return canonicalize_shapes(out)
