"""Debug aids on the GPU: the bounds-check build runs the real kernels without a guard firing,
and repeated forwards are bit-identical (no order-dependent reductions anywhere)."""

import hashlib
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_PROG = r"""
import torch
from difflet_b200 import _native
from difflet_b200.ops import fused as F
from difflet_b200.models.flux.config import get_config
from difflet_b200.models.flux.model import FluxTransformer, pack_latents
assert _native._ext_name().endswith("_bounds")
cfg = get_config("tiny128", heads=4, hidden=512)
m = FluxTransformer.random_init(cfg, device="cuda", dtype=torch.bfloat16, seed=3)
g = torch.Generator().manual_seed(0)
x = pack_latents(torch.randn(1, 16, 64, 64, generator=g)).cuda().bfloat16()
txt = torch.randn(1, 128, cfg.text_dim, generator=g).cuda().bfloat16()
pooled = torch.randn(1, cfg.pooled_dim, generator=g).cuda()
out = m(x, txt, pooled, torch.full((1,), 0.4, device="cuda"), torch.full((1,), 3.5, device="cuda"), img_hw=(32, 32))
q = torch.randn(1, 3, 4608, 128, device="cuda", dtype=torch.bfloat16)
F.attention(q, q, q, 0.088)
torch.cuda.synchronize()
_native.check_device_errors()
assert torch.isfinite(out.float()).all()
print("BOUNDS_OK")
"""


def test_bounds_check_build_runs_clean(native):
    from difflet_b200 import _native

    env = dict(os.environ, DIFFLET_BOUNDS_CHECK="1", PYTHONPATH=_ROOT)
    so = [p for p in os.listdir(_native.BUILD_DIR) if p.startswith("_difflet_C_bounds") and p.endswith(".so")]
    if not so:
        pytest.skip("bounds-check build not present (build with DIFFLET_BOUNDS_CHECK=1)")
    r = subprocess.run([sys.executable, "-c", _PROG], env=env, capture_output=True, text=True, timeout=600)
    assert "BOUNDS_OK" in r.stdout, r.stdout[-2000:] + r.stderr[-3000:]


def test_repeat_forward_bit_identical(native):
    from difflet_b200.models.flux.config import get_config
    from difflet_b200.models.flux.model import FluxTransformer, pack_latents

    cfg = get_config("tiny128", heads=4, hidden=512)
    m = FluxTransformer.random_init(cfg, device="cuda", dtype=torch.bfloat16, seed=5)
    g = torch.Generator().manual_seed(1)
    x = pack_latents(torch.randn(1, 16, 64, 64, generator=g)).cuda().bfloat16()
    txt = torch.randn(1, 128, cfg.text_dim, generator=g).cuda().bfloat16()
    pooled = torch.randn(1, cfg.pooled_dim, generator=g).cuda()
    t, gd = torch.full((1,), 0.4, device="cuda"), torch.full((1,), 3.5, device="cuda")
    hashes = set()
    for _ in range(3):
        out = m(x, txt, pooled, t, gd, img_hw=(32, 32))
        torch.cuda.synchronize()
        hashes.add(hashlib.sha256(out.cpu().view(torch.int16).numpy().tobytes()).hexdigest())
    assert len(hashes) == 1
