"""Ulysses sequence parallelism on CPU gloo ranks: every rank's shard equals the dense forward."""

import pytest
import torch

from difflet_b200.parallel.testing import run_ranks

pytestmark = pytest.mark.multirank


def _sp_forward(rank, world, B):
    import torch.distributed as dist

    from difflet_b200.models.flux.config import get_config
    from difflet_b200.models.flux.model import FluxTransformer, pack_latents
    from difflet_b200.parallel.ulysses import CollectiveUlysses

    cfg = get_config("tiny128", heads=4, hidden=512)
    m = FluxTransformer.random_init(cfg, dtype=torch.float64, seed=11)
    g = torch.Generator().manual_seed(0)
    x = pack_latents(torch.randn(B, 16, 32, 32, generator=g, dtype=torch.float64))
    txt = torch.randn(B, 64, cfg.text_dim, generator=g, dtype=torch.float64)
    pooled = torch.randn(B, cfg.pooled_dim, generator=g, dtype=torch.float64)
    t = torch.full((B,), 0.4, dtype=torch.float64)
    gd = torch.full((B,), 3.5, dtype=torch.float64)
    dense = m(x, txt, pooled, t, gd, img_hw=(16, 16))
    par = CollectiveUlysses(dist.group.WORLD, list(range(world)), torch.device("cpu"))
    m2 = FluxTransformer(cfg, m.w)
    m2.par = par
    out = m2(par.shard_tokens(x), par.shard_tokens(txt), pooled, t, gd, img_hw=(16, 16))
    full = par.gather_tokens(out)
    return (full - dense).abs().max().item()


@pytest.mark.parametrize("world,B", [(2, 1), (4, 1), (2, 2)])
def test_ulysses_matches_dense(world, B):
    errs = run_ranks(_sp_forward, world, B, timeout=240)
    assert max(errs) < 1e-10, errs
