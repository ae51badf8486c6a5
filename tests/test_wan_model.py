"""Wan DiT: fused layout vs the straight-line oracle (float64), and Ulysses on gloo ranks."""

import pytest
import torch

from difflet_b200.models.wan.model import WanTransformer, get_wan_config, patchify, unpatchify
from difflet_b200.models.wan.weights import convert_diffusers_wan, to_diffusers_wan
from difflet_b200.oracle.wan_reference import wan_forward


def _inputs(cfg, B=1, dtype=torch.float64):
    g = torch.Generator().manual_seed(0)
    lat = torch.randn(B, 16, 3, 8, 12, generator=g, dtype=dtype)
    text = torch.randn(B, cfg.text_len, cfg.text_dim, generator=g, dtype=dtype)
    return lat, text


def test_wan_roundtrip_and_patchify():
    cfg = get_wan_config("tiny-wan")
    m = WanTransformer.random_init(cfg, dtype=torch.float32)
    w2 = convert_diffusers_wan(cfg, to_diffusers_wan(cfg, m.w))
    assert set(w2) == set(m.w) and all(torch.equal(w2[k], m.w[k].to(w2[k].dtype)) for k in w2)
    lat = torch.randn(2, 16, 3, 8, 12)
    assert torch.equal(unpatchify(patchify(lat), (3, 4, 6)), lat)


@pytest.mark.parametrize("B", [1, 2])
def test_wan_fused_matches_oracle(B):
    cfg = get_wan_config("tiny-wan")
    m = WanTransformer.random_init(cfg, dtype=torch.float64, seed=4)
    sd = to_diffusers_wan(cfg, m.w)
    sd = {k: v.double() for k, v in sd.items()}
    lat, text = _inputs(cfg, B)
    x = patchify(lat)
    t = torch.tensor([700.0, 20.0][:B], dtype=torch.float64)
    grid = (3, 4, 6)
    ctx = m.prepare_context(text)
    out = m(x, t, ctx, grid=grid)
    ref = wan_forward(cfg, sd, x, t, text, grid)
    assert (out - ref).abs().max().item() < 1e-11 * ref.abs().max().item()


def _sp(rank, world, mode="ulysses"):
    import torch.distributed as dist

    from difflet_b200.parallel.ring import CollectiveGatherKV, CollectiveRing
    from difflet_b200.parallel.ulysses import CollectiveUlysses

    cfg = get_wan_config("tiny-wan", heads=4, hidden=512)
    m = WanTransformer.random_init(cfg, dtype=torch.float64, seed=5)
    lat, text = _inputs(cfg)
    x = patchify(lat)
    t = torch.tensor([500.0], dtype=torch.float64)
    ctx = m.prepare_context(text)
    dense = m(x, t, ctx, grid=(3, 4, 6))
    cls = {"ulysses": CollectiveUlysses, "ring": CollectiveRing, "gather_kv": CollectiveGatherKV}[mode]
    par = cls(dist.group.WORLD, list(range(world)), torch.device("cpu"))
    m2 = WanTransformer(cfg, m.w)
    m2.par = par
    out = par.gather_tokens(m2(par.shard_tokens(x), t, ctx, grid=(3, 4, 6)))
    return (out - dense).abs().max().item()


@pytest.mark.multirank
@pytest.mark.parametrize("mode", ["ulysses", "ring", "gather_kv"])
def test_wan_cp_matches_dense(mode):
    from difflet_b200.parallel.testing import run_ranks

    assert max(run_ranks(_sp, 2, mode, timeout=240)) < 1e-10


def _tp(rank, world):
    import torch.distributed as dist

    from difflet_b200.parallel.tp import CollectiveTP, shard_wan_weights

    cfg = get_wan_config("tiny-wan", heads=4, hidden=512, ffn=1024)
    m = WanTransformer.random_init(cfg, dtype=torch.float64, seed=6)
    lat, text = _inputs(cfg)
    x = patchify(lat)
    t = torch.tensor([500.0], dtype=torch.float64)
    dense = m(x, t, m.prepare_context(text), grid=(3, 4, 6))
    m2 = WanTransformer(cfg, shard_wan_weights(cfg, m.w, world, rank))
    m2.tp = CollectiveTP(dist.group.WORLD, list(range(world)), torch.device("cpu"))
    out = m2(x, t, m2.prepare_context(text), grid=(3, 4, 6))
    return (out - dense).abs().max().item()


@pytest.mark.multirank
@pytest.mark.parametrize("world", [2, 4])
def test_wan_tensor_parallel_matches_dense(world):
    """Heads / FFN columns over tp ranks; the across-heads q/k RMS (self- and cross-attention,
    and the cached text keys) uses per-row sums of squares all-reduced over the ranks."""
    from difflet_b200.parallel.testing import run_ranks

    assert max(run_ranks(_tp, world, timeout=240)) < 1e-10


def _cp_tp(rank, world, mode):
    from difflet_b200.parallel import groups
    from difflet_b200.parallel.tp import make_tensor_parallel, shard_wan_weights
    from difflet_b200.parallel.ulysses import make_sequence_parallel
    from difflet_b200.pipeline.parallel_config import DiffletParallelConfig

    par_cfg = DiffletParallelConfig(tp_degree=2, cp_degree=world // 2, cp_mode=mode)
    groups.init_mesh(par_cfg.mesh_spec)
    dev = torch.device("cpu")
    cfg = get_wan_config("tiny-wan", heads=8, hidden=1024, ffn=1024)
    m = WanTransformer.random_init(cfg, dtype=torch.float64, seed=8)
    lat, text = _inputs(cfg)
    x = patchify(lat)
    t = torch.tensor([500.0], dtype=torch.float64)
    dense = m(x, t, m.prepare_context(text), grid=(3, 4, 6))
    tp = make_tensor_parallel(par_cfg, dev, transport="nccl")
    sp = make_sequence_parallel(par_cfg, dev, transport="nccl")
    m2 = WanTransformer(cfg, shard_wan_weights(cfg, m.w, tp.world, tp.rank))
    m2.tp, m2.par = tp, sp
    out = sp.gather_tokens(m2(sp.shard_tokens(x), t, m2.prepare_context(text), grid=(3, 4, 6)))
    return (out - dense).abs().max().item()


@pytest.mark.multirank
@pytest.mark.parametrize("mode", ["ulysses", "ring"])
def test_wan_context_parallel_inside_tensor_parallel(mode):
    """tp2 x cp2 over gloo ranks: heads / FFN columns over tp (across-heads q/k RMS summed over
    tp), the sequence over cp (Ulysses splits each tp rank's heads again)."""
    from difflet_b200.parallel.testing import run_ranks

    assert max(run_ranks(_cp_tp, 4, mode, timeout=300)) < 1e-10
