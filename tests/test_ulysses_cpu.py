"""Context parallelism on CPU gloo ranks (Ulysses, ring, gather-KV): every rank's shard
equals the dense forward (difflet tests/unit/backends/test_neuron_joint_attention_cp.py:54-72)."""

import pytest
import torch

from difflet_b200.parallel.testing import run_ranks

pytestmark = pytest.mark.multirank


def _context(mode, world):
    import torch.distributed as dist

    from difflet_b200.parallel import ring, ulysses

    cls = {"ulysses": ulysses.CollectiveUlysses, "ring": ring.CollectiveRing,
           "gather_kv": ring.CollectiveGatherKV}[mode]
    return cls(dist.group.WORLD, list(range(world)), torch.device("cpu"))


def _sp_forward(rank, world, B, mode):
    from difflet_b200.models.flux.config import get_config
    from difflet_b200.models.flux.model import FluxTransformer, pack_latents

    cfg = get_config("tiny128", heads=4, hidden=512)
    m = FluxTransformer.random_init(cfg, dtype=torch.float64, seed=11)
    g = torch.Generator().manual_seed(0)
    x = pack_latents(torch.randn(B, 16, 32, 32, generator=g, dtype=torch.float64))
    txt = torch.randn(B, 64, cfg.text_dim, generator=g, dtype=torch.float64)
    pooled = torch.randn(B, cfg.pooled_dim, generator=g, dtype=torch.float64)
    t = torch.full((B,), 0.4, dtype=torch.float64)
    gd = torch.full((B,), 3.5, dtype=torch.float64)
    dense = m(x, txt, pooled, t, gd, img_hw=(16, 16))
    par = _context(mode, world)
    m2 = FluxTransformer(cfg, m.w)
    m2.par = par
    out = m2(par.shard_tokens(x), par.shard_tokens(txt), pooled, t, gd, img_hw=(16, 16))
    full = par.gather_tokens(out)
    return (full - dense).abs().max().item()


@pytest.mark.parametrize("mode", ["ulysses", "ring", "gather_kv"])
@pytest.mark.parametrize("world,B", [(2, 1), (4, 1), (2, 2)])
def test_cp_matches_dense(world, B, mode):
    errs = run_ranks(_sp_forward, world, B, mode, timeout=240)
    assert max(errs) < 1e-10, errs


def _hv_forward(rank, world, mode):
    from difflet_b200.models.mmdit import MMDiT, get_config, pack_latents

    cfg = get_config("tiny-hunyuan")
    m = MMDiT.random_init(cfg, dtype=torch.float64, seed=2)
    g = torch.Generator().manual_seed(1)
    B, T, Hh, Ww = 2, 2, 16, 16
    x = pack_latents(torch.randn(B, 16, T, Hh, Ww, generator=g, dtype=torch.float64))
    txt = torch.randn(B, 32, cfg.text_dim, generator=g, dtype=torch.float64)
    pooled = torch.randn(B, cfg.pooled_dim, generator=g, dtype=torch.float64)
    t = torch.tensor([0.3, 0.9], dtype=torch.float64)
    gd = torch.tensor([6.0, 6.0], dtype=torch.float64)
    valid = torch.tensor([11, 32])  # padded text: a window that ends inside one rank's text block
    grid = (T, Hh // 2, Ww // 2)
    dense = m(x, txt, pooled, t, gd, grid=grid, txt_valid=valid)
    par = _context(mode, world)
    m2 = MMDiT(cfg, m.w)
    m2.par = par
    out = m2(par.shard_tokens(x), txt, pooled, t, gd, grid=grid, txt_valid=valid)
    return (par.gather_tokens(out) - dense).abs().max().item()


@pytest.mark.parametrize("mode", ["ulysses", "ring", "gather_kv"])
def test_hunyuan_padded_text_cp(mode):
    errs = run_ranks(_hv_forward, 2, mode, timeout=240)
    assert max(errs) < 1e-10, errs


def test_block_windows():
    from difflet_b200.parallel.ring import block_windows

    # [img (2 x 4 rows) ; txt (2 x 3 rows)], prefix windows over the global order
    hi = torch.tensor([8 + 4, 8 + 6, 8, 5])
    w = block_windows(hi, 4, 3, 2)
    # rank 0 block = img[0:4] + txt[0:3]; rank 1 block = img[4:8] + txt[3:6]
    assert w.tolist() == [[4 + 3, 4 + 3, 4, 4], [4 + 1, 4 + 3, 4, 1]]


def _tp_forward(rank, world, B, family, sp=False):
    import torch.distributed as dist

    from difflet_b200.models.mmdit import MMDiT, get_config, pack_latents
    from difflet_b200.parallel.tp import CollectiveTP, shard_mmdit_weights

    name = {"flux": "tiny128", "qwen": "tiny-qwen"}[family]
    cfg = get_config(name, heads=4, hidden=512) if family == "flux" else get_config(name)
    m = MMDiT.random_init(cfg, dtype=torch.float64, seed=21)
    g = torch.Generator().manual_seed(3)
    x = pack_latents(torch.randn(B, 16, 16, 16, generator=g, dtype=torch.float64))
    txt = torch.randn(B, 24, cfg.text_dim, generator=g, dtype=torch.float64)
    pooled = torch.randn(B, cfg.pooled_dim, generator=g, dtype=torch.float64) if cfg.pooled_dim else None
    t = torch.full((B,), 0.6, dtype=torch.float64)
    gd = torch.full((B,), 3.5, dtype=torch.float64)
    dense = m(x, txt, pooled, t, gd, grid=(1, 8, 8))
    tp = CollectiveTP(dist.group.WORLD, list(range(world)), torch.device("cpu"))
    m2 = MMDiT(cfg, shard_mmdit_weights(cfg, m.w, world, rank))
    tp.sp = sp
    m2.tp = tp
    out = m2(x, txt, pooled, t, gd, grid=(1, 8, 8))
    return (out - dense).abs().max().item()


@pytest.mark.parametrize("world,B,family,sp", [(2, 1, "flux", False), (4, 2, "flux", False), (2, 2, "qwen", False),
                                               (2, 1, "flux", True), (2, 1, "qwen", True)])
def test_tensor_parallel_matches_dense(world, B, family, sp):
    errs = run_ranks(_tp_forward, world, B, family, sp, timeout=240)
    assert max(errs) < 1e-10, errs


def _cp_tp_forward(rank, world, tp_deg, mode, family):
    """Context parallelism inside tensor parallelism: the mesh's tp axis shards heads / MLP
    columns, its cp axis shards the sequence (Ulysses splits each rank's tp heads further)."""
    from difflet_b200.models.mmdit import MMDiT, get_config, pack_latents
    from difflet_b200.parallel import groups
    from difflet_b200.parallel.tp import make_tensor_parallel, shard_mmdit_weights
    from difflet_b200.parallel.ulysses import make_sequence_parallel
    from difflet_b200.pipeline.parallel_config import DiffletParallelConfig

    par_cfg = DiffletParallelConfig(tp_degree=tp_deg, cp_degree=world // tp_deg, cp_mode=mode)
    groups.init_mesh(par_cfg.mesh_spec)
    dev = torch.device("cpu")
    name = {"flux": "tiny128", "hunyuan": "tiny-hunyuan"}[family]
    cfg = get_config(name, heads=8, hidden=1024) if family == "flux" else get_config(name, heads=4, hidden=512)
    m = MMDiT.random_init(cfg, dtype=torch.float64, seed=31)
    g = torch.Generator().manual_seed(4)
    B = 1
    if family == "flux":
        x = pack_latents(torch.randn(B, 16, 16, 16, generator=g, dtype=torch.float64))
        grid, valid = (1, 8, 8), None
    else:
        x = pack_latents(torch.randn(B, 16, 2, 16, 16, generator=g, dtype=torch.float64))
        grid, valid = (2, 8, 8), torch.tensor([21])
    txt = torch.randn(B, 32, cfg.text_dim, generator=g, dtype=torch.float64)
    pooled = torch.randn(B, cfg.pooled_dim, generator=g, dtype=torch.float64) if cfg.pooled_dim else None
    t = torch.full((B,), 0.6, dtype=torch.float64)
    gd = torch.full((B,), 3.5, dtype=torch.float64)
    dense = m(x, txt, pooled, t, gd, grid=grid, txt_valid=valid)
    tp = make_tensor_parallel(par_cfg, dev, transport="nccl")
    sp = make_sequence_parallel(par_cfg, dev, transport="nccl")
    m2 = MMDiT(cfg, shard_mmdit_weights(cfg, m.w, tp.world, tp.rank))
    m2.tp, m2.par = tp, sp
    txt_in = txt if cfg.refiner_layers else sp.shard_tokens(txt)
    out = m2(sp.shard_tokens(x), txt_in, pooled, t, gd, grid=grid, txt_valid=valid)
    return (sp.gather_tokens(out) - dense).abs().max().item()


@pytest.mark.parametrize("tp_deg,mode,family", [(2, "ulysses", "flux"), (2, "ring", "flux"), (2, "gather_kv", "flux"),
                                                (2, "ulysses", "hunyuan")])
def test_context_parallel_inside_tensor_parallel(tp_deg, mode, family):
    errs = run_ranks(_cp_tp_forward, 4, tp_deg, mode, family, timeout=300)
    assert max(errs) < 1e-10, errs
