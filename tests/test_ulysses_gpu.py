"""Multi-GPU correctness on every GPU of the box (up to 8): fused context parallelism (peer
memory: Ulysses, ring, gather-KV) and its NCCL baseline, tensor parallelism (plain and with
sequence parallelism), context parallelism inside tensor parallelism, the FLUX forward at N GPUs
against the 1-GPU forward; Wan under TP; CFG-parallel x Ulysses Wan generation (the fused
exchange + guidance + UniPC kernel, peer memory and NCCL) against the 1-GPU batched-CFG run.
With DIFFLET_TEST_REPORT set, rank 0 writes the error of every mode there as JSON."""

import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _composed(rank, world, m, cfg, inputs, dense, wcfg):
    """CP inside TP (FLUX), and CFG-parallel x Ulysses Wan generation, on the same ranks."""
    import torch.distributed as dist

    from difflet_b200.models.flux.model import FluxTransformer
    from difflet_b200.models.wan.model import WanTransformer
    from difflet_b200.models.wan.pipeline import WanApplication
    from difflet_b200.parallel import groups
    from difflet_b200.parallel.tp import make_tensor_parallel, shard_mmdit_weights
    from difflet_b200.parallel.ulysses import make_cfg_parallel, make_sequence_parallel
    from difflet_b200.pipeline.parallel_config import DiffletParallelConfig

    errs = {}
    dev = torch.device("cuda", rank)
    x, txt, pooled, t, gd = inputs
    if world >= 4:
        # (the NCCL ring inside TP is disabled on CUDA: it faulted on 4 GPUs, cause open)
        for mode, transport in (("ulysses", "fused"), ("ulysses", "nccl"), ("ring", "fused")):
            pc = DiffletParallelConfig(tp_degree=2, cp_degree=world // 2, cp_mode=mode)
            groups.init_mesh(pc.mesh_spec)
            tp = make_tensor_parallel(pc, dev, transport=transport)
            sp = make_sequence_parallel(pc, dev, transport=transport)
            m2 = FluxTransformer(cfg, shard_mmdit_weights(cfg, m.w, tp.world, tp.rank))
            m2.tp, m2.par = tp, sp
            for _ in range(2):
                out = m2(sp.shard_tokens(x).contiguous(), sp.shard_tokens(txt).contiguous(), pooled, t, gd,
                         img_hw=(32, 32))
            full = sp.gather_tokens(out).float()
            torch.cuda.synchronize()
            errs[f"{transport}_tp2x{mode}{world // 2}"] = ((full - dense).norm() / dense.norm()).item()
            tp.close()
            sp.close()
    # Wan: cfg2 x Ulysses(world / 2) generation against the batched-CFG 1-GPU run
    g = torch.Generator().manual_seed(9)
    pe = torch.randn(1, wcfg.text_len, wcfg.text_dim, generator=g).bfloat16()
    ne = torch.randn(1, wcfg.text_len, wcfg.text_dim, generator=g).bfloat16()
    lat = torch.randn(1, 16, 3, 16, 32, generator=g)
    kw = dict(prompt_embeds=pe, negative_prompt_embeds=ne, height=128, width=256, num_frames=9,
              num_inference_steps=4, guidance_scale=5.0, latents=lat, output_type="latent")
    wm = WanTransformer.random_init(wcfg, device=dev, dtype=torch.bfloat16, seed=13)
    ref = WanApplication([wm], None, flow_shift=5.0).generate(**kw).float()
    cp = world // 2
    for transport in ("fused", "nccl"):
        pc = DiffletParallelConfig(cfg_parallel_enabled=True, cp_degree=cp,
                                   cp_mode="ulysses" if cp > 1 else "gather_kv")
        groups.init_mesh(pc.mesh_spec)
        seq = make_sequence_parallel(pc, dev, transport=transport)
        cfgp = make_cfg_parallel(pc, dev, transport=transport)
        app = WanApplication([WanTransformer(wcfg, wm.w)], None, flow_shift=5.0, cfg_par=cfgp, seq_par=seq)
        out = app.generate(**kw).float()
        torch.cuda.synchronize()
        errs[f"wan_{transport}_cfg2" + (f"xulysses{cp}" if cp > 1 else "")] = ((out - ref).norm() / ref.norm()).item()
        # both CFG ranks hold bit-identical latents (the same update from the same two predictions)
        mine = out.contiguous()
        both = [torch.empty_like(mine) for _ in range(dist.get_world_size())]
        dist.all_gather(both, mine)
        errs[f"wan_{transport}_cfg_ranks_identical"] = float(all(torch.equal(both[0], b) for b in both))
        if seq is not None:
            seq.close()
        cfgp.close()
    # Wan: Ulysses over every rank, both CFG branches batched on each (a single-stream sequence:
    # the attention epilogue stores every output row at its owner's local row)
    for transport in ("fused", "nccl"):
        pc = DiffletParallelConfig(cp_degree=world, cp_mode="ulysses")
        groups.init_mesh(pc.mesh_spec)
        seq = make_sequence_parallel(pc, dev, transport=transport)
        app = WanApplication([WanTransformer(wcfg, wm.w)], None, flow_shift=5.0, seq_par=seq)
        out = app.generate(**kw).float()
        torch.cuda.synchronize()
        errs[f"wan_{transport}_ulysses{world}"] = ((out - ref).norm() / ref.norm()).item()
        seq.close()
    # Wan VAE: row slabs over every rank (halo rows by peer stores / by NCCL) vs one GPU
    from difflet_b200.models.vae.wan_vae import WanVAEConfig, WanVAEDecoder
    from difflet_b200.parallel.slabs import CollectiveSlabs, PeerSlabs

    vcfg = WanVAEConfig(base_dim=32)
    vae = WanVAEDecoder.random_init(vcfg, device=dev, dtype=torch.bfloat16, seed=6)
    zl = torch.randn(1, 16, 3, 20, 24, generator=torch.Generator().manual_seed(2)).cuda().bfloat16()
    vref = vae.decode(zl).float()
    for name, cls in (("fused", PeerSlabs), ("nccl", CollectiveSlabs)):
        v2 = WanVAEDecoder(vcfg, vae.w)
        v2.set_slabs(cls(dist.group.WORLD, list(range(world)), dev, zl.shape[3]))
        vid = v2.decode(zl)
        torch.cuda.synchronize()
        errs[f"vae_{name}_slabs{world}"] = ((vid.float() - vref).norm() / vref.norm()).item() if rank == 0 else 0.0
        v2.slabs.close()
    return errs


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from difflet_b200 import _native
        from difflet_b200.models.flux.config import get_config
        from difflet_b200.models.flux.model import FluxTransformer, pack_latents
        from difflet_b200.parallel.ring import CollectiveGatherKV, CollectiveRing, PeerGatherKV, PeerRing
        from difflet_b200.parallel.ulysses import CollectiveUlysses, PeerUlysses

        cfg = get_config("tiny128", heads=8, hidden=1024)
        m = FluxTransformer.random_init(cfg, device="cuda", dtype=torch.bfloat16, seed=11)
        g = torch.Generator().manual_seed(0)
        x = pack_latents(torch.randn(1, 16, 64, 64, generator=g)).cuda().bfloat16()
        txt = torch.randn(1, 128, cfg.text_dim, generator=g).cuda().bfloat16()
        pooled = torch.randn(1, cfg.pooled_dim, generator=g).cuda()
        t = torch.full((1,), 0.4, device="cuda")
        gd = torch.full((1,), 3.5, device="cuda")
        dense = m(x, txt, pooled, t, gd, img_hw=(32, 32)).float()
        errs = {}
        for name, cls in (("peer", PeerUlysses), ("nccl", CollectiveUlysses), ("peer_ring", PeerRing),
                          ("nccl_ring", CollectiveRing), ("peer_gather", PeerGatherKV),
                          ("nccl_gather", CollectiveGatherKV)):
            par = cls(dist.group.WORLD, list(range(world)), torch.device("cuda", rank))
            m2 = FluxTransformer(cfg, m.w)
            m2.par = par
            for _ in range(2):  # second call reuses buffers / epochs
                out = m2(par.shard_tokens(x).contiguous(), par.shard_tokens(txt).contiguous(), pooled, t, gd,
                         img_hw=(32, 32))
            full = par.gather_tokens(out).float()
            torch.cuda.synchronize()
            errs[name] = ((full - dense).norm() / dense.norm()).item()
            par.close()
        from difflet_b200.parallel.tp import CollectiveTP, PeerTP, shard_mmdit_weights

        for name, cls, sp in (("peer_tp", PeerTP, False), ("nccl_tp", CollectiveTP, False),
                              ("peer_tp_sp", PeerTP, True)):
            tp = cls(dist.group.WORLD, list(range(world)), torch.device("cuda", rank))
            tp.sp = sp
            m2 = FluxTransformer(cfg, shard_mmdit_weights(cfg, m.w, world, rank))
            m2.tp = tp
            for _ in range(2):
                out = m2(x, txt, pooled, t, gd, img_hw=(32, 32)).float()
            torch.cuda.synchronize()
            errs[name] = ((out - dense).norm() / dense.norm()).item()
            tp.close()
        # Wan under TP: across-heads q/k RMS from all-reduced per-row sums (peer memory and NCCL)
        from difflet_b200.models.wan.model import WanTransformer, get_wan_config, patchify
        from difflet_b200.parallel.tp import shard_wan_weights

        wcfg = get_wan_config("tiny-wan", heads=8, hidden=1024, ffn=1024)
        wm = WanTransformer.random_init(wcfg, device="cuda", dtype=torch.bfloat16, seed=12)
        lat = torch.randn(1, 16, 3, 16, 24, generator=g).cuda().bfloat16()
        text = torch.randn(1, wcfg.text_len, wcfg.text_dim, generator=g).cuda().bfloat16()
        tw = torch.tensor([500.0], device="cuda")
        wx = patchify(lat)
        wdense = wm(wx, tw, wm.prepare_context(text), grid=(3, 8, 12)).float()
        for name, cls in (("wan_peer_tp", PeerTP), ("wan_nccl_tp", CollectiveTP)):
            tp = cls(dist.group.WORLD, list(range(world)), torch.device("cuda", rank))
            w2 = WanTransformer(wcfg, shard_wan_weights(wcfg, wm.w, world, rank))
            w2.tp = tp
            for _ in range(2):
                out = w2(wx, tw, w2.prepare_context(text), grid=(3, 8, 12)).float()
            torch.cuda.synchronize()
            errs[name] = ((out - wdense).norm() / wdense.norm()).item()
            tp.close()
        errs.update(_composed(rank, world, m, cfg, (x, txt, pooled, t, gd), dense, wcfg))
        _native.check_device_errors()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", errs))
    except BaseException as exc:  # noqa: BLE001
        import traceback

        q.put((rank, "err", traceback.format_exc()))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_context_parallel_matches_single_gpu():
    import torch.multiprocessing as mp

    from difflet_b200.parallel.testing import free_port

    world = min(8, torch.cuda.device_count())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in ps:
        p.join(timeout=30)
    for r, status, payload in res:
        assert status == "ok", payload
    report = os.environ.get("DIFFLET_TEST_REPORT")
    if report:
        import json

        with open(report, "w") as f:
            json.dump({"world": world, "errors": {str(r): p for r, _, p in res}}, f, indent=1)
    for r, status, payload in res:
        same = {k: v for k, v in payload.items() if k.endswith("ranks_identical")}
        rel = {k: v for k, v in payload.items() if k not in same}
        # bf16 per-rank vs single-GPU: identical math, different launch shapes
        assert max(rel.values()) < 2e-2, payload
        assert all(v == 1.0 for v in same.values()), payload
