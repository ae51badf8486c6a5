"""Headline benchmark: FLUX.1-dev 1024x1024 DiT denoise step (and e2e s/image) on N B200s.
``--model wan``: Wan2.2-T2V-A14B 1280x720x81 (40 steps, CFG 5, CFG2 x Ulysses-4 on 8 GPUs) DiT step / decode / e2e s/video.

Contract (one rank per GPU; the driver launches N > 1 under torch.distributed.run):
  python bench.py --gpus N --steps K --warmup W [--impl ours|reference]

* ``value``: DiT denoise-step latency in ms (one full FLUX.1-dev step at 1024^2:
  timestep/guidance/pooled embedders, all-block adaLN GEMV, 19 double + 38 single
  blocks, final layer, Euler update), timed with CUDA events over exactly K steps
  after W warm-up steps, bracketed by barrier + synchronize, max over ranks.
  Strong scaling: the one image's token sequence is split over the N GPUs with
  Ulysses sequence parallelism (fused peer-memory all-to-alls).
* ``e2e``: seconds per image through the public API (``DiffletPipeline`` ->
  28-step generate -> VAE decode), including every run's host->device copy of
  the inputs (T5-shaped text states, CLIP pooled vector, initial noise, from
  pinned memory) and the device->host read of the decoded uint8 image.
* Weights are random-init bf16 of the FLUX.1-dev architecture (12B); inputs are
  synthetic N(0, 1) (no network).  The 24 GB of weights stream from HBM every
  step, far larger than the 126 MB L2, so no extra L2 flush is needed.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

REF_PUBLISHED_STEP_MS = 134.1  # reference FLUX.1-dev 1024^2 DiT per-step (1x B300, stock diffusers)
REF_PUBLISHED_E2E_S = 7.9      # reference FLUX.1-dev e2e warm (1x B300)


def _log(msg: str) -> None:
    print(f"[bench {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def _dist_setup():
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    if world > 1 and not dist.is_initialized():
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=600))
    return world, rank, local


def _max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    import torch

    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def run_reference(args, world, rank):
    """Reference arm: the unmodified reference from baseline/_ref through its own API."""
    here = os.path.dirname(os.path.abspath(__file__))
    ref = os.path.join(here, "baseline", "_ref")
    reason = None
    if not os.path.isdir(os.path.join(ref, "difflet")):
        reason = "reference not installed under baseline/_ref"
    else:
        sys.path.insert(0, ref)
        try:
            import difflet.backends.cuda.flux.transformer  # noqa: F401  (its CUDA FLUX path)
        except Exception as exc:  # diffusers is a hard dependency of the reference CUDA path
            reason = (f"reference CUDA FLUX path cannot import ({type(exc).__name__}: {exc}); "
                      "diffusers==0.38.0 is not installed in this image and has no offline wheel")
    if reason is not None:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": reason}))
        return 0
    raise RuntimeError("unreachable: reference CUDA path imported but no runner is defined")


def _profile_step(path: str, rank: int, world: int, fwd) -> None:
    """One eager forward on every rank under torch.profiler (same collectives everywhere);
    rank 0 writes kernel name, launches and total device microseconds."""
    import csv
    from collections import defaultdict

    import torch
    from torch.profiler import ProfilerActivity, profile

    _barrier(world)
    torch.cuda.synchronize()
    # every rank runs under the profiler, so no rank's device waits time out on a slower peer
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fwd()
        torch.cuda.synchronize()
    _barrier(world)
    if rank != 0:
        return
    tot, cnt = defaultdict(float), defaultdict(int)
    for ev in prof.events():
        if ev.device_type.name == "CUDA":
            tot[ev.name] += ev.device_time_total if hasattr(ev, "device_time_total") else ev.cuda_time_total
            cnt[ev.name] += 1
    with open(path, "w", newline="") as f:
        w = csv.writer(f)
        w.writerow(["kernel", "launches", "device_us"])
        for name, us in sorted(tot.items(), key=lambda kv: -kv[1]):
            w.writerow([name[:160], cnt[name], round(us, 1)])
    _log(f"profiled one eager step of rank 0 into {path}")


def _flux_layout_name(par, args) -> str:
    if par.cp_degree == 1:
        return f"tp{par.tp_degree}" + ("+sp" if args.sp else "")
    name = f"{par.cp_mode}{par.cp_degree}"
    return name if par.tp_degree == 1 else f"tp{par.tp_degree}x{name}"


def wan_layout(world: int, spec: str | None):
    """DiffletParallelConfig of a Wan layout: cfg2 / ulysses<N> / tp<N> factors joined by 'x'."""
    from difflet_b200.pipeline.parallel_config import DiffletParallelConfig

    if spec is None:
        spec = {1: "single", 2: "cfg2", 4: "cfg2xulysses2", 8: "cfg2xulysses4"}.get(world, f"cfg2xulysses{world // 2}")
    if spec == "single":
        return DiffletParallelConfig(), spec
    cfg, cp, tp, mode = False, 1, 1, "gather_kv"
    for part in spec.split("x"):
        if part == "cfg2":
            cfg = True
        elif part.startswith("tp"):
            tp = int(part[2:])
        else:
            for m in ("ulysses", "ring", "gather_kv"):
                if part.startswith(m):
                    mode, cp = m, int(part[len(m):])
    par = DiffletParallelConfig(tp_degree=tp, cp_degree=cp, cfg_parallel_enabled=cfg, cp_mode=mode)
    if par.world_size != world:
        raise SystemExit(f"layout {spec} needs {par.world_size} ranks, launched with {world}")
    return par, spec


def run_wan(args, world, rank):
    """Wan2.2-T2V-A14B (two 14B experts) at 1280x720x81 frames: 40 UniPC steps, true CFG 5.0.

    * ``value``: one denoise step (high-noise expert, both CFG branches, the fused CFG + UniPC
      kernel), device-timed over K steps after W warm-up steps, max over ranks.  The 28 GB expert
      and the ~20 GB of per-step activations stream through HBM every step (far above L2).
    * ``decode`` (``--decode``): one causal VAE decode of the 21x90x160 latents to 81 frames.
    * ``e2e`` (``--e2e``): a whole video through the public API -- host->device copies of the
      text states and noise from pinned memory, 40 steps, decode, uint8 frames back to the host."""
    import torch

    from difflet_b200 import _native
    from difflet_b200.bench.clocks import ClockSampler
    from difflet_b200.pipeline.difflet_pipeline import DiffletPipeline

    par, layout = wan_layout(world, args.layout)
    H, W, Fr = args.height if args.height != 1024 else 720, args.width if args.width != 1024 else 1280, args.frames
    t_load = time.time()
    pipe = DiffletPipeline.from_pretrained("Wan-AI/Wan2.2-T2V-A14B-Diffusers", parallel=par, height=H, width=W,
                                           num_frames=Fr, random_init=True, skip_warmup=True)
    load_s = time.time() - t_load
    _log(f"Wan pipeline loaded in {load_s:.1f}s ({layout})")
    app = pipe.app.app
    cfg = app.cfg
    steps_total = 40
    gen = torch.Generator().manual_seed(11)
    T = (Fr - 1) // cfg.vae_scale_t + 1
    emb = torch.randn(1, cfg.text_len, cfg.text_dim, generator=gen).to(torch.bfloat16).pin_memory()
    neg = torch.randn(1, cfg.text_len, cfg.text_dim, generator=gen).to(torch.bfloat16).pin_memory()
    noise = torch.randn(1, cfg.in_channels, T, H // cfg.vae_scale, W // cfg.vae_scale, generator=gen).pin_memory()
    if args.warmup + args.steps > 26:
        raise SystemExit("warm-up + timed steps must stay on the high-noise expert (<= 26 of 40 steps)")
    run = app.prepare(prompt_embeds=emb, negative_prompt_embeds=neg, height=H, width=W, num_frames=Fr,
                      num_inference_steps=steps_total, guidance_scale=5.0, latents=noise)
    S_tok = run.grid[0] * run.grid[1] * run.grid[2]
    _log(f"{S_tok} tokens per branch; warming up {args.warmup} steps")
    for i in range(args.warmup):
        run.step(i)
    torch.cuda.synchronize()
    n0 = _launch_count()
    run.step(args.warmup)
    launches_per_step = _launch_count() - n0
    _barrier(world)
    sampler = ClockSampler(_gpu_ids(world) if rank == 0 else [])
    with sampler:
        _barrier(world)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(args.steps):
            run.step(args.warmup + 1 + i)
        end.record()
        _barrier(world)
    ms = _max_over_ranks(start.elapsed_time(end) / args.steps, world)
    clocks = sampler.summary() if rank == 0 else {}
    _log(f"timed {args.steps} steps: {ms:.1f} ms/step")
    _native.check_device_errors()

    decode = None
    if args.decode:
        lat = run.latents()
        _barrier(world)
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        video = app.decode(lat)
        t1.record()
        torch.cuda.synchronize()
        dec_ms = _max_over_ranks(t0.elapsed_time(t1), world)
        decode = {"ms": round(dec_ms, 1), "frames": Fr,
                  "shape": None if video is None else list(video.shape)}
        _log(f"decode: {dec_ms:.1f} ms")
        del video
    del run
    e2e = None
    if args.e2e:
        h2d = sum(t.numel() * t.element_size() for t in (emb, neg, noise))
        d2h = 0

        def one_video():
            nonlocal d2h
            vid = pipe(prompt_embeds=emb, negative_prompt_embeds=neg, latents=noise, num_inference_steps=steps_total,
                       guidance_scale=5.0, height=H, width=W, num_frames=Fr)
            if vid is not None:
                host = vid.to("cpu")
                d2h = host.numel() * host.element_size()

        _barrier(world)
        t0 = time.perf_counter()
        one_video()
        _barrier(world)
        e2e_s = _max_over_ranks(time.perf_counter() - t0, world)
        e2e = {"value": round(e2e_s, 3), "unit": "s/video", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h), "steps_per_video": steps_total,
               "note": "first call of the process (includes per-prompt context setup; no separate warm-up video)"}
        _native.check_device_errors()
    if rank == 0:
        out = {
            "metric": "Wan2.2-T2V-A14B 1280x720x81 DiT denoise step latency (both CFG branches, max over ranks)",
            "value": round(ms, 2), "unit": "ms/step", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 2), "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (random-init Wan2.2-A14B experts, N(0,1) umT5-shaped text / noise)",
            "config": {"model": "Wan2.2-T2V-A14B", "global_batch": 1, "seq_len": S_tok, "height": H, "width": W,
                       "frames": Fr, "guidance": 5.0, "parallelism": layout, "load_s": round(load_s, 1),
                       "l2": "28 GB expert + activations stream from HBM every step; no flush"},
            "clocks": clocks, "gpu_launches": int(launches_per_step * args.steps), "decode": decode, "e2e": e2e,
        }
        print(json.dumps(out), flush=True)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_mmdit(args, world, rank):
    """The HunyuanVideo benchmark (HunyuanVideo 13B, 720x1280x129, 118,800 image tokens, embedded guidance,
    ring-attention CP over N) or the Qwen-Image benchmark (Qwen-Image 20B, 1328^2 = 6,889 tokens, MXFP8 block
    linears, true CFG 4.0 batched on one GPU / CFG-parallel pairs, TP over the rest).

    ``value``: one DiT denoise step (every CFG branch, guidance combine, Euler update), device-timed
    over K steps after W warm-up steps, max over ranks.  Weights (26 / 40 GB) and activations
    stream through HBM every step (far above L2).  ``--layout`` overrides the default by N."""
    import torch

    from difflet_b200 import _native
    from difflet_b200.bench.clocks import ClockSampler
    from difflet_b200.models.mmdit.model import pack_latents
    from difflet_b200.ops import fused as F
    from difflet_b200.pipeline.difflet_pipeline import DiffletPipeline

    hv = args.model == "hunyuan"
    default = ({1: "single"}.get(world, f"ring{world}") if hv else {1: "single"}.get(world, f"tp{world}"))
    par, layout = wan_layout(world, args.layout or default)
    if hv:
        Fr = 129 if args.frames == 81 else args.frames  # HunyuanVideo clip: 129 frames (the Wan default is 81)
        model_id, H, W, steps_total, text_len = "hunyuanvideo-community/HunyuanVideo", 720, 1280, 50, 256
        kw = {}
    else:
        model_id, H, W, Fr, steps_total, text_len = "Qwen/Qwen-Image", 1328, 1328, None, 50, 256
        kw = {"quant": "mxfp8"} if args.quant != "none" else {}
    t_load = time.time()
    pipe = DiffletPipeline.from_pretrained(model_id, parallel=par, height=H, width=W, num_frames=Fr, random_init=True,
                                           skip_warmup=True, application_kwargs=kw)
    load_s = time.time() - t_load
    app = pipe.app.app
    cfg, dit, dev, dt = app.cfg, app.dit, app.device, app.dit.dtype
    gen = torch.Generator().manual_seed(21)
    lh, lw = H // cfg.vae_scale, W // cfg.vae_scale
    T = (Fr - 1) // cfg.vae_scale_t + 1 if hv else 1
    grid = (T // cfg.patch_t, lh // cfg.patch, lw // cfg.patch)
    S_img = grid[0] * grid[1] * grid[2]
    lat = torch.randn(1, cfg.latent_channels, *((T, lh, lw) if hv else (lh, lw)), generator=gen)
    x32 = pack_latents(lat.to(dev), cfg.patch).contiguous()
    true_cfg = not hv
    cfg_par = app.cfg_par if true_cfg else None
    nb = 2 if (true_cfg and cfg_par is None) else 1
    txt = torch.randn(nb, text_len, cfg.text_dim, generator=gen).to(dev, dt)
    pool = torch.randn(nb, cfg.pooled_dim, generator=gen).to(dev) if cfg.pooled_dim else None
    tv = torch.full((nb,), text_len, dtype=torch.int32, device=dev) if hv else None
    par_seq = dit.par
    if par_seq is not None:
        x32 = par_seq.shard_tokens(x32).contiguous()
        if not cfg.refiner_layers:
            txt = par_seq.shard_tokens(txt).contiguous()
    x16 = torch.empty((nb,) + tuple(x32.shape[1:]), device=dev, dtype=dt)
    tvec = torch.full((nb,), 0.8, device=dev)
    gvec = torch.full((nb,), 6.0, device=dev)
    scale, dt_step = 4.0, -1.0 / steps_total

    def one_step():
        x16[:1].copy_(x32)
        if nb == 2:
            x16[1:].copy_(x16[:1])
        v = dit(x16, txt, pool, tvec, gvec, grid=grid, txt_valid=tv)
        if cfg_par is not None:
            v32 = cfg_par.combine(v, scale)
        elif nb == 2:
            u, c = v[:1].float(), v[1:].float()
            v32 = u + scale * (c - u)
            v32 = v32 * (c.norm(dim=-1, keepdim=True) / v32.norm(dim=-1, keepdim=True).clamp_min(1e-12))
        else:
            v32 = v.float()
        x32.add_(v32, alpha=dt_step)

    _log(f"{model_id}: {S_img} image tokens, layout {layout}, loaded in {load_s:.1f}s; warming up")
    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    n0 = _launch_count()
    one_step()
    launches = _launch_count() - n0
    _barrier(world)
    sampler = ClockSampler(_gpu_ids(world) if rank == 0 else [])
    with sampler:
        _barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            one_step()
        b.record()
        _barrier(world)
    ms = _max_over_ranks(a.elapsed_time(b) / args.steps, world)
    _native.check_device_errors()
    del F
    decode = None
    if args.decode and hv and app.vae is not None and rank == 0:
        # one VAE decode of the clip's latents on rank 0 (spatially tiled, the native channels-last
        # decoder on the GPU): latents [1, 16, T, h, w] -> frames [1, 3, Fr, H, W]
        zlat = torch.randn(1, cfg.latent_channels, T, lh, lw, generator=gen).to(dev)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        video = app.vae.decode(zlat)
        t1.record()
        torch.cuda.synchronize()
        decode = {"ms": round(t0.elapsed_time(t1), 1), "frames": int(video.shape[2]), "shape": list(video.shape),
                  "decoder": type(app.vae).__name__}
        if args.decode_compare:  # the same decode by the PyTorch statement of the decoder (cuDNN)
            from difflet_b200.models.vae.hunyuan_vae import HunyuanVAEDecoder

            ref = HunyuanVAEDecoder(app.vae.cfg, app.vae.w)
            t0.record()
            vref = ref.decode(zlat)
            t1.record()
            torch.cuda.synchronize()
            decode["torch_cudnn_ms"] = round(t0.elapsed_time(t1), 1)
            decode["rel_l2_vs_torch"] = round(float((video.float() - vref.float()).norm() / vref.float().norm()), 5)
            del vref
        del video
        _native.check_device_errors()
    if rank == 0:
        name = "HunyuanVideo 720x1280x129" if hv else "Qwen-Image 1328x1328 " + ("MXFP8" if kw else "bf16")
        print(json.dumps({
            "metric": f"{name} DiT denoise step latency (max over ranks)", "value": round(ms, 2), "unit": "ms/step",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 2),
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16" + (" + mxfp8 block linears" if kw else ""),
            "data": "synthetic (random-init weights of the named architecture, N(0,1) text states / latents)",
            "config": {"model": model_id, "global_batch": 1, "seq_len": S_img + text_len, "height": H, "width": W,
                       "frames": Fr, "true_cfg": true_cfg, "parallelism": layout, "load_s": round(load_s, 1),
                       "l2": "weights + activations stream from HBM every step; no flush"},
            "clocks": sampler.summary(), "gpu_launches": int(launches * args.steps), "e2e": None,
            "decode": decode}), flush=True)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    return 0


def _launch_count() -> int:
    from difflet_b200.ops import fused as F

    return F.LAUNCHES[0]


def _gpu_ids(world: int) -> list:
    ids = [int(x) for x in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if x.strip().isdigit()]
    return ids[:world] if ids else list(range(world))


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--height", type=int, default=1024)
    ap.add_argument("--width", type=int, default=1024)
    ap.add_argument("--e2e-images", type=int, default=1)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--profile-step", default=None,
                    help="after timing, profile one eager DiT step (torch.profiler, rank 0) and write the "
                         "per-kernel device time to this CSV (analysis only: numbers under a profiler are "
                         "never the bench value)")
    ap.add_argument("--cp-mode", default="ulysses", choices=["ulysses", "ring", "gather_kv", "tp"],
                    help="how N>1 GPUs split the step: a context-parallel mode, or tensor parallelism")
    ap.add_argument("--sp", action="store_true", help="with --cp-mode tp: Megatron sequence parallelism")
    ap.add_argument("--tp", type=int, default=1,
                    help="with a context-parallel --cp-mode: tensor-parallel degree inside each cp group "
                         "(heads / MLP columns over tp, the sequence over the remaining N / tp ranks)")
    ap.add_argument("--quant", default=None, choices=[None, "mxfp8", "none"],
                    help="MXFP8 block linears (default targets); the headline number is bf16")
    ap.add_argument("--model", default="flux", choices=["flux", "wan", "hunyuan", "qwen"],
                    help="flux: the headline FLUX.1-dev config; wan: Wan2.2-T2V-A14B 720p x 81 frames; "
                         "hunyuan: HunyuanVideo 720p x 129 frames (ring CP); qwen: Qwen-Image 1328^2 MXFP8 true CFG (TP)")
    ap.add_argument("--layout", default=None,
                    help="wan: parallel layout (default by N: 1 batched CFG, 2 cfg2, 4 cfg2xulysses2, "
                         "8 cfg2xulysses4; also e.g. ulysses8, cfg2xtp2xulysses2)")
    ap.add_argument("--frames", type=int, default=81)
    ap.add_argument("--decode-compare", action="store_true",
                    help="hunyuan --decode: also time the PyTorch (cuDNN) decoder on the same latents")
    ap.add_argument("--decode", action="store_true",
                    help="wan / hunyuan: also time one VAE decode of the clip's latents (rank 0 for hunyuan)")
    ap.add_argument("--e2e", action="store_true",
                    help="wan: time the full 40-step generate + decode through the public API (minutes at N=1)")
    args = ap.parse_args(argv)
    import faulthandler

    faulthandler.enable()
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)

    world, rank, local = _dist_setup()
    if args.impl == "reference":
        return run_reference(args, world, rank)
    if args.model == "wan":
        return run_wan(args, world, rank)
    if args.model in ("hunyuan", "qwen"):
        return run_mmdit(args, world, rank)

    import torch

    from difflet_b200.bench.clocks import ClockSampler
    from difflet_b200.ops import fused as F
    from difflet_b200.pipeline.difflet_pipeline import DiffletPipeline
    from difflet_b200.pipeline.parallel_config import DiffletParallelConfig

    if world == 1:
        par = DiffletParallelConfig()
    elif args.cp_mode == "tp":
        par = DiffletParallelConfig(tp_degree=world, sp_enabled=args.sp)
    elif args.tp > 1 and args.tp < world:
        if world % args.tp:
            raise SystemExit(f"--tp {args.tp} does not divide {world} GPUs")
        par = DiffletParallelConfig(tp_degree=args.tp, cp_degree=world // args.tp, cp_mode=args.cp_mode)
    else:
        par = DiffletParallelConfig(cp_degree=world, cp_mode=args.cp_mode)
    t_load = time.time()
    pipe = DiffletPipeline.from_pretrained(
        "black-forest-labs/FLUX.1-dev", parallel=par, height=args.height, width=args.width, random_init=True,
        skip_warmup=True, application_kwargs={"cuda_graph": not args.no_graph,
                                              **({"quant": args.quant} if args.quant else {})})
    load_s = time.time() - t_load
    _log(f"pipeline loaded in {load_s:.1f}s")
    app = pipe.app.app
    dit = app.dit
    cfg = dit.cfg
    dev = dit.device
    B = 1
    h_tok, w_tok = args.height // 16, args.width // 16
    S_img, S_txt = h_tok * w_tok, 512
    shards = par.cp_degree  # TP replicates the tokens; CP shards them
    cp_rank = (rank // par.tp_degree) % par.cp_degree
    S_img_l, S_txt_l = S_img // shards, S_txt // shards

    # ---------------- DiT step (device-timed) ----------------
    g = torch.Generator(device=dev).manual_seed(1234 + cp_rank)
    x32 = torch.randn(B, S_img_l, cfg.in_channels, device=dev, generator=g)
    x16 = x32.to(torch.bfloat16)
    txt = torch.randn(B, S_txt_l, cfg.text_dim, device=dev, generator=g).to(torch.bfloat16)
    pooled = torch.randn(B, cfg.pooled_dim, device=dev, generator=g)
    t_buf = torch.full((B,), 0.75, device=dev)
    gvec = torch.full((B,), 3.5, device=dev)
    step_fn = app._step_fn(("bench", B, S_txt_l, S_img_l), x16, txt, pooled, t_buf, gvec, None, (h_tok, w_tok))
    dt = -1.0 / 28

    def one_step():
        v = step_fn()
        F.euler_step(x32, v, dt, x16=x16)

    _log("capturing / warming the DiT step")
    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    _log("warm-up done")
    # kernel launches per step, counted on an eager forward
    n0 = F.LAUNCHES[0]
    v = dit(x16, txt, pooled, t_buf, gvec, img_hw=(h_tok, w_tok))
    F.euler_step(x32, v, 0.0, x16=x16)
    launches_per_step = F.LAUNCHES[0] - n0
    _barrier(world)
    gpu_ids = [int(x) for x in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if x.strip().isdigit()]
    gpu_ids = gpu_ids[:world] if gpu_ids else list(range(world))
    sampler = ClockSampler(gpu_ids if rank == 0 else [])
    with sampler:
        _barrier(world)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            one_step()
        end.record()
        _barrier(world)
    ms = start.elapsed_time(end) / args.steps
    ms = _max_over_ranks(ms, world)
    _log(f"timed {args.steps} steps: {ms:.3f} ms/step")
    clocks = sampler.summary() if rank == 0 else {}
    if args.profile_step:
        _profile_step(args.profile_step, rank, world, lambda: dit(x16, txt, pooled, t_buf, gvec, img_hw=(h_tok, w_tok)))
    from difflet_b200 import _native

    _native.check_device_errors()

    # ---------------- end to end through the public API ----------------
    e2e = None
    if not args.no_e2e:
        gen = torch.Generator().manual_seed(7)
        emb = torch.randn(B, S_txt, cfg.text_dim, generator=gen).to(torch.bfloat16).pin_memory()
        pool = torch.randn(B, cfg.pooled_dim, generator=gen).pin_memory()
        noise = torch.randn(B, cfg.latent_channels, args.height // 8, args.width // 8, generator=gen).pin_memory()
        h2d = emb.numel() * emb.element_size() + pool.numel() * pool.element_size() + noise.numel() * noise.element_size()
        d2h = 0

        def one_image():
            nonlocal d2h
            img = pipe(prompt_embeds=emb, pooled_prompt_embeds=pool, latents=noise, num_inference_steps=28,
                       guidance_scale=3.5, height=args.height, width=args.width)
            if img is not None:
                host = img.to("cpu")
                d2h = host.numel() * host.element_size()
            return img

        _log("e2e warm-up image")
        one_image()  # warm-up (captures the graph for the pipeline shapes)
        _barrier(world)
        t0 = time.perf_counter()
        for _ in range(args.e2e_images):
            one_image()
        _barrier(world)
        e2e_s = (time.perf_counter() - t0) / args.e2e_images
        e2e_s = _max_over_ranks(e2e_s, world)
        e2e = {"value": round(e2e_s, 4), "unit": "s/image", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h), "steps_per_image": 28,
               "vs_published_reference_s": round(e2e_s / REF_PUBLISHED_E2E_S, 4)}
        _native.check_device_errors()

    if rank == 0:
        out = {
            "metric": "FLUX.1-dev 1024x1024 DiT denoise step latency (max over ranks)",
            "value": round(ms, 3),
            "unit": "ms/step",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 3),
            "higher_is_better": False,
            "scaling": "strong",
            "vs_baseline": round(ms / REF_PUBLISHED_STEP_MS, 4),
            "dtype": "bf16" if not args.quant else "bf16 + mxfp8 block linears",
            "data": "synthetic (random-init FLUX.1-dev weights, N(0,1) text states / pooled / latents)",
            "config": {"model": "FLUX.1-dev", "global_batch": B, "seq_len": S_img + S_txt,
                       "height": args.height, "width": args.width,
                       "parallelism": _flux_layout_name(par, args) if world > 1 else "single",
                       "l2": "weights (24 GB) stream from HBM every step, larger than L2; no flush",
                       "cuda_graph": not args.no_graph, "load_s": round(load_s, 1)},
            "clocks": clocks,
            "gpu_launches": int(launches_per_step * args.steps),
            "e2e": e2e,
        }
        try:  # traceability extras: peak device memory, source revision, versions, GPU
            from difflet_b200.bench import provenance

            out["memory"] = provenance.memory()
            out["provenance"] = provenance.collect()
        except Exception as exc:  # noqa: BLE001 - never lose the result line over metadata
            out["provenance"] = {"error": repr(exc)}
        print(json.dumps(out), flush=True)
    # release CUDA graphs (and any NCCL work they hold) before tearing anything down
    app._graphs.clear()
    del step_fn
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    _log("done")
    return 0


if __name__ == "__main__":
    sys.exit(main())
