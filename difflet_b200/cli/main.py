"""``difflet`` command line: download -> compile -> generate (or ``run`` = all three), plan,
serve, cache, clean, bench.

Same commands and flags as the reference CLI (``difflet/cli/main.py:47-938,1300-1499``;
flag table ``README.md:615-651``).  Multi-GPU runs re-exec under
``torch.distributed.run`` (one rank per GPU); ``--dp N`` splits a ``--requests``
JSONL batch over N replicas with the filesystem claim protocol.
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import sys
import time
from pathlib import Path


def _add_common(p: argparse.ArgumentParser) -> None:
    p.add_argument("--model-id", required=True)
    p.add_argument("--revision", default=None)
    p.add_argument("--backend", default=None, choices=[None, "cuda", "cpu"])
    p.add_argument("--tp-degree", type=int, default=None)
    p.add_argument("--cp-degree", type=int, default=None)
    p.add_argument("--cp-mode", default=None, choices=[None, "gather_kv", "ring", "ulysses"])
    p.add_argument("--cfg-parallel", action="store_true")
    p.add_argument("--sp", action="store_true")
    p.add_argument("--dp", type=int, default=None)
    p.add_argument("--dp-schedule", default="claim", choices=["claim", "static"],
                   help="--dp batches: replicas claim requests as they free up (claim), or replica r takes "
                        "requests r, r + dp, ... (static)")
    p.add_argument("--mode", default=None, choices=[None, "latency", "throughput", "mixed"],
                   help="parallel layout preset for this node's GPUs (explicit parallel flags win)")
    p.add_argument("--height", type=int, default=None)
    p.add_argument("--width", type=int, default=None)
    p.add_argument("--num-frames", type=int, default=None)
    p.add_argument("--shapes", default=None)
    p.add_argument("--cache-dir", default=None)
    p.add_argument("--force", action="store_true")
    p.add_argument("--random-weights", action="store_true", help="seeded random init (offline)")
    p.add_argument("--preset", default=None, help="architecture preset override (e.g. tiny128)")
    p.add_argument("--quant", default=None, choices=[None, "mxfp8"])
    p.add_argument("--quant-compute", default="native", choices=["native", "dequant"])
    p.add_argument("--teacache-cadence", type=int, default=None)
    p.add_argument("--teacache-speedup", type=float, default=None)
    p.add_argument("--teacache-calibration", default=None)
    p.add_argument("--teacache-online-delta", type=float, default=None)
    p.add_argument("--torch-compile", action="store_true", help="accepted for compatibility (no-op: native kernels)")
    p.add_argument("--host-vae", action="store_true", help="decode on the host CPU in fp32 (frees device memory)")
    p.add_argument("--device-vae", action="store_true", help="decode on the GPU (the default)")


def _add_gen(p: argparse.ArgumentParser) -> None:
    p.add_argument("--prompt", default="A photo of a cat")
    p.add_argument("--negative-prompt", default="")
    p.add_argument("--steps", type=int, default=None)
    p.add_argument("--guidance-scale", type=float, default=None)
    p.add_argument("--guidance-scale-2", type=float, default=None)
    p.add_argument("--true-cfg-scale", type=float, default=None)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--output", default="output")
    p.add_argument("--requests", default=None, help="JSONL batch of requests")
    p.add_argument("--work-dir", default=None)
    p.add_argument("--keep-work-dir", action="store_true",
                   help="keep a --dp batch's claim / result directory after a successful run")


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="difflet", description="Blackwell-native diffusion inference")
    sub = ap.add_subparsers(dest="cmd", required=True)
    _add_common(sub.add_parser("download", help="download model weights from Hugging Face"))
    _add_common(sub.add_parser("compile", help="build / verify the sm_100a kernels and write the cache manifest"))
    g = sub.add_parser("generate", help="run inference")
    _add_common(g)
    _add_gen(g)
    r = sub.add_parser("run", help="download + compile + generate")
    _add_common(r)
    _add_gen(r)
    pl = sub.add_parser("plan", help="rank parallel configurations for a model on this machine")
    pl.add_argument("--model-id", required=True)
    pl.add_argument("--gpus", type=int, default=None, help="GPU count (default: detected through NVML, else 8)")
    pl.add_argument("--height", type=int, default=None)
    pl.add_argument("--width", type=int, default=None)
    pl.add_argument("--num-frames", type=int, default=None)
    pl.add_argument("--top", type=int, default=5)
    pl.add_argument("--json", action="store_true")
    s = sub.add_parser("serve", help="OpenAI-compatible image / video server")
    _add_common(s)
    s.add_argument("--host", default="127.0.0.1")
    s.add_argument("--port", type=int, default=8000)
    s.add_argument("--api-key", default=None)
    s.add_argument("--dp-degree", type=int, default=None)
    s.add_argument("--max-queued-requests", type=int, default=8, help="waiting requests per replica before HTTP 429")
    s.add_argument("--queue-timeout", type=float, default=None, help="seconds a request may wait for its replica")
    s.add_argument("--request-timeout", type=float, default=600.0, help="seconds before a request is cancelled")
    s.add_argument("--heartbeat-interval", type=float, default=None, help="worker heartbeat period (s)")
    s.add_argument("--log-dir", default=None, help="serve log files (default: ./logs), one per 5 MB and per day")
    s.add_argument("--video-retention-hours", type=float, default=25.0,
                   help="video models: finished jobs and their files are deleted after this long")
    s.add_argument("--max-video-jobs", type=int, default=4096,
                   help="video models: job records kept at most (new jobs beyond: HTTP 429)")
    q = sub.add_parser("quant", help="write the MXFP8 checkpoint of a model (or print its plan)")
    q.add_argument("--model-id", required=True)
    q.add_argument("--revision", default=None)
    q.add_argument("--cache-dir", default=None)
    q.add_argument("--out", default=None, help="output directory (default: under the cache dir)")
    q.add_argument("--random-weights", action="store_true", help="plan only, from the architecture's shapes")
    q.add_argument("--json", action="store_true")
    c = sub.add_parser("cache", help="inspect the artefact cache")
    c.add_argument("--cache-dir", default=None)
    c.add_argument("--json", action="store_true")
    cl = sub.add_parser("clean", help="remove cache entries")
    cl.add_argument("--cache-dir", default=None)
    cl.add_argument("--model", default=None)
    cl.add_argument("--key", default=None, help="one entry (its hash directory name)")
    cl.add_argument("--older-than-days", type=float, default=None, help="entries whose manifest is older")
    cl.add_argument("--dry-run", action="store_true", help="list what would be removed")
    cl.add_argument("--all", action="store_true")
    b = sub.add_parser("bench", help="kernel microbenchmarks (or the headline bench with --headline)")
    b.add_argument("--only", default="gemm,attn,ln")
    b.add_argument("--headline", action="store_true")
    b.add_argument("--suite", default=None, help="run a bench suite (name under bench/suites or a YAML path)")
    b.add_argument("--out", default="bench_results", help="suite results directory (JSONL per suite)")
    b.add_argument("--dry-run", action="store_true", help="print the suite's launches without running them")
    b.add_argument("--no-idle-check", action="store_true", help="skip the GPU idle check before each launch")
    b.add_argument("--compare", nargs=2, metavar=("A", "B"), default=None,
                   help="compare result B against result A (bench.py lines or suite JSONL)")
    b.add_argument("--report", metavar="DIR", default=None, help="write DIR/SUMMARY.md from the results under DIR")
    b.add_argument("--timing", metavar="DIR", default=None,
                   help="summarise a launch's telemetry (DIFFLET_BENCH_TIMING_DIR files)")
    return ap


def parallel_from_args(a):
    from difflet_b200.pipeline.parallel_config import DiffletParallelConfig

    tp, cp = a.tp_degree or 1, a.cp_degree or 1
    cp_mode = a.cp_mode or ("ulysses" if cp > 1 else "gather_kv")
    return DiffletParallelConfig(tp_degree=tp, cp_degree=cp, cfg_parallel_enabled=a.cfg_parallel,
                                 cp_mode=cp_mode, sp_enabled=a.sp, dp_degree=1)


def _app_kwargs(a) -> dict:
    kw = {}
    if a.random_weights:
        kw["random_init"] = True
    if a.preset:
        kw["preset"] = a.preset
    if a.quant:
        kw["quant"] = a.quant
        kw["quant_compute"] = a.quant_compute
    if getattr(a, "host_vae", False):
        kw["host_vae"] = True
    for k in ("teacache_cadence", "teacache_speedup", "teacache_calibration", "teacache_online_delta"):
        v = getattr(a, k, None)
        if v is not None:
            kw[k] = v
    return kw


def _pipeline(a, load=True):
    from difflet_b200.pipeline.bucketing import parse_shapes
    from difflet_b200.pipeline.difflet_pipeline import DiffletPipeline

    return DiffletPipeline.from_pretrained(
        a.model_id, parallel=parallel_from_args(a), backend=a.backend, height=a.height, width=a.width,
        num_frames=a.num_frames, shapes=parse_shapes(a.shapes) if a.shapes else None, revision=a.revision,
        compile_cache_dir=a.cache_dir, force_compile=a.force, load=load, random_init=a.random_weights,
        application_kwargs=_app_kwargs(a))


def _gen_kwargs(a, req: dict | None = None) -> dict:
    kw = {"prompt": a.prompt, "seed": a.seed}
    if a.steps:
        kw["num_inference_steps"] = a.steps
    if a.guidance_scale is not None:
        kw["guidance_scale"] = a.guidance_scale
    if a.guidance_scale_2 is not None:
        kw["guidance_scale_2"] = a.guidance_scale_2
    if a.true_cfg_scale is not None:
        kw["true_cfg_scale"] = a.true_cfg_scale
    if a.negative_prompt:
        kw["negative_prompt"] = a.negative_prompt
    if a.height:
        kw["height"] = a.height
    if a.width:
        kw["width"] = a.width
    if a.num_frames:
        kw["num_frames"] = a.num_frames
    if req:
        kw.update({k: v for k, v in req.items() if k != "output"})
    return kw


def save_result(out, path: str, entry) -> str:
    from difflet_b200.utils.media import save_image, save_video

    if out is None:
        return ""
    if out.dim() == 5:  # [B, F, H, W, 3]
        return save_video(out[0], path if path.endswith(".avi") else path + ".avi")
    return save_image(out[0], path if path.endswith(".png") else path + ".png")


def _world_needed(a) -> int:
    return parallel_from_args(a).world_size


def _check_spec(a) -> None:
    """Refuse options the model does not take before any process or weight is started."""
    from difflet_b200.models.spec import check_cli_args, check_generate_kwargs, spec_for_model_id

    spec = spec_for_model_id(a.model_id)
    if spec is not None:
        check_cli_args(spec, a)
        check_generate_kwargs(spec, {k: v for k, v in _gen_kwargs(a).items() if k != "prompt"})


def cmd_generate(a) -> int:
    from difflet_b200.models.spec import SpecRefusal

    try:
        _check_spec(a)
    except SpecRefusal as e:
        print(f"difflet: {e}", file=sys.stderr)
        return 2
    world = _world_needed(a)
    if a.dp > 1 and a.requests and not os.environ.get("DIFFLET_DP_RANK"):
        from difflet_b200.cli.dp import run_router

        work = a.work_dir or (a.output + ".work")
        # a directory that held files before this batch is not the batch's to delete
        foreign = Path(work).is_symlink() or (Path(work).is_dir() and any(Path(work).iterdir()))
        rc = run_router(sys.argv[1:], a.dp, world, work, schedule=a.dp_schedule)
        if rc == 0 and not a.keep_work_dir:
            if foreign:
                print(f"difflet: keeping {work}: it was not empty before this batch", file=sys.stderr)
            else:
                shutil.rmtree(work, ignore_errors=True)
        return rc
    if world > 1 and not os.environ.get("DIFFLET_UNDER_TORCHRUN"):
        from difflet_b200.cli.runner import run_torchrun

        return run_torchrun(sys.argv[1:], world)
    from difflet_b200.cli.prewarm import prewarm_cuda

    prewarm_cuda()  # the CUDA context comes up while the weights load
    pipe = _pipeline(a)
    entry = pipe.model_entry
    outputs = []
    if a.requests:
        from difflet_b200.cli.dp import load_requests, worker_loop

        work = Path(a.work_dir or (a.output + ".work"))
        work.mkdir(parents=True, exist_ok=True)

        def one(req, i):
            out = pipe(**_gen_kwargs(a, req))
            return save_result(out, req.get("output", f"{a.output}_{i}"), entry)

        dp_rank = int(os.environ.get("DIFFLET_DP_RANK", "0"))
        fails = worker_loop(load_requests(a.requests), work, one,
                            replica=(dp_rank, a.dp) if a.dp_schedule == "static" else None)
        return 1 if fails else 0
    t0 = time.time()
    out = pipe(**_gen_kwargs(a))
    path = save_result(out, a.output, entry)
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps({"output": path, "seconds": round(time.time() - t0, 3)}))
    return 0


def _dir_size(path: Path) -> int:
    """Bytes under ``path``, each inode once (weight shards hard-linked between entries are
    counted in every entry that links them, but once within one)."""
    seen, total = set(), 0
    for root, _dirs, files in os.walk(path):
        for f in files:
            try:
                st = os.lstat(os.path.join(root, f))
            except OSError:
                continue
            if st.st_ino not in seen:
                seen.add(st.st_ino)
                total += st.st_size
    return total


def _cache_entries(root: Path) -> list[dict]:
    """Every cache entry (a ``<model>/<key>`` directory holding a manifest), never following links."""
    rows = []
    for m in sorted(root.glob("*/*/manifest.json")):
        entry = m.parent
        if entry.is_symlink() or entry.parent.is_symlink():
            continue
        try:
            doc = json.loads(m.read_text())
        except (OSError, ValueError):
            doc = {}
        inputs = doc.get("inputs", {})
        rows.append({"model": entry.parent.name, "key": entry.name, "path": str(entry),
                     "parallel": inputs.get("parallel"), "shapes": inputs.get("shapes"), "dtype": inputs.get("dtype"),
                     "bytes": _dir_size(entry), "mtime": m.stat().st_mtime})
    return rows


def cmd_cache(a) -> int:
    from difflet_b200 import envs

    root = Path(a.cache_dir or envs.DIFFLET_COMPILE_CACHE)
    rows = _cache_entries(root) if root.exists() else []
    if a.json:
        print(json.dumps(rows, indent=2))
    else:
        for r in rows:
            print(f"{r['model']:20s} {r['key']}  {r['bytes'] / 2**20:9.1f} MiB  {r['dtype']}  {r['parallel']}  "
                  f"{r['shapes']}")
        print(f"{len(rows)} entries, {sum(r['bytes'] for r in rows) / 2**30:.2f} GiB")
    return 0


def cmd_clean(a) -> int:
    """Remove cache entries: all, one model's, one key, or those older than N days.  Only
    directories holding a manifest are removed, links are never followed, and names are plain
    directory names (no path can reach outside the cache)."""
    from difflet_b200 import envs

    root = Path(a.cache_dir or envs.DIFFLET_COMPILE_CACHE)
    for name, val in (("--model", a.model), ("--key", a.key)):
        if val is not None and (not val or "/" in val or os.sep in val or val in (".", "..")):
            print(f"{name} must be a plain name, got {val!r}", file=sys.stderr)
            return 2
    if not (a.all or a.model or a.key or a.older_than_days is not None):
        print("nothing selected: give --all, --model, --key or --older-than-days", file=sys.stderr)
        return 2
    now = time.time()
    doomed = []
    for r in (_cache_entries(root) if root.exists() else []):
        if a.model and r["model"] != a.model:
            continue
        if a.key and r["key"] != a.key:
            continue
        if a.older_than_days is not None and now - r["mtime"] < a.older_than_days * 86400:
            continue
        doomed.append(r)
    for r in doomed:
        print(("would remove " if a.dry_run else "removing ") + r["path"])
        if not a.dry_run:
            shutil.rmtree(r["path"], ignore_errors=True)
            try:
                Path(r["path"]).parent.rmdir()  # the model directory, once empty
            except OSError:
                pass
    return 0


def cmd_plan(a) -> int:
    from difflet_b200.planner import plan

    if a.gpus is None:
        from difflet_b200.planner.hardware import detect

        hw = detect()
        a.gpus = hw.gpus or 8
    res = plan(a.model_id, gpus=a.gpus, height=a.height, width=a.width, num_frames=a.num_frames)
    res = res[: a.top]
    if a.json:
        print(json.dumps(res, indent=2))
    else:
        for r in res:
            print(f"{r['est_step_ms']:9.1f} ms  world={r['world']}  {r['parallel']}")
    return 0


def cmd_quant(a) -> int:
    """MXFP8 checkpoint of a model: which linears are quantized (the model's default targets, or
    DIFFLET_QUANT_TARGETS), written once under the cache dir (or --out) and reused by
    ``--quant mxfp8`` loads."""
    from difflet_b200 import envs
    from difflet_b200.quant import checkpoint as QC
    from difflet_b200.quant.targets import default_spec
    from difflet_b200.registry import resolve_model

    entry = resolve_model(a.model_id)
    spec = default_spec(entry.name)
    if a.random_weights:
        info = _quant_plan_from_shapes(entry)
        print(json.dumps(info, indent=1) if a.json else
              f"{entry.name}: {len(info['targets'])} of {info['linears']} linears in MXFP8, "
              f"{len(info['mxfp8_fused_weights'])} fused engine weights")
        return 0
    from difflet_b200.pipeline.path_resolver import resolve_model_path

    model_dir = resolve_model_path(a.model_id, revision=a.revision, allow_patterns=entry.download_patterns)
    src = Path(model_dir) / "transformer" if (Path(model_dir) / "transformer").is_dir() else Path(model_dir)
    out = QC.write_quantized_dir(src, a.out, spec) if a.out else \
        QC.ensure_quantized_dir(a.cache_dir or envs.DIFFLET_COMPILE_CACHE, src, spec)
    man = QC.read_manifest(out)
    print(json.dumps({"quantized": str(out), "counts": man["counts"], "digest": man["digest"]}))
    return 0


def _quant_plan_from_shapes(entry) -> dict:
    """Which diffusers linears of the architecture the model's MXFP8 spec quantizes, and which
    fused engine weights that makes MXFP8 (all their parts targeted) -- no weights needed."""
    from difflet_b200.quant import apply as QA
    from difflet_b200.quant.targets import default_spec

    spec = default_spec(entry.name)
    if entry.name == "wan":
        from difflet_b200.models.wan.model import get_wan_config

        parts = QA.wan_fused_parts(get_wan_config("wan2.2-t2v-a14b"))
    else:
        from difflet_b200.models.mmdit import get_config

        preset = {"flux": "flux-dev", "hunyuan_video": "hunyuan-video", "qwen_image": "qwen-image"}.get(entry.name)
        if preset is None:
            raise SystemExit(f"difflet quant: no architecture plan for {entry.name!r}; give a checkpoint instead")
        parts = QA.mmdit_fused_parts(get_config(preset))
    linears = sorted({n for names in parts.values() for n in names})
    targets = [n for n in linears if spec.matches(n)]
    fused = [k for k, names in parts.items() if all(spec.matches(n) for n in names)]
    return {"model": entry.name, "linears": len(linears), "targets": targets, "mxfp8_fused_weights": fused}


def cmd_serve(a) -> int:
    from difflet_b200.serving.server import serve_main

    return serve_main(a)


def cmd_bench(a) -> int:
    if a.compare:
        from difflet_b200.bench.compare import main as cmain

        return cmain(list(a.compare))
    if a.report:
        from difflet_b200.bench.report import report

        print(report(a.report))
        return 0
    if a.timing:
        from difflet_b200.bench import timing

        print(json.dumps(timing.summarize(timing.read_launch(a.timing)), indent=1))
        return 0
    if a.suite:
        from difflet_b200.bench import suite as S

        su = S.load_suite(a.suite)
        launches = S.plan(su)
        idle = None
        if not (a.dry_run or a.no_idle_check):
            from difflet_b200.bench.host import check_idle

            idle = check_idle
        sampler = None
        if not a.dry_run:
            from difflet_b200.bench.memory import DeviceMemorySampler

            sampler = DeviceMemorySampler
        recs = S.run(su, launches, a.out, idle=idle, dry_run=a.dry_run, memory_sampler=sampler)
        if a.dry_run:
            for r in recs:
                print(json.dumps({"run": r["run"], "launch": r["launch"], "argv": r["argv"]}))
            return 0
        print(json.dumps(S.summarize(su, recs), indent=1))
        return 1 if any(r.get("error") for r in recs) else 0
    if a.headline:
        import runpy

        sys.argv = ["bench.py"]
        runpy.run_path(str(Path(__file__).resolve().parents[2] / "bench.py"), run_name="__main__")
        return 0
    from difflet_b200.bench.kernels import main as kmain

    kmain(["--only", a.only])
    return 0


def main(argv=None) -> int:
    a = build_parser().parse_args(argv)
    if hasattr(a, "tp_degree"):
        if getattr(a, "host_vae", False) and getattr(a, "device_vae", False):
            print("difflet: --host-vae and --device-vae exclude each other", file=sys.stderr)
            return 2
        from difflet_b200.cli.modes import apply_mode

        apply_mode(a)
        if getattr(a, "torch_compile", False):
            print("difflet: --torch-compile has no effect here: the hot ops are sm_100a kernels and the "
                  "denoise step already replays as a CUDA graph", file=sys.stderr)
    if a.cmd == "download":
        from difflet_b200.pipeline.path_resolver import resolve_model_path
        from difflet_b200.registry import resolve_model

        e = resolve_model(a.model_id)
        print(resolve_model_path(a.model_id, revision=a.revision, allow_patterns=e.download_patterns,
                                 random_init=a.random_weights))
        return 0
    if a.cmd == "compile":
        p = _pipeline(a, load=False)
        print(json.dumps({"compiled_path": str(p.compiled_path)}))
        return 0
    if a.cmd in ("generate", "run"):
        return cmd_generate(a)
    return {"plan": cmd_plan, "serve": cmd_serve, "cache": cmd_cache, "clean": cmd_clean, "bench": cmd_bench,
            "quant": cmd_quant}[a.cmd](a)


if __name__ == "__main__":
    sys.exit(main())
