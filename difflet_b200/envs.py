"""Typed, lazily evaluated environment variables.

Same pattern as the reference's env registry (``difflet/envs.py:65-232``): every
variable is declared once with a parser and a default, and read on attribute
access (``difflet_b200.envs.DIFFLET_BACKEND``), so tests can monkeypatch the
environment.  B200 additions: kernel switches, the communication timeout in
GPU cycles, and the bounds-check debug build.
"""

from __future__ import annotations

import os
from typing import Any, Callable


def _bool(v: str | None, default: bool) -> bool:
    if v is None or v == "":
        return default
    return v.strip().lower() in ("1", "true", "yes", "on")


def _int(v: str | None, default: int | None) -> int | None:
    if v is None or v == "":
        return default
    return int(v)


def _float(v: str | None, default: float | None) -> float | None:
    if v is None or v == "":
        return default
    return float(v)


def _str(v: str | None, default: str | None) -> str | None:
    return default if v is None or v == "" else v


environment_variables: dict[str, Callable[[], Any]] = {
    # backend selection: "cuda" (sm_100a native) or "cpu" (fp32/fp64 oracle)
    "DIFFLET_BACKEND": lambda: _str(os.environ.get("DIFFLET_BACKEND"), None),
    # artefact cache root (content-addressed manifests, kernel tuning)
    "DIFFLET_COMPILE_CACHE": lambda: _str(
        os.environ.get("DIFFLET_COMPILE_CACHE"), os.path.expanduser("~/.cache/difflet_b200")
    ),
    # "graph" captures the denoise step in a CUDA graph, "eager" launches kernels directly
    "DIFFLET_EXEC_MODE": lambda: _str(os.environ.get("DIFFLET_EXEC_MODE"), "graph"),
    # process-group timeout (seconds) for NCCL / gloo groups
    "DIFFLET_PG_TIMEOUT_S": lambda: _int(os.environ.get("DIFFLET_PG_TIMEOUT_S"), 600),
    # pre-sharded weight store directory (per-rank slices written on first load)
    "DIFFLET_WEIGHT_STORE": lambda: _str(os.environ.get("DIFFLET_WEIGHT_STORE"), None),
    # JSONL timing events directory (one file per process)
    "DIFFLET_BENCH_TIMING_DIR": lambda: _str(os.environ.get("DIFFLET_BENCH_TIMING_DIR"), None),
    # per-step wall/device times appended here
    "DIFFLET_STEP_TIMES_FILE": lambda: _str(os.environ.get("DIFFLET_STEP_TIMES_FILE"), None),
    # latent dumps for debugging (one .pt per step)
    "DIFFLET_DUMP_LATENTS_DIR": lambda: _str(os.environ.get("DIFFLET_DUMP_LATENTS_DIR"), None),
    # bounded device waits on peers: cycles before a comm kernel gives up (~2 s at 1.9 GHz)
    "DIFFLET_COMM_TIMEOUT_CYCLES": lambda: _int(os.environ.get("DIFFLET_COMM_TIMEOUT_CYCLES"), 4_000_000_000),
    # compile kernels with index guards that record the first violation in the error word
    "DIFFLET_BOUNDS_CHECK": lambda: _bool(os.environ.get("DIFFLET_BOUNDS_CHECK"), False),
    # force the NCCL baseline for collectives instead of the fused peer-memory kernels
    "DIFFLET_KERNEL_COMM": lambda: _str(os.environ.get("DIFFLET_KERNEL_COMM"), "fused"),
    # attention implementation: "native" (tcgen05) or "sdpa" (library baseline, A/B only)
    "DIFFLET_KERNEL_ATTN": lambda: _str(os.environ.get("DIFFLET_KERNEL_ATTN"), "native"),
    # GEMM implementation: "native" (tcgen05) or "cublas" (library baseline, A/B only)
    "DIFFLET_KERNEL_GEMM": lambda: _str(os.environ.get("DIFFLET_KERNEL_GEMM"), "native"),
    # 1: wide GEMMs with M >= 1024 run on CTA pairs (cta_group::2, 256 x 256 tiles); 0: one CTA per tile
    "DIFFLET_GEMM_PAIR": lambda: _str(os.environ.get("DIFFLET_GEMM_PAIR"), "1"),
    # 1: q/k RMSNorm + RoPE + head scatter run in the qkv projection's GEMM epilogue; 0: separate kernel
    "DIFFLET_FUSE_QKV": lambda: _str(os.environ.get("DIFFLET_FUSE_QKV"), "1"),
    # 1: small-M GEMMs that leave SMs idle split K in two across SMs (serial fixup); 0: never
    "DIFFLET_GEMM_SPLITK": lambda: _str(os.environ.get("DIFFLET_GEMM_SPLITK"), "1"),
    # 1: the text- and image-stream GEMMs of a dual block share one grouped launch; 0: two launches
    "DIFFLET_GEMM_GROUP": lambda: _str(os.environ.get("DIFFLET_GEMM_GROUP"), "1"),
    # epilogue warps of the 2-SM GEMM: 0 = 8 for the q/k/v head-scatter epilogue and 4 otherwise; 4 or 8 = always
    "DIFFLET_GEMM_EPI_WARPS": lambda: _int(os.environ.get("DIFFLET_GEMM_EPI_WARPS"), 0),
    # "auto": attention launches whose query blocks leave SMs idle split the key range; "0": never
    "DIFFLET_ATTN_SPLIT": lambda: _str(os.environ.get("DIFFLET_ATTN_SPLIT"), "auto"),
    # serving
    "DIFFLET_API_KEY": lambda: _str(os.environ.get("DIFFLET_API_KEY"), None),
    "DIFFLET_SERVE_QUEUE_TIMEOUT_S": lambda: _float(os.environ.get("DIFFLET_SERVE_QUEUE_TIMEOUT_S"), 30.0),
    "DIFFLET_HEARTBEAT_S": lambda: _float(os.environ.get("DIFFLET_HEARTBEAT_S"), 5.0),
    # torchrun-provided
    "RANK": lambda: _int(os.environ.get("RANK"), 0),
    "LOCAL_RANK": lambda: _int(os.environ.get("LOCAL_RANK"), 0),
    "WORLD_SIZE": lambda: _int(os.environ.get("WORLD_SIZE"), 1),
    "MASTER_ADDR": lambda: _str(os.environ.get("MASTER_ADDR"), "127.0.0.1"),
    "MASTER_PORT": lambda: _int(os.environ.get("MASTER_PORT"), 29500),
}


def __getattr__(name: str) -> Any:
    if name in environment_variables:
        return environment_variables[name]()
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


def __dir__():
    return list(environment_variables.keys())
