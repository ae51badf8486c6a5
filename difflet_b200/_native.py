"""Build and load the in-tree sm_100a extension (``difflet_b200/_build/_difflet_C*.so``).

The CUDA sources under ``csrc/`` are plain CUDA translation units (no torch
headers) plus one torch binding file.  ``build()`` compiles them for
``sm_100a`` with ``torch.utils.cpp_extension`` into ``difflet_b200/_build``;
``load()`` imports the built module straight from that directory when the
source hash matches, so a machine that received the built ``.so`` (a GPU box)
does not rebuild.  On a machine with a GPU the native module is mandatory:
``require()`` raises instead of silently falling back to eager PyTorch.
"""

from __future__ import annotations

import hashlib
import importlib.machinery
import importlib.util
import os
import sys
import threading
from pathlib import Path

_PKG_DIR = Path(__file__).resolve().parent
_REPO = _PKG_DIR.parent
CSRC = _REPO / "csrc"
BUILD_DIR = _PKG_DIR / "_build"
EXT_NAME = "_difflet_C"

CUDA_SOURCES = [
    "gemm.cu",
    "gemm2.cu",
    "norm.cu",
    "attention.cu",
    "comm.cu",
    "mx.cu",
    "conv.cu",
    "probe.cu",
    "probe_noalloc.cu",
    "sched.cu",
    "vae.cu",
    "vae_gn.cu",
]
CPP_SOURCES = ["bindings.cpp"]
HEADERS = ["common.cuh", "kernels.h", "probe_noalloc.h", "gemm_epilogue.cuh"]

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
CXX_FLAGS = ["-O3", "-std=c++17"]
# Link the C++ runtime torch itself uses (the shared libstdc++.so.6).  A toolchain whose
# unversioned libstdc++.so link is missing falls back to the static archive; the extension then
# carries a second copy of the C++ runtime whose iostream / locale state is not the process's,
# and formatting a number into an error message (TORCH_CHECK with an int) dereferences a null
# locale facet instead of raising.
LD_FLAGS = ["-l:libstdc++.so.6"]


def _bounds_check() -> bool:
    from difflet_b200 import envs

    return bool(envs.DIFFLET_BOUNDS_CHECK)


def _ext_name(bounds: bool | None = None) -> str:
    """The release module, or the debug build with device index guards (DIFFLET_BOUNDS_CHECK=1)."""
    return EXT_NAME + ("_bounds" if (_bounds_check() if bounds is None else bounds) else "")


def _nvcc_flags(bounds: bool | None = None) -> list:
    return NVCC_FLAGS + (["-DDFL_BOUNDS_CHECK"] if (_bounds_check() if bounds is None else bounds) else [])

_lock = threading.Lock()
_module = None
_load_error: Exception | None = None


def _sources() -> list[Path]:
    out = []
    for name in CUDA_SOURCES + CPP_SOURCES:
        p = CSRC / name
        if p.exists():
            out.append(p)
    return out


def source_hash(bounds: bool | None = None) -> str:
    h = hashlib.sha256()
    for p in sorted(_sources() + [CSRC / n for n in HEADERS if (CSRC / n).exists()]):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(_nvcc_flags(bounds) + CXX_FLAGS + LD_FLAGS).encode())
    return h.hexdigest()[:24]


def _so_path(bounds: bool | None = None) -> Path | None:
    for suffix in importlib.machinery.EXTENSION_SUFFIXES + [".so"]:
        p = BUILD_DIR / f"{_ext_name(bounds)}{suffix}"
        if p.exists():
            return p
    return None


def _stamp(bounds: bool | None = None) -> Path:
    return BUILD_DIR / f"{_ext_name(bounds)}.hash"


def _build_dir(bounds: bool) -> Path:
    # each variant keeps its own object files (the flags differ); every .so lands in _build/
    return BUILD_DIR if not bounds else BUILD_DIR / "bounds"


def build(verbose: bool = False, force: bool = False):
    """Compile every CUDA source for sm_100a (the variant the environment selects: release, or
    the bounds-check build under DIFFLET_BOUNDS_CHECK=1) and return the loaded module."""
    global _module
    from torch.utils import cpp_extension

    variant = _bounds_check()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    want = source_hash()
    if not force and _so_path() is not None and _stamp().exists() and _stamp().read_text() == want:
        return load()
    os.environ.setdefault("MAX_JOBS", str(min(8, os.cpu_count() or 4)))
    # torch's own arch list must not add other targets: the -gencode above is the only one.
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    bdir = _build_dir(variant)
    bdir.mkdir(parents=True, exist_ok=True)
    mod = cpp_extension.load(
        name=_ext_name(),
        sources=[str(p) for p in _sources()],
        extra_cflags=CXX_FLAGS,
        extra_cuda_cflags=_nvcc_flags(),
        extra_ldflags=LD_FLAGS,
        extra_include_paths=[str(CSRC)],
        build_directory=str(bdir),
        verbose=verbose,
        with_cuda=True,
    )
    if bdir != BUILD_DIR:  # the loader looks for every variant's .so in _build/
        import shutil

        for f in bdir.glob(f"{_ext_name()}*.so"):
            shutil.copy2(f, BUILD_DIR / f.name)
    _stamp().write_text(want)
    _module = mod
    return mod


def build_bounds_variant(verbose: bool = False) -> None:
    """Build the bounds-check variant (``_difflet_C_bounds``) in a child process, so this process
    keeps the release module it may already have loaded."""
    import subprocess

    env = dict(os.environ, DIFFLET_BOUNDS_CHECK="1")
    code = f"from difflet_b200 import _native; _native.build(verbose={bool(verbose)})"
    subprocess.run([sys.executable, "-c", code], env=env, cwd=str(_REPO), check=True)


def load():
    """Import the built extension (building it first if it is missing or stale)."""
    global _module, _load_error
    if _module is not None:
        return _module
    with _lock:
        if _module is not None:
            return _module
        try:
            so = _so_path()
            if so is None or not _stamp().exists() or _stamp().read_text() != source_hash():
                return build()
            import torch  # noqa: F401  (libtorch symbols must be loaded first)

            spec = importlib.util.spec_from_file_location(_ext_name(), str(so))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            sys.modules[_ext_name()] = mod
            _module = mod
            return mod
        except Exception as exc:  # pragma: no cover - surfaced by require()
            _load_error = exc
            raise


def available() -> bool:
    try:
        load()
        return True
    except Exception:
        return False


def require():
    """Return the native module; raise loudly when it cannot be loaded."""
    try:
        return load()
    except Exception as exc:
        raise RuntimeError(
            "difflet_b200 native extension (sm_100a) is not available; build it with "
            "`python -c 'import difflet_b200._native as n; n.build(verbose=True)'`"
        ) from exc


def check_device_errors(device=None) -> None:
    """Raise if any kernel recorded an error in the per-device error word.

    A communication timeout (a peer flag that never arrived) raises ``CommTimeoutError`` and stays
    recorded: every later peer barrier on the device returns at once instead of waiting again, so
    the ranks that are still alive fail fast until ``clear_device_errors`` (after the process group
    was rebuilt).  Other errors are cleared once reported."""
    import torch

    mod = require()
    dev = torch.cuda.current_device() if device is None else int(device)
    word = mod.error_word(dev).cpu().tolist()
    if word[0] != 0:
        from difflet_b200.utils.errors import CommTimeoutError, DeviceError

        if word[0] == 2:
            raise CommTimeoutError(code=word[0], kernel=word[1], detail=(word[2], word[3]))
        mod.error_word(dev).zero_()
        raise DeviceError(code=word[0], kernel=word[1], detail=(word[2], word[3]))


def clear_device_errors(device=None) -> None:
    """Forget a recorded device error (after recovery), re-arming the bounded waits."""
    import torch

    dev = torch.cuda.current_device() if device is None else int(device)
    require().error_word(dev).zero_()
