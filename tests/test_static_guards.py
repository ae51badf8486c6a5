"""Static guards (CPU): every module imports without a GPU, no collective runs over the
data-parallel axis, and the artefact-cache key keeps its field set.

Mirrors the reference's guards: the import sweep (scripts/test_imports.sh), the "no dp-axis
collective" test (tests/unit/test_no_dp_parasites.py) and the drift guard on the cache-key
tables (difflet/pipeline/difflet_pipeline.py:271-277).  A deliberate change to the key updates
the frozen sets below in the same commit.
"""

import importlib
import pkgutil
import re
from pathlib import Path

import pytest

import difflet_b200
from difflet_b200.parallel.mesh import MeshSpec
from difflet_b200.pipeline import compile_cache as cc
from difflet_b200.pipeline.parallel_config import DiffletParallelConfig

PKG = Path(difflet_b200.__file__).parent


def _modules():  # ``__main__`` is the CLI entry script: importing it runs the CLI
    return sorted(m.name for m in pkgutil.walk_packages([str(PKG)], prefix="difflet_b200.")
                  if not m.name.endswith("__main__"))


@pytest.mark.parametrize("name", _modules())
def test_module_imports_on_cpu(name):
    importlib.import_module(name)


def test_no_collective_over_the_dp_axis():
    """Replicas never synchronise with each other: no code asks for the dp group ..."""
    pat = re.compile(r"""(get_group|get_group_ranks|_axis)\(\s*["']dp["']""")
    hits = [f"{p.relative_to(PKG)}:{i + 1}" for p in PKG.rglob("*.py")
            for i, line in enumerate(p.read_text().splitlines()) if pat.search(line)]
    assert not hits, f"collective group on the dp axis requested at {hits}"
    # ... and every group that collectives use stays inside one replica
    for shape in ((2, 2, 2, 2), (4, 1, 2, 1), (2, 2, 1, 2), (8, 1, 1, 1), (1, 2, 4, 1)):
        m = MeshSpec(dp=shape[0], cfg=shape[1], cp=shape[2], tp=shape[3])
        for axis in ("tp", "cp", "cfg"):
            for ranks in m.axis_groups(axis):
                assert len({m.coords_of(r).dp for r in ranks}) == 1, (shape, axis, ranks)


KEY_FIELDS = {"schema", "model_id", "model_name", "revision", "parallel", "dtype", "shapes", "application_kwargs",
              "backend", "toolchain"}
RUNTIME_ONLY = {"prompt", "negative_prompt", "seed", "num_inference_steps", "guidance_scale", "true_cfg_scale",
                "output", "output_type", "teacache_speedup", "teacache_calibration", "teacache_calibration_path",
                "teacache_cadence", "teacache_online_delta", "requests", "random_init"}


def _spec(**kw):
    base = dict(model_id="black-forest-labs/FLUX.1-dev", model_path="/x", model_name="flux",
                parallel=DiffletParallelConfig(), dtype="bfloat16", height=1024, width=1024, backend="cuda",
                toolchain={"nvcc": "12.9"}, application_kwargs={})
    base.update(kw)
    return cc.CacheSpec(**base)


def test_cache_key_field_sets_are_frozen():
    assert set(_spec().cache_inputs()) == KEY_FIELDS
    assert set(cc.RUNTIME_ONLY_APP_KWARGS) == RUNTIME_ONLY


def test_cache_key_semantics():
    k0 = cc.cache_key(_spec())
    assert cc.cache_key(_spec(model_path="/elsewhere")) == k0  # local path never enters the key
    assert cc.cache_key(_spec(application_kwargs={"seed": 3, "prompt": "x"})) == k0
    assert cc.cache_key(_spec(application_kwargs={"preset": "flux-schnell"})) != k0
    assert cc.cache_key(_spec(parallel=DiffletParallelConfig(tp_degree=2))) != k0
    assert cc.cache_key(_spec(height=768)) != k0
    assert cc.cache_key(_spec(toolchain={"nvcc": "13.0"})) != k0


def test_every_env_variable_is_read_somewhere():
    """No variable in the env registry is declared and then ignored (a silently dead knob)."""
    import re
    from pathlib import Path

    root = Path(__file__).resolve().parents[1] / "difflet_b200"
    names = set(re.findall(r'"(DIFFLET_[A-Z0-9_]+)"\s*:', (root / "envs.py").read_text()))
    assert names
    other = "\n".join(p.read_text() for p in root.rglob("*.py") if p.name != "envs.py")
    other += (root.parent / "bench.py").read_text()
    dead = sorted(n for n in names if n not in other)
    assert not dead, dead


def test_every_cli_flag_is_read_somewhere():
    """Every flag the CLI parses is read by some code path (no silently ignored flags)."""
    import re
    from pathlib import Path

    root = Path(__file__).resolve().parents[1] / "difflet_b200"
    flags = set(re.findall(r'add_argument\("--([a-z0-9-]+)"', (root / "cli" / "main.py").read_text()))
    assert flags
    pkg = "\n".join(p.read_text() for p in root.rglob("*.py"))
    dead = sorted(f for f in flags if not any(p in pkg for p in (f"a.{f.replace('-', '_')}",
                                                                   f"args.{f.replace('-', '_')}",
                                                                   f'"{f.replace("-", "_")}"')))
    assert not dead, dead
