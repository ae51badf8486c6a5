"""Bench recipes and suites on the CPU: extends / env layering, argv translation, refusals,
ABBA planning, the GPU idle check against a fake NVML, and the runner with a fake launcher."""

import json
import subprocess
from types import SimpleNamespace

import pytest

from difflet_b200.bench import host as H
from difflet_b200.bench import recipe as R
from difflet_b200.bench import suite as S


def _write(tmp_path, name, text):
    p = tmp_path / name
    p.write_text(text)
    return p


RECIPES = """
_base:
  args: {backend: cuda, seed: 1, prompt: a cat}
  env: {default: {DIFFLET_ATTN_SPLIT: auto}}
one:
  extends: _base
  args: {model-id: black-forest-labs/FLUX.1-dev, height: 512, width: 512, steps: 4, cfg-parallel: false}
  env: {force: {DIFFLET_GEMM_PAIR: "1"}}
two:
  extends: one
  args: {cp-degree: 2, cp-mode: ulysses, cfg-parallel: true}
"""


def test_extends_env_and_argv(tmp_path):
    rs = R.load_recipes(_write(tmp_path, "r.yaml", RECIPES))
    assert set(rs) == {"one", "two"}  # _base is abstract
    two = rs["two"]
    assert two.args["height"] == 512 and two.args["cp-degree"] == 2 and two.args["prompt"] == "a cat"
    argv = two.argv()
    assert "--cfg-parallel" in argv and "true" not in argv
    assert "--cfg-parallel" not in rs["one"].argv()  # false = switch left out
    env = two.env({"DIFFLET_ATTN_SPLIT": "0", "DIFFLET_GEMM_PAIR": "0"})
    assert env["DIFFLET_ATTN_SPLIT"] == "0" and env["DIFFLET_GEMM_PAIR"] == "1"  # default vs force
    R.validate(two)
    assert S.gpus_needed(two) == 4
    cmd = S.command(two, "/tmp/x")
    assert cmd[1:3] == ["-m", "torch.distributed.run"] and "127.0.0.1" in cmd and cmd[-2:] == ["--output", "/tmp/x"]


@pytest.mark.parametrize("bad,msg", [
    ({"args": {"output": "x"}}, "owns"),
    ({"args": {"prompt": "x"}}, "lacks"),
    ({"args": {"model-id": "m", "prompt": "x", "no-such-flag": 3}}, "rejects"),
])
def test_refusals(bad, msg):
    r = R.resolve("x", {"x": bad})
    with pytest.raises(R.RecipeError, match=msg):
        R.validate(r)


def test_resolve_errors():
    with pytest.raises(R.RecipeError, match="cycle"):
        R.resolve("a", {"a": {"extends": "b"}, "b": {"extends": "a"}})
    with pytest.raises(R.RecipeError, match="unknown keys"):
        R.resolve("a", {"a": {"argz": {}}})


def test_shipped_recipes_and_suites_validate():
    for r in R.load_recipes().values():
        R.validate(r)
    for p in sorted(S.SUITES_DIR.glob("*.yaml")):
        assert S.plan(S.load_suite(str(p)))


def test_abba_plan(tmp_path):
    _write(tmp_path, "r.yaml", RECIPES)
    su = S.load_suite(str(_write(tmp_path, "ab.yaml", """
recipes: [one]
variants: {a: {}, b: {args: {steps: 8}}}
compare: {control: a, candidate: b}
order: ABBA
repeats: 2
""")))
    ls = S.plan(su, R.load_recipes(tmp_path / "r.yaml"))
    assert [x.run_key for x in ls] == ["one/a", "one/b", "one/b", "one/a"] * 2
    assert [x.index for x in ls if x.run_key == "one/b"] == [0, 1, 2, 3]
    assert ls[1].recipe.args["steps"] == 8
    with pytest.raises(R.RecipeError, match="ABBA"):
        S.load_suite(str(_write(tmp_path, "bad.yaml", "recipes: [one]\norder: ABBA\n")))


class FakeNVML:
    def __init__(self, states):
        self.states = states

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetComputeRunningProcesses(self, h):
        return [object()] * self.states[h][0]

    def nvmlDeviceGetUtilizationRates(self, h):
        return SimpleNamespace(gpu=self.states[h][1])

    def nvmlDeviceGetMemoryInfo(self, h):
        return SimpleNamespace(used=int(self.states[h][2] * (1 << 20)))


def test_idle_check_fake_nvml():
    rep = H.check_idle([0, 1], FakeNVML({0: (0, 0, 500), 1: (0, 0, 300)}))
    assert rep.idle and len(rep.devices) == 2
    rep = H.check_idle([0, 1], FakeNVML({0: (1, 0, 500), 1: (0, 90, 90000)}))
    assert not rep.idle
    txt = "; ".join(rep.reasons())
    assert "gpu0: 1 compute" in txt and "gpu1: utilisation 90" in txt and "MiB in use" in txt


def test_runner_records_and_summary(tmp_path):
    _write(tmp_path, "r.yaml", RECIPES)
    su = S.load_suite(str(_write(tmp_path, "ab.yaml", """
recipes: [one]
variants: {a: {}, b: {args: {steps: 8}}}
compare: {control: a, candidate: b}
order: ABBA
""")))
    ls = S.plan(su, R.load_recipes(tmp_path / "r.yaml"))
    seen = []

    def launcher(cmd, **kw):
        seen.append((cmd, kw["env"]))
        sec = 2.0 if "8" in cmd else 1.0
        return subprocess.CompletedProcess(cmd, 0, stdout=f"log\n{json.dumps({'output': 'x', 'seconds': sec})}\n",
                                           stderr="")

    idle = lambda devs: H.check_idle(devs, FakeNVML({0: (0, 0, 10)}))  # noqa: E731
    class Mem:  # stands in for bench.memory.DeviceMemorySampler
        def __init__(self, devices):
            self.devices = devices

        def __enter__(self):
            return self

        def __exit__(self, *exc):
            pass

        def summary(self):
            return {"gpu_peak_gib": {str(d): 1.5 for d in self.devices}}

    recs = S.run(su, ls, tmp_path / "out", launcher=launcher, idle=idle, memory_sampler=Mem)
    assert len(recs) == 4 and all(r["returncode"] == 0 and r["idle_check"]["idle"] for r in recs)
    assert recs[0]["device_memory"] == {"gpu_peak_gib": {"0": 1.5}}
    assert seen[0][1]["DIFFLET_GEMM_PAIR"] == "1"
    lines = (tmp_path / "out" / "ab.jsonl").read_text().splitlines()
    assert len(lines) == 4 and json.loads(lines[0])["run"] == "one/a"
    summ = S.summarize(su, recs)
    assert summ["runs"]["one/a"]["median_s"] == 1.0 and summ["candidate_over_control"]["one"] == 2.0
    # a busy lane is refused, not measured
    busy = lambda devs: H.check_idle(devs, FakeNVML({0: (2, 50, 10)}))  # noqa: E731
    recs = S.run(su, ls[:1], tmp_path / "out2", launcher=launcher, idle=busy)
    assert "not idle" in recs[0]["error"] and "wall_s" not in recs[0]
