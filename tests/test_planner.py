"""Planner: legal candidates only, ranking, calibration."""

from difflet_b200.planner import calibrate, enumerate_candidates, plan
from difflet_b200.registry import resolve_model


def test_flux_candidates_respect_capabilities():
    e = resolve_model("black-forest-labs/FLUX.1-dev")
    cands = enumerate_candidates(e, 8)
    assert cands and all(not p.cfg_parallel_enabled for p in cands)  # distilled
    assert all(24 % (p.tp_degree * (p.cp_degree if p.cp_mode == "ulysses" else 1)) == 0 for p in cands)
    assert all(p.world_size == 8 for p in cands)


def test_wan_plan_ranks_and_offers_cfg():
    rows = plan("Wan-AI/Wan2.2-T2V-A14B-Diffusers", gpus=8)
    assert rows and rows == sorted(rows, key=lambda r: (r["est_step_ms"], -r["dp"]))
    assert any(r["parallel"].get("cfg_parallel_enabled") for r in rows)


def test_calibrate_moves_scale(monkeypatch):
    from difflet_b200 import planner as P

    monkeypatch.setattr(P, "_EFF_SCALE", [0.85])  # calibrate() writes the module-level scale: undone after
    s = calibrate([(1.0, 2.0)])
    assert 0.05 <= s <= 1.0


def test_flux_estimates_track_measured_steps(monkeypatch):
    """The cost model against FLUX.1-dev 1024² DiT steps measured on B200 with this engine
    (Ulysses): 65.3 / 37.7 / 22.8 / 17.4 ms at 1 / 2 / 4 / 8 GPUs."""
    from difflet_b200 import planner as P
    from difflet_b200.pipeline.parallel_config import DiffletParallelConfig
    from difflet_b200.registry import resolve_model

    monkeypatch.setattr(P, "_EFF_SCALE", [0.85])  # the shipped scale (another test calibrates it)
    e = resolve_model("black-forest-labs/FLUX.1-dev")
    shape = P.model_shape(e)
    for n, measured_ms in ((1, 65.3), (2, 37.7), (4, 22.8), (8, 17.4)):
        p = DiffletParallelConfig(cp_degree=n, cp_mode="ulysses") if n > 1 else DiffletParallelConfig()
        est_ms = P.estimate_step_s(e, p, shape, 1397.4e12) * 1e3
        assert abs(est_ms - measured_ms) / measured_ms < 0.2, (n, est_ms, measured_ms)


def test_wan_estimates_track_measured_steps(monkeypatch):
    """The cost model against Wan2.2-A14B 1280x720x81 steps (both CFG branches) measured on
    B200 with this engine: 12076 ms on 1 GPU (batched CFG), 5953 ms on 2 (CFG-parallel), 2914 ms
    on 4 (CFG2 x Ulysses-2)."""
    from difflet_b200 import planner as P
    from difflet_b200.pipeline.parallel_config import DiffletParallelConfig
    from difflet_b200.registry import resolve_model

    monkeypatch.setattr(P, "_EFF_SCALE", [0.85])
    e = resolve_model("Wan-AI/Wan2.2-T2V-A14B-Diffusers")
    shape = P.model_shape(e, 720, 1280, 81)
    layouts = ((DiffletParallelConfig(), 12076.0), (DiffletParallelConfig(cfg_parallel_enabled=True), 5953.0),
               (DiffletParallelConfig(cfg_parallel_enabled=True, cp_degree=2, cp_mode="ulysses"), 2914.0))
    for p, measured_ms in layouts:
        est_ms = P.estimate_step_s(e, p, shape, 1397.4e12) * 1e3
        assert abs(est_ms - measured_ms) / measured_ms < 0.1, (p, est_ms, measured_ms)


def test_hunyuan_estimates_track_measured_steps(monkeypatch):
    """HunyuanVideo 720x1280x129 (119,056 tokens, attention-bound) under ring CP: 10606 / 5304 /
    2713 ms measured on 1 / 2 / 4 B200s."""
    from difflet_b200 import planner as P
    from difflet_b200.pipeline.parallel_config import DiffletParallelConfig
    from difflet_b200.registry import resolve_model

    monkeypatch.setattr(P, "_EFF_SCALE", [0.85])
    e = resolve_model("hunyuanvideo-community/HunyuanVideo")
    shape = P.model_shape(e, 720, 1280, 129)
    for cp, measured_ms in ((1, 10606.0), (2, 5304.0), (4, 2713.0)):
        p = DiffletParallelConfig(cp_degree=cp, cp_mode="ring") if cp > 1 else DiffletParallelConfig()
        est_ms = P.estimate_step_s(e, p, shape, 1397.4e12) * 1e3
        assert abs(est_ms - measured_ms) / measured_ms < 0.1, (cp, est_ms, measured_ms)


class _FakeNVML:
    """A stand-in for pynvml: 8 GPUs of 183,359 MiB with 18 active NVLinks each."""

    NVML_NVLINK_MAX_LINKS = 18

    def __init__(self, n=8, links=18):
        self.n, self.links, self.calls = n, links, []

    def nvmlInit(self):
        self.calls.append("init")

    def nvmlShutdown(self):
        self.calls.append("shutdown")

    def nvmlDeviceGetCount(self):
        return self.n

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetName(self, h):
        return b"NVIDIA B200"

    def nvmlDeviceGetMemoryInfo(self, h):
        class M:
            total = 183359 * 2**20
        return M()

    def nvmlDeviceGetNvLinkState(self, h, link):
        return 1 if link < self.links else 0


def test_hardware_detection_reads_nvml_only():
    from difflet_b200.planner.hardware import detect

    fake = _FakeNVML()
    hw = detect(fake)
    assert (hw.gpus, hw.sku, hw.nvlink, hw.nvlink_links, hw.source) == (8, "NVIDIA B200", True, 18, "nvml")
    assert abs(hw.hbm_gb - 179.1) < 0.2
    assert fake.calls == ["init", "shutdown"]  # queries only: no setter exists on the fake

    class Broken:
        def nvmlInit(self):
            raise OSError("no driver")

    assert detect(Broken()).source == "none"
