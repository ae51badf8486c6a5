"""CLI presets and flags: --mode layouts per model class and GPU count, explicit flags winning,
--host-vae decode on the host, --dp-schedule static assignment, difflet quant plans."""

import json
import os
import subprocess
import sys
import time
from pathlib import Path

import pytest
import torch

from difflet_b200.cli.main import build_parser
from difflet_b200.cli.modes import apply_mode, preset


def test_presets_by_model_class():
    flux, wan = "black-forest-labs/FLUX.1-dev", "Wan-AI/Wan2.2-T2V-A14B-Diffusers"
    assert preset(flux, "latency", 8) == preset(flux, "latency", 8).__class__(1, False, 8, "ulysses")
    p = preset(wan, "latency", 8)
    assert (p.dp, p.cfg_parallel, p.cp_degree) == (1, True, 4)  # 40 heads: cp 4
    p = preset(wan, "mixed", 8)
    assert (p.dp, p.cfg_parallel, p.cp_degree) == (2, True, 2)
    p = preset(flux, "throughput", 8)
    assert (p.dp, p.cfg_parallel, p.cp_degree) == (8, False, 1)
    p = preset(flux, "latency", 5)  # 24 heads: the largest cp dividing both
    assert p.cp_degree == 1 or 24 % p.cp_degree == 0


def test_explicit_flags_win_over_the_mode():
    a = build_parser().parse_args(["generate", "--model-id", "Wan-AI/Wan2.2-T2V-A14B-Diffusers", "--mode", "latency",
                                   "--cp-degree", "2"])
    apply_mode(a, gpus=8)
    assert a.cp_degree == 2 and a.cfg_parallel and a.dp == 1 and a.tp_degree == 1
    b = build_parser().parse_args(["generate", "--model-id", "black-forest-labs/FLUX.1-dev"])
    apply_mode(b, gpus=8)
    assert (b.dp, b.cp_degree, b.tp_degree) == (1, 1, 1)


def test_host_vae_decodes_on_cpu(tmp_path, monkeypatch):
    from difflet_b200.models.vae.autoencoder_kl import KLDecoder, KLDecoderConfig
    from difflet_b200.utils.host_vae import for_vae, move_to_host, vae_device

    vae = KLDecoder.random_init(KLDecoderConfig(block_out_channels=(32, 32, 32, 32)), dtype=torch.bfloat16)
    move_to_host(vae)
    assert vae_device(vae).type == "cpu" and next(iter(vae.w.values())).dtype == torch.float32
    z = for_vae(vae, torch.randn(1, 16, 4, 4, dtype=torch.bfloat16))
    assert z.dtype == torch.float32 and vae.decode(z).shape == (1, 3, 32, 32)


def test_dp_static_schedule(tmp_path):
    from difflet_b200.cli.dp import worker_loop

    reqs = [{"i": i} for i in range(7)]
    got = {0: [], 1: []}
    for r in (0, 1):
        worker_loop(reqs, tmp_path, lambda req, i, r=r: got[r].append(i) or "ok", replica=(r, 2))
    assert got == {0: [0, 2, 4, 6], 1: [1, 3, 5]}
    assert sorted(p.name for p in Path(tmp_path).glob("*.done")) == sorted(f"{i}.done" for i in range(7))


def test_quant_plan_command():
    r = subprocess.run([sys.executable, "-m", "difflet_b200", "quant", "--model-id", "black-forest-labs/FLUX.1-dev",
                        "--random-weights", "--json"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    info = json.loads(r.stdout)
    assert info["model"] == "flux" and info["targets"] and info["mxfp8_fused_weights"]
    assert all("norm" not in t for t in info["targets"])


def test_host_and_device_vae_exclusive():
    from difflet_b200.cli.main import main

    assert main(["generate", "--model-id", "black-forest-labs/FLUX.1-dev", "--host-vae", "--device-vae"]) == 2


@pytest.mark.parametrize("flag", ["--keep-work-dir"])
def test_work_dir_flag_parses(flag):
    a = build_parser().parse_args(["generate", "--model-id", "x", flag])
    assert a.keep_work_dir


def test_children_die_with_their_parent():
    """A DP worker / torchrun child is signalled when the process that started it exits, so no
    orphan keeps holding its GPUs."""
    import textwrap

    code = textwrap.dedent("""
        import signal, subprocess, sys
        from difflet_b200.cli.runner import die_with_parent
        p = subprocess.Popen([sys.executable, "-c", "import time; time.sleep(60)"],
                             preexec_fn=die_with_parent(signal.SIGKILL))
        print(p.pid, flush=True)
    """)
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=60, check=True)
    pid = int(out.stdout.split()[0])

    def alive():
        try:
            with open(f"/proc/{pid}/status") as f:
                state = [ln for ln in f if ln.startswith("State:")][0]
            return "Z" not in state.split()[1]
        except (FileNotFoundError, IndexError):
            return False

    deadline = time.time() + 10
    while alive() and time.time() < deadline:
        time.sleep(0.1)
    assert not alive()


def test_cache_listing_and_clean_selection(tmp_path, capsys):
    """``cache`` lists entries with their sizes (hard links counted once per entry); ``clean``
    removes only manifest-holding entries chosen by model / key / age, refuses path-like names
    and never follows links out of the cache."""
    from difflet_b200.cli.main import main

    root = tmp_path / "cache"
    outside = tmp_path / "precious"
    outside.mkdir()
    (outside / "keep.txt").write_text("x")
    for model, key, age_days in (("flux", "aaaa", 0), ("flux", "bbbb", 10), ("wan", "cccc", 0)):
        d = root / model / key
        d.mkdir(parents=True)
        (d / "manifest.json").write_text(json.dumps({"inputs": {"dtype": "bf16", "parallel": {}, "shapes": []}}))
        (d / "w.bin").write_bytes(b"0" * 1000)
        t = time.time() - age_days * 86400
        os.utime(d / "manifest.json", (t, t))
    os.link(root / "flux" / "aaaa" / "w.bin", root / "flux" / "aaaa" / "w2.bin")
    (root / "linked").mkdir()
    (root / "linked" / "evil").symlink_to(outside, target_is_directory=True)
    (outside / "manifest.json").write_text("{}")
    assert main(["cache", "--cache-dir", str(root), "--json"]) == 0
    rows = json.loads(capsys.readouterr().out)
    sizes = {r["key"]: r["bytes"] for r in rows}
    assert set(sizes) == {"aaaa", "bbbb", "cccc"} and sizes["aaaa"] == sizes["bbbb"]  # the hard link once
    assert main(["clean", "--cache-dir", str(root), "--model", "../precious"]) == 2
    assert main(["clean", "--cache-dir", str(root)]) == 2
    assert main(["clean", "--cache-dir", str(root), "--older-than-days", "5", "--dry-run"]) == 0
    assert (root / "flux" / "bbbb").exists()
    assert main(["clean", "--cache-dir", str(root), "--older-than-days", "5"]) == 0
    assert not (root / "flux" / "bbbb").exists() and (root / "flux" / "aaaa").exists()
    assert main(["clean", "--cache-dir", str(root), "--key", "cccc"]) == 0
    assert not (root / "wan").exists()
    assert main(["clean", "--cache-dir", str(root), "--all"]) == 0
    assert not (root / "flux").exists() and (outside / "keep.txt").exists()


def test_dp_claims_of_a_dead_worker_are_taken_over(tmp_path):
    """A rerun after a crash claims the requests whose worker is gone; a live worker's claim
    and a finished request are left alone."""
    from difflet_b200.cli.dp import try_claim

    dead = subprocess.Popen([sys.executable, "-c", "pass"])
    dead.wait()
    (tmp_path / "0.claim").write_text(str(dead.pid))      # crashed earlier batch
    (tmp_path / "1.claim").write_text(str(os.getpid()))   # still running
    (tmp_path / "2.claim").write_text(str(dead.pid))
    (tmp_path / "2.done").write_text("{}")
    assert try_claim(tmp_path, 0) and (tmp_path / "0.claim").read_text() == str(os.getpid())
    assert not try_claim(tmp_path, 0)  # now ours: not claimed twice
    assert not try_claim(tmp_path, 1) and not try_claim(tmp_path, 2)
    assert try_claim(tmp_path, 3)
