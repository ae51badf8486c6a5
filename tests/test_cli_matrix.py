"""The CLI end to end on the CPU backend: ``generate`` for every model family with a tiny random-init
preset, in a fresh process, writing the image or video file (the reference checks its CLI as a
model x mode matrix, ``scripts/verify_cli.py``)."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]

CASES = [
    ("black-forest-labs/FLUX.1-dev", "tiny128", ["--height", "64", "--width", "64"], ".png"),
    ("Wan-AI/Wan2.2-T2V-A14B-Diffusers", "tiny-wan", ["--height", "32", "--width", "32", "--num-frames", "5"], ".avi"),
    ("hunyuanvideo-community/HunyuanVideo", "tiny-hunyuan", ["--height", "32", "--width", "32", "--num-frames", "5"],
     ".avi"),
    ("Qwen/Qwen-Image", "tiny-qwen", ["--height", "32", "--width", "32"], ".png"),
]


@pytest.mark.parametrize("model_id,preset,shape,suffix", CASES)
def test_generate_writes_the_output(tmp_path, model_id, preset, shape, suffix):
    env = dict(os.environ, PYTHONPATH=str(REPO) + os.pathsep + os.environ.get("PYTHONPATH", ""))
    out = tmp_path / "out"
    cmd = [sys.executable, "-m", "difflet_b200", "generate", "--model-id", model_id, "--backend", "cpu",
           "--random-weights", "--preset", preset, "--steps", "2", "--output", str(out), "--cache-dir",
           str(tmp_path / "cache"), *shape]
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=str(tmp_path))
    assert proc.returncode == 0, proc.stderr[-3000:]
    line = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")][-1]
    res = json.loads(line)
    path = Path(res["output"])
    assert path.suffix == suffix and path.exists() and path.stat().st_size > 0
    head = path.read_bytes()[:12]
    assert head[:4] == (b"\x89PNG" if suffix == ".png" else b"RIFF")


def test_dp_batch_writes_every_output(tmp_path):
    """``--dp 2 --requests batch.jsonl``: two replica processes claim the requests; every output
    is written once and the work directory is removed after a successful batch."""
    env = dict(os.environ, PYTHONPATH=str(REPO) + os.pathsep + os.environ.get("PYTHONPATH", ""))
    reqs = tmp_path / "batch.jsonl"
    reqs.write_text("".join(json.dumps({"prompt": p, "output": str(tmp_path / p)}) + "\n" for p in "abc"))
    cmd = [sys.executable, "-m", "difflet_b200", "generate", "--model-id", "black-forest-labs/FLUX.1-dev",
           "--backend", "cpu", "--random-weights", "--preset", "tiny128", "--height", "64", "--width", "64",
           "--steps", "2", "--dp", "2", "--requests", str(reqs), "--work-dir", str(tmp_path / "work"),
           "--cache-dir", str(tmp_path / "cache")]
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=str(tmp_path))
    assert proc.returncode == 0, proc.stderr[-3000:]
    assert all((tmp_path / f"{p}.png").exists() for p in "abc")
    assert not (tmp_path / "work").exists()


def test_dp_batch_keeps_a_work_dir_that_held_files(tmp_path):
    """A ``--work-dir`` that already held files is left in place after the batch."""
    env = dict(os.environ, PYTHONPATH=str(REPO) + os.pathsep + os.environ.get("PYTHONPATH", ""))
    work = tmp_path / "mine"
    work.mkdir()
    (work / "notes.txt").write_text("keep me")
    reqs = tmp_path / "batch.jsonl"
    reqs.write_text(json.dumps({"prompt": "a", "output": str(tmp_path / "a")}) + "\n")
    cmd = [sys.executable, "-m", "difflet_b200", "generate", "--model-id", "black-forest-labs/FLUX.1-dev",
           "--backend", "cpu", "--random-weights", "--preset", "tiny128", "--height", "64", "--width", "64",
           "--steps", "2", "--dp", "2", "--requests", str(reqs), "--work-dir", str(work),
           "--cache-dir", str(tmp_path / "cache")]
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env, cwd=str(tmp_path))
    assert proc.returncode == 0, proc.stderr[-3000:]
    assert (tmp_path / "a.png").exists() and (work / "notes.txt").read_text() == "keep me"
