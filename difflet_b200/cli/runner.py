"""Multi-process launch: re-exec a command under ``torch.distributed.run`` (one rank per GPU).

Same role as the reference's ``run_torchrun`` (``difflet/cli/runner.py:127-272``):
rendezvous on 127.0.0.1, children die with the parent (PR_SET_PDEATHSIG), a
bounded stop timeout.
"""

from __future__ import annotations

import os
import signal
import subprocess
import sys


def _pdeathsig():
    try:
        import ctypes

        libc = ctypes.CDLL("libc.so.6")
        libc.prctl(1, signal.SIGTERM)  # PR_SET_PDEATHSIG
    except Exception:
        pass


def run_torchrun(argv: list[str], nproc: int, *, port: int | None = None, timeout_s: float | None = None,
                 env: dict | None = None) -> int:
    from difflet_b200.parallel.testing import free_port

    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", f"--master-port={port or free_port()}", "-m", "difflet_b200"] + argv
    e = dict(os.environ)
    e.update(env or {})
    e["DIFFLET_UNDER_TORCHRUN"] = "1"
    p = subprocess.Popen(cmd, env=e, preexec_fn=_pdeathsig)
    try:
        return p.wait(timeout=timeout_s)
    except subprocess.TimeoutExpired:
        p.terminate()
        try:
            p.wait(timeout=30)
        except subprocess.TimeoutExpired:
            p.kill()
        return 124
