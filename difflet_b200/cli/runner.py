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


def die_with_parent(sig: int):
    """A ``preexec_fn`` asking the kernel to send ``sig`` to the child when its parent exits
    (Linux ``PR_SET_PDEATHSIG``; a no-op elsewhere).  A child whose parent already exited
    between the fork and this call (re-parented to init) signals itself."""

    def _preexec():
        if not sys.platform.startswith("linux"):
            return
        try:
            import ctypes

            libc = ctypes.CDLL("libc.so.6", use_errno=True)
            libc.prctl(1, int(sig), 0, 0, 0)  # PR_SET_PDEATHSIG
        except Exception:  # noqa: BLE001 - best effort: the child still runs
            return
        if os.getppid() == 1:
            os.kill(os.getpid(), int(sig))

    return _preexec


# torchrun's agent stops its ranks on SIGTERM (a SIGKILLed agent would orphan them)
_pdeathsig = die_with_parent(signal.SIGTERM)


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
