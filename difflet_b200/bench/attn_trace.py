"""Per-key-tile timeline of the flash-attention kernel (diagnostic build).

Run with the trace build of the extension (``DIFFLET_ATTN_TRACE=1`` compiles ``csrc/`` with
``-DDFL_ATTN_TRACE`` into ``_difflet_C_trace``)::

    DIFFLET_ATTN_TRACE=1 python -m difflet_b200.bench.attn_trace [--heads 24] [--seq 4608]

Lane 0 of every warp of CTA (0, 0, 0) records ``clock64`` at fixed points of each key tile
(at most 64 tiles): softmax warps (0-7) after the S barrier (0), S loaded (1), exponent base
known (2), first / second half of P stored and signalled (3, 4); the MMA warp (9) at K ready (0),
after PV of Q tile 0 (1), QK of Q tile 0 (2), PV of Q tile 1 (3), QK of Q tile 1 (4) and at the
loop top (5).  The summary gives the mean cycles of each softmax phase, the MMA warp's waits and
the steady-state period per key tile (the dense tensor work of one tile is 2048 cycles).
"""

from __future__ import annotations

import argparse
import json


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--heads", type=int, default=24)
    ap.add_argument("--seq", type=int, default=4608)
    a = ap.parse_args(argv)
    import torch

    from difflet_b200 import _native

    if not _native._attn_trace():
        raise SystemExit("set DIFFLET_ATTN_TRACE=1 (the release build records no events)")
    nat = _native.require()
    q = torch.randn(1, a.heads, a.seq, 128, device="cuda", dtype=torch.bfloat16)
    k, v = torch.randn_like(q), torch.randn_like(q)
    tr = torch.zeros(16 * 64 * 8, dtype=torch.int64, device="cuda")
    for _ in range(3):
        nat.attention(q, k, v, 0.088)
    nat.attention(q, k, v, 0.088, trace=tr)
    torch.cuda.synchronize()
    t = tr.view(16, 64, 8).cpu()
    base = t[t > 0].min().item()
    nt = min(64, -(-a.seq // 128))
    out = {}
    for w in (0, 4):
        e = (t[w, :nt, :5] - base).double()
        out[f"softmax_warp{w}"] = {
            "s_wait_to_loaded": (e[:, 1] - e[:, 0]).mean().item(), "max": (e[:, 2] - e[:, 1]).mean().item(),
            "half0": (e[:, 3] - e[:, 2]).mean().item(), "half1": (e[:, 4] - e[:, 3]).mean().item(),
            "idle_to_next_s": (e[1:, 0] - e[:-1, 4]).mean().item(),
            "period": (e[-1, 0] - e[1, 0]).item() / max(1, nt - 2)}
    e = (t[9, :nt, :6] - base).double()
    out["mma_warp"] = {"pv0_wait_issue": (e[1:, 1] - e[1:, 0]).mean().item(), "qk0": (e[:, 2] - e[:, 1]).mean().item(),
                       "pv1_wait_issue": (e[1:, 3] - e[1:, 2]).mean().item(), "qk1": (e[:, 4] - e[:, 3]).mean().item(),
                       "k_wait": (e[1:, 0] - e[1:, 5]).mean().item(),
                       "period": (e[-1, 0] - e[1, 0]).item() / max(1, nt - 2)}
    print(json.dumps({k: {kk: round(vv, 1) for kk, vv in v.items()} for k, v in out.items()}, indent=1))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
