"""Fused compute + collective paths against their roofline and their NCCL baselines.

Run under torchrun, one rank per GPU::

    python -m torch.distributed.run --nnodes 1 --nproc-per-node N --master-addr 127.0.0.1 \\
        -m difflet_b200.bench.collectives [--iters 20] [--out results.json]

Every path is timed with CUDA events over ``--iters`` back-to-back calls after warm-up (max over
ranks), at FLUX.1-dev shapes (1024^2: 4096 image + 512 text tokens, hidden 3072, 24 heads of 128)
and, for the CFG step, at the Wan 720p x 81 latent (75,600 tokens x 64 values per CFG rank pair).
Roofline of a path = the slower of (its FLOPs at the measured bf16 GEMM peak) and (the bytes it must
move off this GPU over NVLink at the measured 770 GB/s peer copy rate), plus, for the memory-bound
CFG step, its HBM bytes at the measured copy bandwidth; ``frac`` = roofline time / measured time.

  qkv_scatter     the Ulysses seq->heads all-to-all in the q/k/v projection epilogue (the GEMM
                  stores normed, rotated head blocks straight into every owner's q/k/v buffer);
                  baseline: the same GEMM + NCCL all_to_all of q/k/v
  attn_scatter    attention whose epilogue stores each output row to the rank that owns it
                  (heads->seq), between the two device barriers the model runs; baseline: local
                  attention + NCCL all_to_all of the output rows
  tp_row_reduce   row-parallel GEMM whose epilogue scatters partial rows to their owners, then the
                  fixed-order reducer storing finished rows to every rank (all-reduce);
                  baseline: GEMM + NCCL all_reduce
  sp_ln_gather    sequence-parallel LayerNorm + modulation storing its rows into every rank (the
                  all-gather), then the column GEMM; baseline: LN + NCCL all_gather + GEMM
  cfg_step        CFG exchange (the partner's prediction read over NVLink) + guidance combine +
                  UniPC update in one kernel; baseline: NCCL all_gather + the same update

Reference precedent for fusing a collective into the matmul: the TPU collective matmul of
difflet/backends/tpu/ops_impl/collective_matmul.py:14-17,140-203.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys

import torch
import torch.distributed as dist

LINK_GBS = 770.0  # measured NVLink peer copy per direction per GPU on this pool


def _peaks():
    here = os.path.dirname(os.path.abspath(__file__))
    p = os.path.join(here, "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]) * 1e12, float(d["hbm_gbs"]) * 1e9, "measured"
    except (OSError, KeyError, ValueError):
        return 1.59e15, 6.65e12, "fallback"


def _timeit(fn, iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()) * 1e-3  # seconds


def _row(name, fused_s, base_s, flops, link_bytes, hbm_bytes, peak, hbm):
    roof = max(flops / peak, link_bytes / (LINK_GBS * 1e9), hbm_bytes / hbm)
    return {"path": name, "fused_us": round(fused_s * 1e6, 1), "nccl_us": round(base_s * 1e6, 1),
            "speedup_vs_nccl": round(base_s / fused_s, 3), "flops": flops, "nvlink_bytes": link_bytes,
            "hbm_bytes": hbm_bytes, "roofline_us": round(roof * 1e6, 1), "frac": round(roof / fused_s, 3),
            "bound": "compute" if roof == flops / peak else ("nvlink" if roof == link_bytes / (LINK_GBS * 1e9)
                                                             else "hbm")}


def bench_qkv(world, rank, iters, peak, hbm):
    from difflet_b200.layers.rope import rope_tables, joint_ids
    from difflet_b200.ops import fused as F
    from difflet_b200.parallel.ulysses import PeerUlysses

    D, H, dh, S = 3072, 24, 128, 4608
    S_loc = S // world
    par = PeerUlysses(dist.group.WORLD, list(range(world)), torch.device("cuda", rank))
    Hl = H // world
    q, k, v = par.layout(1, H, dh, S_loc, S, torch.bfloat16)
    x = torch.randn(S_loc, D, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(3 * D, D, device="cuda", dtype=torch.bfloat16) * 0.02
    b = torch.zeros(3 * D, device="cuda", dtype=torch.bfloat16)
    wq = torch.ones(dh, device="cuda", dtype=torch.bfloat16)
    cos, sin = rope_tables(joint_ids("flux", 512, (1, 64, 64), "txt_img"), (16, 56, 56), 10000.0, device="cuda")
    sc = dict(q_off=0, k_off=D, v_off=2 * D, S_src=S_loc, H=H, dh=dh, norm_mode=1, wq=wq, wk=wq, eps=1e-6,
              cos=cos, sin=sin, rope_pos_off=rank * S_loc, **par.scatter_kwargs(q, k, v, 0, rank * S_loc, S_loc, S, H))

    def fused():
        F.linear_qkv(x, w, b, scatter=sc)

    y = torch.empty(S_loc, 3 * D, device="cuda", dtype=torch.bfloat16)
    send = torch.empty(3 * S_loc * D, device="cuda", dtype=torch.bfloat16)
    recv = torch.empty_like(send)

    def baseline():
        F.linear(x, w, b, out=y)
        # head-major pack for the exchange: [dest rank][q|k|v][rows][Hl*dh]
        send.view(world, 3, S_loc, Hl * dh).copy_(y.view(S_loc, 3, world, Hl * dh).permute(2, 1, 0, 3))
        dist.all_to_all_single(recv, send)

    tf, tb = _timeit(fused, iters), _timeit(baseline, iters)
    flops = 2.0 * S_loc * 3 * D * D
    link = 3.0 * S_loc * D * 2 * (world - 1) / world
    hbm_b = (S_loc * D + 3 * D * D + 3 * S_loc * D) * 2.0
    par.close()
    return _row(f"qkv_scatter (M {S_loc}, N {3 * D}, K {D})", tf, tb, flops, link, hbm_b, peak, hbm)


def bench_attn(world, rank, iters, peak, hbm):
    from difflet_b200.ops import fused as F
    from difflet_b200.parallel.ulysses import PeerUlysses

    D, H, dh, S = 3072, 24, 128, 4608
    S_loc = S // world
    Hl = H // world
    par = PeerUlysses(dist.group.WORLD, list(range(world)), torch.device("cuda", rank))
    q, k, v = par.layout(1, H, dh, S_loc, S, torch.bfloat16)
    for t in (q, k, v):
        t.normal_()
    target = par.empty((S_loc, D), torch.bfloat16)
    n0, n1 = 512 // world, 4096 // world

    def fused():
        par.attention(q, k, v, 1.0 / math.sqrt(dh), target, 1, n0, n1, D)

    o = torch.empty(1, S, Hl * dh, device="cuda", dtype=torch.bfloat16)
    recv = torch.empty(world, S_loc, Hl * dh, device="cuda", dtype=torch.bfloat16)

    def baseline():
        F.attention(q, k, v, 1.0 / math.sqrt(dh), out=o.view(1, S, Hl, dh).permute(0, 2, 1, 3))
        dist.all_to_all_single(recv, o.view(world, S_loc, Hl * dh))

    tf, tb = _timeit(fused, iters), _timeit(baseline, iters)
    flops = 4.0 * Hl * S * S * dh
    link = S * Hl * dh * 2.0 * (world - 1) / world
    hbm_b = 4.0 * Hl * S * dh * 2
    par.close()
    return _row(f"attn_scatter ({Hl} heads x {S}^2)", tf, tb, flops, link, hbm_b, peak, hbm)


def bench_tp(world, rank, iters, peak, hbm):
    from difflet_b200.ops import fused as F
    from difflet_b200.parallel.tp import PeerTP

    D, Fh, M = 3072, 12288, 4608
    K = (D + Fh) // world  # FLUX single block proj_out over [attn | mlp], row-parallel
    tp = PeerTP(dist.group.WORLD, list(range(world)), torch.device("cuda", rank))
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(D, K, device="cuda", dtype=torch.bfloat16) * 0.02
    b = torch.zeros(D, device="cuda", dtype=torch.bfloat16)
    gate = torch.ones(1, D, device="cuda")
    out = tp.empty((M, D), torch.bfloat16)
    out.zero_()

    def fused():
        tp.row_linear(x, w, b, out=out, gate=gate, resid=out, rows_per_batch=M)

    y = torch.empty(M, D, device="cuda", dtype=torch.bfloat16)

    def baseline():
        F.linear(x, w, None, out=y)
        dist.all_reduce(y)

    tf, tb = _timeit(fused, iters), _timeit(baseline, iters)
    # where the fused path's time goes: the GEMM alone (local output), the GEMM whose epilogue
    # stores partial rows to their owners, one device barrier, the reducer alone
    nat = F.native()
    rpr = -(-M // world)
    slots = tp.slots(rpr, D, torch.bfloat16)
    peers = tp.heap.peer_ptrs(slots)
    rows = max(0, min(rpr, M - rank * rpr))
    outs = tp.heap.peer_ptrs(out)
    parts = {
        "gemm_local_us": _timeit(lambda: F.linear(x, w, None, out=y), iters),
        "gemm_scatter_us": _timeit(lambda: nat.gemm(x, w, None, None, 0, out_peer=peers, rows_per_rank=rpr,
                                                    peer_row_off=rank * rpr, ldd=D), iters),
        "barrier_us": _timeit(tp.heap.barrier, iters),
        "reduce_us": _timeit(lambda: nat.tp_reduce(slots, rpr, world, rows, D, rank * rpr, b, gate, M, out, outs,
                                                   out.stride(0), rank * rpr), iters),
        "allreduce_nccl_us": _timeit(lambda: dist.all_reduce(y), iters),
    }
    flops = 2.0 * M * D * K
    link = 2.0 * M * D * 2 * (world - 1) / world  # partial rows out + finished rows out
    hbm_b = (M * K + D * K + 3 * M * D) * 2.0
    tp.close()
    row = _row(f"tp_row_reduce (M {M}, N {D}, K {K})", tf, tb, flops, link, hbm_b, peak, hbm)
    row["parts"] = {k: round(v * 1e6, 1) for k, v in parts.items()}
    return row


def bench_sp(world, rank, iters, peak, hbm):
    from difflet_b200.ops import fused as F
    from difflet_b200.parallel.tp import PeerTP

    D, M = 3072, 4608
    N = 3 * D // world  # the column-parallel q/k/v GEMM that reads the gathered rows
    tp = PeerTP(dist.group.WORLD, list(range(world)), torch.device("cuda", rank))
    tp.sp = True
    x = torch.randn(M, D, device="cuda", dtype=torch.bfloat16)
    shift = torch.zeros(1, D, device="cuda")
    scale = torch.zeros(1, D, device="cuda")
    norm = tp.empty((M, D), torch.bfloat16)
    w = torch.randn(N, D, device="cuda", dtype=torch.bfloat16) * 0.02
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    r0, n = tp.row_range(M)

    def fused():
        tp.ln_gather(x, norm, shift=shift, scale=scale, eps=1e-6, rows_per_batch=M)
        F.linear(norm, w, None, out=y)

    part = torch.empty(n, D, device="cuda", dtype=torch.bfloat16)
    full = torch.empty(world * n, D, device="cuda", dtype=torch.bfloat16)

    def baseline():
        F.ln_modulate(x[r0:r0 + n], shift=shift, scale=scale, eps=1e-6, rows_per_batch=M, out=part)
        dist.all_gather_into_tensor(full, part)
        F.linear(full[:M], w, None, out=y)

    tf, tb = _timeit(fused, iters), _timeit(baseline, iters)
    flops = 2.0 * M * N * D
    link = n * D * 2.0 * (world - 1)
    hbm_b = (2 * M * D + N * D + M * N) * 2.0
    tp.close()
    return _row(f"sp_ln_gather + GEMM (M {M}, N {N}, K {D})", tf, tb, flops, link, hbm_b, peak, hbm)


def bench_cfg(world, rank, iters, peak, hbm):
    from difflet_b200.parallel import groups
    from difflet_b200.parallel.cfg import CollectiveCfg, PeerCfg
    from difflet_b200.pipeline.parallel_config import DiffletParallelConfig
    from difflet_b200.schedulers.guided import GuidedSampler
    from difflet_b200.schedulers.unipc import UniPCScheduler

    cp = world // 2
    pc = DiffletParallelConfig(cfg_parallel_enabled=True, cp_degree=cp, cp_mode="ulysses" if cp > 1 else "gather_kv")
    groups.init_mesh(pc.mesh_spec)
    group, ranks = groups.get_group("cfg"), groups.get_group_ranks("cfg")
    n = 75600 // cp * 64
    dev = torch.device("cuda", rank)
    peer = PeerCfg(group, ranks, dev)
    coll = CollectiveCfg(group, ranks, dev)
    pred = torch.randn(n, device="cuda").bfloat16()

    def sampler():
        return GuidedSampler(UniPCScheduler(shift=12.0).set_timesteps(10_000), torch.zeros(n, device="cuda"),
                             torch.empty(n, device="cuda", dtype=torch.bfloat16))

    s1, s2 = sampler(), sampler()
    # the device work of one step: the scheduler's per-step weights are host scalars, computed
    # once here so the loop times the exchange + update (not Python bookkeeping)
    k_v, e, gw, _ = s1.coeffs()
    buf = peer.next_pred_buffer(pred.shape, pred.dtype)
    buf.copy_(pred)
    from difflet_b200.ops import fused as F

    def fused():
        peer.heap.barrier()  # the partner's prediction is complete
        F.guided_step(buf, None, scale=5.0, x=s1.x, x16=s1.x16, last=s1.last, m1=s1.m1, m2=s1.m2, m_out=s1.m2,
                      k_v=k_v, e=e, g=gw, store_last=True, b_ptr=peer.heap.peer_ptrs(buf)[1 - peer.rank],
                      swap=peer.is_cond)

    parts = [torch.empty_like(pred) for _ in range(2)]

    def baseline():
        dist.all_gather(parts, pred, group=group)
        F.guided_step(parts[0], parts[1], scale=5.0, x=s2.x, x16=s2.x16, last=s2.last, m1=s2.m1, m2=s2.m2,
                      m_out=s2.m2, k_v=k_v, e=e, g=gw, store_last=True)

    tf, tb = _timeit(fused, iters), _timeit(baseline, iters)
    link = n * 2.0
    hbm_b = n * (2 + 2 + 4 * 4 + 4 * 3 + 2.0)  # a, b, x / last / m1 / m2 in; x / last / m / x16 out
    peer.close()
    return _row(f"cfg_step (Wan 720p x 81, {n} values per rank)", tf, tb, 0.0, link, hbm_b, peak, hbm)


def bench_barrier(world, rank, iters, peak, hbm):
    """The device epoch barrier every fused path uses (flag stores into every peer + bounded
    polling), against NCCL's barrier-equivalent all-reduce of one value."""
    from difflet_b200.parallel.symm import SymmetricHeap

    heap = SymmetricHeap(dist.group.WORLD, list(range(world)), torch.device("cuda", rank))
    one = torch.ones(1, device="cuda")
    tf = _timeit(heap.barrier, iters * 10)
    tb = _timeit(lambda: dist.all_reduce(one), iters * 10)
    heap.close()
    return _row("peer_barrier", tf, tb, 0.0, 4.0 * world, 0.0, peak, hbm)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", default=None, help="comma list of paths: qkv,attn,tp,sp,cfg")
    ap.add_argument("--out", default=None)
    args = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world < 2:
        print("run under torchrun with 2 or more ranks", file=sys.stderr)
        return 2
    torch.cuda.set_device(local)
    from datetime import timedelta

    dist.init_process_group("nccl", device_id=torch.device("cuda", local), timeout=timedelta(seconds=300))
    peak, hbm, src = _peaks()
    torch.manual_seed(rank)
    rows = []
    todo = (args.only or "barrier,qkv,attn,tp,sp,cfg").split(",")
    fns = {"barrier": bench_barrier, "qkv": bench_qkv, "attn": bench_attn, "tp": bench_tp, "sp": bench_sp,
           "cfg": bench_cfg}
    for name in todo:
        rows.append(fns[name](world, rank, args.iters, peak, hbm))
        if rank == 0:
            print(json.dumps(rows[-1]), flush=True)
    from difflet_b200 import _native

    _native.check_device_errors()
    if rank == 0 and args.out:
        with open(args.out, "w") as f:
            json.dump({"world": world, "peaks": src, "bf16_flops": peak, "hbm_Bps": hbm, "link_GBps": LINK_GBS,
                       "rows": rows}, f, indent=1)
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
