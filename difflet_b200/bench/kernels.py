"""Kernel microbenchmarks on one GPU: our sm_100a kernels vs the library path.

Every number is a CUDA-event time on the launching stream after warm-up, with
an L2 flush (a 256 MB write) before each timed launch, reported as the median
of the timed launches.  Usage::

    python -m difflet_b200.bench.kernels [--only gemm,attn,ln,mx,gemv,qkv] [--cases flux_1gpu,...]
                                         [--iters 20] [--no-ref]

``--no-ref`` skips the library comparison (used for ncu captures so the
profiled process launches only our kernels).
"""

from __future__ import annotations

import argparse
import json
import math

import torch

GEMM_SHAPES = [
    # FLUX.1-dev 1024^2 on one GPU: the GEMMs that dominate the step
    ("flux_qkv_img", 4096, 9216, 3072),
    ("flux_out_img", 4096, 3072, 3072),
    ("flux_mlp_up", 4096, 12288, 3072),
    ("flux_mlp_down", 4096, 3072, 12288),
    ("flux_single_fused", 4608, 21504, 3072),
    ("flux_single_proj_out", 4608, 3072, 15360),
    # Ulysses-8 (576 rows per rank) and tp2 x Ulysses-4 (1152 rows, half the columns / K)
    ("flux_u8_qkv_img", 512, 9216, 3072),
    ("flux_u8_single_fused", 576, 21504, 3072),
    ("flux_u8_single_proj_out", 576, 3072, 15360),
    ("flux_u8_mlp_down", 512, 3072, 12288),
    ("flux_tp2u4_single_fused", 1152, 10752, 3072),
    ("flux_tp2u4_single_proj_out", 1152, 3072, 7680),
    # Wan2.2 720p x 81 (75,600 tokens; Ulysses-4 per rank 18,900)
    ("wan_qkv_1gpu", 75600, 15360, 5120),
    ("wan_ffn_up_sp4", 18900, 13824, 5120),
    ("wan_ffn_down_sp4", 18900, 5120, 13824),
    ("square_8192", 8192, 8192, 8192),
]
ATTN_CASES = [("flux_1gpu", 1, 24, 4608), ("flux_sp2_heads", 1, 12, 4608), ("flux_sp4_heads", 1, 6, 4608),
              ("flux_sp8_heads", 1, 3, 4608), ("wan_ulysses4", 1, 10, 75600 // 4),
              ("wan_ulysses4_rank", 1, 10, 75600), ("hunyuan_ulysses8_rank", 1, 3, 118800)]
LN_CASES = [("flux_ln", 4608, 3072), ("wan_ln_sp4", 18900, 5120)]


def time_fn(fn, iters=20, warmup=3, flush=None):
    """Median CUDA-event time of fn().  ``flush`` (a buffer larger than L2) is READ before
    each call: the L2 then holds clean lines, so the timed kernel does not pay for writing
    back a flush's dirty lines (which a write-based flush would charge to it)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    sink = None if flush is None else torch.empty((), device=flush.device, dtype=flush.dtype)
    for _ in range(iters):
        if flush is not None:
            torch.sum(flush, dim=0, out=sink)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def _sel(items, cases):
    return [it for it in items if not cases or it[0] in cases]


def bench_gemm(nat, iters, flush, peaks, cases, ref, splits=False):
    rows = []
    for name, M, N, K in _sel(GEMM_SHAPES, cases):
        a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        t_ours = time_fn(lambda: nat.gemm(a, b, None, out=out, cta_mode=1), iters, flush=flush)
        t_pair = time_fn(lambda: nat.gemm(a, b, None, out=out, cta_mode=2), iters, flush=flush)
        t_narrow = time_fn(lambda: nat.gemm(a, b, None, out=out, cta_mode=3), iters, flush=flush)
        t_auto = time_fn(lambda: nat.gemm(a, b, None, out=out), iters, flush=flush)
        fl = 2.0 * M * N * K
        r = {"kernel": "gemm_tcgen05", "shape": name, "M": M, "N": N, "K": K, "ms": round(t_ours, 4),
             "tflops": round(fl / t_ours / 1e9, 1),
             "frac_of_measured_peak": round(fl / t_ours / 1e9 / peaks["bf16_tflops"], 3),
             "pair_ms": round(t_pair, 4), "pair_tflops": round(fl / t_pair / 1e9, 1),
             "narrow_ms": round(t_narrow, 4), "narrow_tflops": round(fl / t_narrow / 1e9, 1),
             "auto_ms": round(t_auto, 4), "auto_tflops": round(fl / t_auto / 1e9, 1)}
        if ref:
            t_ref = time_fn(lambda: torch.matmul(a, b.t(), out=out), iters, flush=flush)
            r.update({"cublas_ms": round(t_ref, 4), "cublas_tflops": round(fl / t_ref / 1e9, 1)})
        if M <= 1152 and splits:  # small M: every split-K count, one CTA per tile and CTA pairs
            sweep = {}
            for sp in (1, 2, 3, 4):
                nat.gemm_set_split_force(sp)
                for mode, name in ((1, "single"), (2, "pair")):
                    sweep[f"{name}_s{sp}"] = round(time_fn(lambda: nat.gemm(a, b, None, out=out, cta_mode=mode),
                                                           iters, flush=flush), 4)
            nat.gemm_set_split_force(0)
            r["split_sweep_ms"] = sweep
        rows.append(r)
        del a, b, out
    return rows


QKV_CASES = [("flux_single_qkv_epilogue", 4608, 24, 128, 12288, 3072), ("flux_double_qkv_epilogue", 4096, 24, 128, 0, 3072)]


def bench_qkv(nat, iters, flush, peaks, cases, ref):
    """The projection feeding attention with the q/k RMSNorm + RoPE + head scatter in its
    epilogue (FLUX single block: [q | mlp | k | v] with GELU on the MLP columns)."""
    from difflet_b200.ops import fused as F

    rows = []
    for name, M, H, dh, Fm, K in _sel(QKV_CASES, cases):
        D = H * dh
        N = 3 * D + Fm
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
        b = torch.randn(N, device="cuda", dtype=torch.bfloat16)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        q, k, v = (torch.empty(1, H, M, dh, device="cuda", dtype=torch.bfloat16) for _ in range(3))
        wq = torch.ones(dh, device="cuda", dtype=torch.bfloat16)
        ang = torch.rand(M, dh // 2, device="cuda")
        cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
        sc = dict(q_off=0, k_off=D + Fm, v_off=2 * D + Fm, S_src=M, H=H, dh=dh, q_dst=[q], k_dst=[k], v_dst=[v],
                  S_dst=M, norm_mode=1, wq=wq, wk=wq, eps=1e-6, cos=cos, sin=sin)
        kw = dict(act="gelu", act_lo=D, act_hi=D + Fm) if Fm else {}
        t = time_fn(lambda: F.linear_qkv(x, w, b, scatter=sc, out=out, **kw), iters, flush=flush)
        fl = 2.0 * M * N * K
        r = {"kernel": "gemm_qkv_epilogue", "shape": name, "M": M, "N": N, "K": K, "ms": round(t, 4),
             "tflops": round(fl / t / 1e9, 1), "frac_of_measured_peak": round(fl / t / 1e9 / peaks["bf16_tflops"], 3)}
        if ref:  # the epilogue's parts: plain GEMM, GELU window only, then the scatter without norm / RoPE
            t_plain = time_fn(lambda: nat.gemm(x, w, b, out=out), iters, flush=flush)
            r["plain_gemm_ms"] = round(t_plain, 4)
            if Fm:
                t_gelu = time_fn(lambda: F.linear(x, w, b, out=out, act="gelu", act_lo=D, act_hi=D + Fm), iters,
                                 flush=flush)
                r["gelu_window_ms"] = round(t_gelu, 4)
            for tag, upd in (("no_rope", dict(cos=None, sin=None)), ("no_norm_no_rope", dict(cos=None, sin=None,
                                                                                            norm_mode=0))):
                sc2 = dict(sc, **upd)
                r[f"qkv_{tag}_ms"] = round(time_fn(lambda: F.linear_qkv(x, w, b, scatter=sc2, out=out, **kw), iters,
                                                   flush=flush), 4)
        rows.append(r)
    return rows


def bench_mx(nat, iters, flush, peaks, cases, ref):
    """MXFP8 block-scaled GEMM (operands pre-quantized, as weights are offline) and the
    activation quantizer (bytes: bf16 in + fp8 out + scales)."""
    rows = []
    for name, M, N, K in _sel(GEMM_SHAPES, cases):
        if K % 128:
            continue
        a = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
        aq, asf = nat.mx_quantize(a, True)
        bq, bsf = nat.mx_quantize(b, True)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        t = time_fn(lambda: nat.gemm_mx(aq, asf, bq, bsf, None, out=out), iters, flush=flush)
        tq = time_fn(lambda: nat.mx_quantize(a, True), iters, flush=flush)
        fl = 2.0 * M * N * K
        r = {"kernel": "gemm_mx_tcgen05", "shape": name, "M": M, "N": N, "K": K, "ms": round(t, 4),
             "tflops": round(fl / t / 1e9, 1),
             "x_measured_bf16_peak": round(fl / t / 1e9 / peaks["bf16_tflops"], 3),
             "quantize_ms": round(tq, 4), "quantize_gbs": round(M * K * 3.03125 / tq / 1e6, 1)}
        if ref:
            t_ref = time_fn(lambda: torch.matmul(a, b.t(), out=out), iters, flush=flush)
            r.update({"cublas_bf16_ms": round(t_ref, 4), "cublas_bf16_tflops": round(fl / t_ref / 1e9, 1)})
        rows.append(r)
        del a, b, aq, bq, out
    return rows


CONV_CASES = [("kl_512_128", 1, 1, 128, 128, 512, 512, (1, 3, 3)), ("kl_256_512", 1, 1, 512, 512, 256, 256, (1, 3, 3)),
              ("kl_128_1024", 1, 1, 1024, 1024, 128, 128, (1, 3, 3)),
              ("wan_384_180x320", 1, 4, 180, 320, 384, 384, (3, 3, 3)), ("wan_96_720x1280", 1, 2, 720, 1280, 96, 96, (3, 3, 3))]


def bench_conv(nat, iters, flush, peaks, cases, ref):
    """Implicit-GEMM conv vs cuDNN (channels-last bf16) on VAE decoder layers."""
    from difflet_b200.ops import fused as F

    rows = []
    for name, N, T, H, W, Ci, Co, k in _sel(CONV_CASES, cases):
        x = torch.randn(N, T, H, W, Ci, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(Co, Ci, *k, device="cuda", dtype=torch.bfloat16) * 0.02
        w2 = F.conv_weight(w)
        b = torch.zeros(Co, device="cuda", dtype=torch.bfloat16)
        out = torch.empty(N, T, H, W, Co, device="cuda", dtype=torch.bfloat16)
        t = time_fn(lambda: nat.conv3d(x, w2, b, k[0], k[1], k[2], True, None, False, out), iters, flush=flush)
        fl = 2.0 * N * T * H * W * Ci * Co * k[0] * k[1] * k[2]
        r = {"kernel": "conv_tcgen05", "shape": name, "ms": round(t, 4), "tflops": round(fl / t / 1e9, 1),
             "frac_of_measured_peak": round(fl / t / 1e9 / peaks["bf16_tflops"], 3)}
        if ref:
            if k[0] == 1:
                xc = x[:, 0].permute(0, 3, 1, 2)  # NCHW view of channels-last data
                wc = w[:, :, 0].contiguous(memory_format=torch.channels_last)
                fn = lambda: torch.nn.functional.conv2d(xc, wc, b, padding=1)  # noqa: E731
            else:
                xc = torch.nn.functional.pad(x.permute(0, 4, 1, 2, 3), (1, 1, 1, 1, 2, 0))
                xc = xc.contiguous(memory_format=torch.channels_last_3d)
                wc = w.contiguous(memory_format=torch.channels_last_3d)
                fn = lambda: torch.nn.functional.conv3d(xc, wc, b)  # noqa: E731
            tr = time_fn(fn, iters, flush=flush)
            r.update({"cudnn_ms": round(tr, 4), "cudnn_tflops": round(fl / tr / 1e9, 1)})
        rows.append(r)
        del x, out
    return rows


def bench_attn(nat, iters, flush, peaks, cases, ref):
    """Flash attention at the per-rank shapes of the benchmark configs, against torch SDPA (cuDNN
    on sm_100) with ``ref``."""
    rows = []
    for name, B, H, S in _sel(ATTN_CASES, cases):
        q = torch.randn(B, H, S, 128, device="cuda", dtype=torch.bfloat16)
        k = torch.randn_like(q)
        v = torch.randn_like(q)
        o = torch.empty_like(q)
        sc = 1 / math.sqrt(128)
        fl = 4.0 * B * H * S * S * 128
        it = max(2, min(iters, int(2e14 / fl)))  # long sequences: fewer repeats
        t_ours = time_fn(lambda: nat.attention(q, k, v, sc, out=o), it, flush=flush)
        r = {"kernel": "attn_tcgen05", "shape": name, "B": B, "H": H, "S": S, "ms": round(t_ours, 4),
             "tflops": round(fl / t_ours / 1e9, 1),
             "frac_of_measured_peak": round(fl / t_ours / 1e9 / peaks["bf16_tflops"], 3)}
        if ref:
            t_ref = time_fn(lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v, scale=sc), it,
                            flush=flush)
            r.update({"sdpa_ms": round(t_ref, 4), "sdpa_tflops": round(fl / t_ref / 1e9, 1),
                      "vs_sdpa": round(t_ref / t_ours, 3)})
        rows.append(r)
    return rows


def bench_ln(nat, iters, flush, peaks, cases, ref):
    rows = []
    for name, M, D in _sel(LN_CASES, cases):
        x = torch.randn(M, D, device="cuda", dtype=torch.bfloat16)
        y = torch.empty_like(x)
        sh = torch.randn(1, D, device="cuda")
        scl = torch.randn(1, D, device="cuda")
        t = time_fn(lambda: nat.ln_modulate(x, out=y, shift=sh, scale=scl), iters, flush=flush)
        byts = 2 * M * D * 2
        rows.append({"kernel": "ln_modulate", "shape": name, "ms": round(t, 4),
                     "gbs": round(byts / t / 1e6, 1),
                     "frac_of_measured_hbm": round(byts / t / 1e6 / peaks["hbm_gbs"], 3)})
    return rows


GEMV_CASES = [("flux_double_mod", 1, 2 * 6 * 3072, 3072), ("flux_all_mod", 1, 19 * 12 * 3072, 3072)]


def bench_gemv(nat, iters, flush, peaks, cases, ref):
    """adaLN modulation GEMVs (batch 1): weight bytes streamed once per call."""
    rows = []
    for name, B, N, K in _sel(GEMV_CASES, cases):
        W = torch.randn(N, K, device="cuda", dtype=torch.bfloat16)
        x = torch.randn(B, K, device="cuda")
        y = torch.empty(B, N, device="cuda")
        t = time_fn(lambda: nat.gemv(W, x, None, y, True, False), iters, flush=flush)
        byts = N * K * 2
        rows.append({"kernel": "gemv", "shape": name, "ms": round(t, 4), "gbs": round(byts / t / 1e6, 1),
                     "frac_of_measured_hbm": round(byts / t / 1e6 / peaks["hbm_gbs"], 3)})
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="gemm,attn,ln")
    ap.add_argument("--cases", default="")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--no-ref", action="store_true")
    ap.add_argument("--split-sweep", action="store_true", help="small-M GEMMs: time every forced split-K count")
    ap.add_argument("--out", default=None, help="also write the rows as JSON here")
    args = ap.parse_args(argv)
    from difflet_b200 import _native
    from difflet_b200.ops.fused import _lib
    from difflet_b200.utils.peaks import load_peaks

    nat = _lib()  # the native module with the DIFFLET_* kernel switches applied
    peaks = load_peaks()
    flush = torch.empty(256 * 1024 * 1024 // 4, device="cuda", dtype=torch.float32)
    only = set(args.only.split(","))
    cases = set(c for c in args.cases.split(",") if c)
    ref = not args.no_ref
    rows = []
    if "gemm" in only:
        rows += bench_gemm(nat, args.iters, flush, peaks, cases, ref, args.split_sweep)
    if "attn" in only:
        rows += bench_attn(nat, args.iters, flush, peaks, cases, ref)
    if "ln" in only:
        rows += bench_ln(nat, args.iters, flush, peaks, cases, ref)
    if "qkv" in only:
        rows += bench_qkv(nat, args.iters, flush, peaks, cases, ref)
    if "gemv" in only:
        rows += bench_gemv(nat, args.iters, flush, peaks, cases, ref)
    if "mx" in only:
        rows += bench_mx(nat, args.iters, flush, peaks, cases, ref)
    if "conv" in only:
        rows += bench_conv(nat, args.iters, flush, peaks, cases, ref)
    _native.check_device_errors()
    for r in rows:
        print(json.dumps(r))
    if args.out:
        with open(args.out, "w") as f:
            json.dump({"peaks": peaks, "rows": rows}, f, indent=1)


if __name__ == "__main__":
    main()
