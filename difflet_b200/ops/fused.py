"""Fused device ops used by every model: one entry point, two implementations.

CUDA tensors go to the sm_100a kernels in ``csrc/`` (through ``_native``);
CPU tensors go to a plain PyTorch implementation of the same math, which is
the oracle the kernel tests compare against and which also runs in float64 for
the tiny-model parity check.  There is no silent fallback: a CUDA tensor with a
missing extension raises.

Ops:
  linear        y = epi(x W^T + b): epi in {none, gelu (column window), silu,
                gate_resid (resid + gate[b] * y)}; strided outputs allowed
  ln_modulate   LayerNorm / RMSNorm (+affine) (* (1 + scale) + shift)
  qkv_scatter   per-head / across-heads q,k RMSNorm + RoPE + scatter to
                head-major (or token-major) destinations, one per rank
  linear_qkv    linear whose q/k/v column blocks go through qkv_scatter inside the
                GEMM epilogue (no round trip of the qkv rows through HBM)
  linear_group  two linear / linear_qkv calls with one epilogue kind as one launch
  row_sumsq     per-row sums of squares of q / k column blocks (TP across-heads RMS)
  attention     softmax(scale q k^T) v with key window and LSE
  gemv          modulation linears (M <= 8), f32 in/out, optional SiLU
  euler_step    x += dt * (u + s (c - u)) on f32 latents (+ bf16 mirror)
  timestep_embed sinusoidal features
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from difflet_b200 import envs

EPI_NONE, EPI_GELU, EPI_GATE_RESID, EPI_SILU, EPI_SWIGLU, EPI_QKV = 0, 1, 2, 3, 4, 5
_ACT = {None: EPI_NONE, "none": EPI_NONE, "gelu": EPI_GELU, "gelu_tanh": EPI_GELU, "silu": EPI_SILU,
        "swiglu": EPI_SWIGLU}


def swiglu_interleave(w_h: torch.Tensor, w_g: torch.Tensor) -> torch.Tensor:
    """Rows of the value half ``w_h`` and the gate half ``w_g`` ([F, ...] each) interleaved in
    32-row groups [h_32 | g_32 | h_32 | ...]: the layout the SwiGLU GEMM epilogue reads."""
    F_ = w_h.shape[0]
    if F_ % 32:
        raise ValueError("SwiGLU width must be a multiple of 32")
    rest = w_h.shape[1:]
    return torch.stack([w_h.reshape(F_ // 32, 32, *rest), w_g.reshape(F_ // 32, 32, *rest)], 1).reshape(2 * F_, *rest)

_nat = None
# Host-side count of native kernel launches (each fused-op call is one launch).
LAUNCHES = [0]


def _lib():
    """The native module, without counting a launch (host-only helpers)."""
    global _nat
    if _nat is None:
        from difflet_b200 import _native

        _nat = _native.require()
        _nat.gemm_set_pair_auto(envs.DIFFLET_GEMM_PAIR != "0")
        _nat.gemm_set_epi_warps(envs.DIFFLET_GEMM_EPI_WARPS)
    _split_workspace(_nat)
    return _nat


_SPLIT_WS = {}


def _split_workspace(nat) -> None:
    """Split-K workspace of the current device (64 MB f32 partial tiles + zeroed counters),
    registered once per device; small-M GEMMs split K across SMs with it."""
    if envs.DIFFLET_GEMM_SPLITK == "0" or not torch.cuda.is_available():
        return
    dev = torch.cuda.current_device()
    if dev in _SPLIT_WS:
        return
    ws = torch.empty(16 << 20, device=f"cuda:{dev}", dtype=torch.float32)
    sem = torch.zeros(1 << 14, device=f"cuda:{dev}", dtype=torch.int32)
    _SPLIT_WS[dev] = (ws, sem)
    nat.gemm_set_split_workspace(ws, sem)


def native():
    LAUNCHES[0] += 1
    return _lib()


def _rows2d(x: torch.Tensor) -> torch.Tensor:
    return x if x.dim() == 2 else x.reshape(-1, x.shape[-1])


class MXWeight:
    """A Linear weight held in MXFP8: FP8 E4M3 [N, K] + blocked E8M0 scales.  ``linear``
    quantizes its input on the fly (``compute="mx"``, block-scaled tensor cores) or
    dequantizes the weight to bf16 per call (``compute="dequant"``, memory only)."""

    def __init__(self, q: torch.Tensor, sf_blocked: torch.Tensor, compute: str = "mx"):
        self.q, self.sf, self.compute = q, sf_blocked, compute

    @classmethod
    def quantize(cls, w: torch.Tensor, compute: str = "mx") -> "MXWeight":
        q, sf = mx_quantize(w.to(torch.bfloat16).contiguous(), blocked=True)
        return cls(q, sf, compute)

    @property
    def shape(self):
        return self.q.shape

    @property
    def device(self):
        return self.q.device

    @property
    def dtype(self):
        return self.q.dtype

    def dequantize(self, dtype=torch.bfloat16) -> torch.Tensor:
        from difflet_b200.ops.mx import dequantize_mx

        N, K = self.q.shape
        return dequantize_mx(self.q, unblock_scales(self.sf, N, K), output_dtype=dtype)

    def to(self, device=None, dtype=None):
        if device is None:
            return self
        return MXWeight(self.q.to(device), self.sf.to(device), self.compute)


# ---------------------------------------------------------------------------
def linear(x, w, b=None, *, out=None, act=None, act_lo=0, act_hi=None, gate=None, resid=None,
           rows_per_batch=0, alpha=1.0, out_f32=False, gate_row_map=None):
    """``act(alpha * x @ w.T + b)`` or ``resid + gate * (...)``.

    x: [M, K]; w: [N, K] (or an ``MXWeight``); b: [N]; gate: f32 [B, N] (rows_per_batch
    rows each); resid: [M, N] (may be ``out``).  ``act`` applies to columns [act_lo, act_hi).
    """
    x2 = _rows2d(x)
    if isinstance(w, MXWeight):
        if w.compute == "mx":
            xq, xs = mx_quantize(x2, blocked=True)
            return linear_mx(xq, xs, w.q, w.sf, b, out=out, act=act, act_lo=act_lo, act_hi=act_hi, gate=gate,
                             resid=resid, rows_per_batch=rows_per_batch, alpha=alpha, out_f32=out_f32)
        w = w.dequantize(x2.dtype if not x2.is_cuda else torch.bfloat16)
    N = w.shape[0]
    act_hi = N if act_hi is None else act_hi
    if x2.is_cuda and envs.DIFFLET_KERNEL_GEMM != "cublas":
        epi = EPI_GATE_RESID if gate is not None else _ACT[act]
        return native().gemm(x2, w, b, out, epi, act_lo, act_hi, gate, rows_per_batch, resid, alpha, out_f32,
                             gate_row_map=gate_row_map)
    # reference path: the CPU oracle (any dtype), or the cuBLAS A/B baseline on CUDA
    if x2.is_cuda:
        y = torch.matmul(x2, w.t()).float()
    else:
        y = x2 @ w.t().to(x2.dtype)
    y = y * alpha
    if b is not None:
        y = y + b.to(y.dtype)
    if act in ("gelu", "gelu_tanh"):
        y[:, act_lo:act_hi] = F.gelu(y[:, act_lo:act_hi], approximate="tanh")
    elif act == "silu":
        y[:, act_lo:act_hi] = F.silu(y[:, act_lo:act_hi])
    elif act == "swiglu":
        yy = y.view(y.shape[0], N // 64, 2, 32)
        y = (yy[:, :, 0] * F.silu(yy[:, :, 1])).reshape(y.shape[0], N // 2)
    if gate is not None:
        M = y.shape[0]
        if gate_row_map is not None:
            g = gate[:, :N].to(y.dtype)[gate_row_map.long().to(gate.device)]
        else:
            rpb = rows_per_batch if rows_per_batch > 0 else M
            g = gate[:, :N].to(y.dtype).repeat_interleave(rpb, 0)[:M]
        y = resid.to(y.dtype) + g * y
    dt = torch.float32 if out_f32 else (x2.dtype if not x2.is_cuda else torch.bfloat16)
    if out is not None:
        out.copy_(y.to(out.dtype))
        return out
    return y.to(dt)


def ln_modulate(x, *, shift=None, scale=None, w=None, b=None, eps=1e-6, rms=False, rows_per_batch=0,
                out=None, row_map=None, y_peer=None, row0=0, rows=None):
    """``row_map`` (int32 [M]): the shift / scale row of every row (packed sequences).
    ``y_peer`` (device pointers of every rank's ``out``), ``row0`` / ``rows``: normalise only
    rows [row0, row0 + rows) and store them into every rank's buffer (sequence parallelism)."""
    x2 = _rows2d(x)
    if x2.is_cuda:
        return native().ln_modulate(x2, out, w, b, shift, scale, rows_per_batch, eps, rms, row_map,
                                    list(y_peer or []), int(row0), -1 if rows is None else int(rows))
    xf = x2.to(torch.float64 if x2.dtype == torch.float64 else torch.float32)
    if rms:
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    else:
        y = F.layer_norm(xf, (xf.shape[-1],), eps=eps)
    if w is not None:
        y = y * w.to(y.dtype)
    if b is not None:
        y = y + b.to(y.dtype)
    M = y.shape[0]
    rpb = rows_per_batch if rows_per_batch > 0 else M

    def rows(t):
        t = t.to(y.dtype)
        return t[row_map.long().to(t.device)] if row_map is not None else t.repeat_interleave(rpb, 0)[:M]

    if scale is not None:
        y = y * (1 + rows(scale))
    if shift is not None:
        y = y + rows(shift)
    y = y.to(x2.dtype)
    if out is not None:
        out.copy_(y)
        return out
    return y


def _rope_cpu(x, cos, sin, half):
    # x [..., S, dh]; cos/sin [S, dh/2]
    if half:
        d2 = x.shape[-1] // 2
        x1, x2 = x[..., :d2], x[..., d2:]
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1)
    x0, x1 = x[..., 0::2], x[..., 1::2]
    return torch.stack([x0 * cos - x1 * sin, x1 * cos + x0 * sin], -1).flatten(-2)


def qkv_scatter(qkv, *, q_off, k_off, v_off, S_src, H, dh, q_dst, k_dst, v_dst, S_dst, seq_off=0,
                norm_mode=1, wq=None, wk=None, eps=1e-6, cos=None, sin=None, rope_pos_off=0,
                rope_half=False, heads_per_rank=None, token_major=False, kv_replicate=False, q_S_dst=0,
                q_seq_off=0, seg_rows=0, seg1_seq_off=0, seg1_rope_off=0, row_sumsq=None, norm_total=0):
    """Normalise + rotate q/k of a token-major qkv buffer and scatter q/k/v by head.

    ``q_dst`` etc. are lists (one tensor per destination rank; a single-GPU call
    passes one).  Destination layout [B, H_local, S_dst, dh] (or [B, S_dst,
    H_local*dh] when ``token_major``); row ``s`` of the source lands at
    position ``seq_off + s``.  ``heads_per_rank`` splits heads over the list.
    ``kv_replicate`` (gather-KV context parallelism): k and v of all heads go to
    every destination, q only to ``q_dst[0]`` ([B, H, q_S_dst, dh], row
    ``q_seq_off + s``).  ``seg_rows`` > 0: rows ``s >= seg_rows`` of each batch form a
    second segment placed at ``seg1_seq_off + (s - seg_rows)`` with RoPE row
    ``seg1_rope_off + (s - seg_rows)`` (a rank's [text ; image] slice of a joint sequence).
    ``norm_mode`` 3: across-heads RMS whose per-row sums of squares over all heads
    (``row_sumsq`` f32 [rows, 2]: q, k; already reduced over tensor-parallel ranks) are
    given; ``norm_total`` = number of values they sum (all heads x dh).
    """
    qkv2 = _rows2d(qkv)
    world = len(q_dst if q_dst is not None else (k_dst if k_dst is not None else v_dst))
    hpr = H if kv_replicate else (heads_per_rank or (H // world))
    # a negative offset skips that stream (q-only / k,v-only passes); its destinations may be None
    q_dst = q_dst if q_dst is not None else [None] * world
    k_dst = k_dst if k_dst is not None else [None] * world
    v_dst = v_dst if v_dst is not None else [None] * world
    if qkv2.is_cuda:
        native().qkv_scatter(qkv2, *_scatter_args(q_off, k_off, v_off, S_src, H, dh, q_dst, k_dst, v_dst, S_dst,
                                                  seq_off, norm_mode, wq, wk, eps, cos, sin, rope_pos_off, rope_half,
                                                  hpr, token_major, kv_replicate, q_S_dst, q_seq_off, seg_rows,
                                                  seg1_seq_off, seg1_rope_off, row_sumsq, norm_total))
        return
    if 0 < seg_rows < S_src:  # oracle: one call per segment
        Bn = qkv2.shape[0] // S_src
        x3 = qkv2.view(Bn, S_src, -1)
        common = dict(q_off=q_off, k_off=k_off, v_off=v_off, H=H, dh=dh, q_dst=q_dst, k_dst=k_dst, v_dst=v_dst,
                      S_dst=S_dst, norm_mode=norm_mode, wq=wq, wk=wk, eps=eps, cos=cos, sin=sin, rope_half=rope_half,
                      heads_per_rank=heads_per_rank, token_major=token_major, kv_replicate=kv_replicate,
                      q_S_dst=q_S_dst)
        n1 = S_src - seg_rows
        rs3 = None if row_sumsq is None else row_sumsq.view(Bn, S_src, 2)
        qkv_scatter(x3[:, :seg_rows].reshape(Bn * seg_rows, -1), S_src=seg_rows, seq_off=seq_off,
                    rope_pos_off=rope_pos_off, q_seq_off=q_seq_off, norm_total=norm_total,
                    row_sumsq=None if rs3 is None else rs3[:, :seg_rows].reshape(-1, 2), **common)
        qkv_scatter(x3[:, seg_rows:].reshape(Bn * n1, -1), S_src=n1, seq_off=seg1_seq_off,
                    rope_pos_off=seg1_rope_off, q_seq_off=q_seq_off + seg_rows, norm_total=norm_total,
                    row_sumsq=None if rs3 is None else rs3[:, seg_rows:].reshape(-1, 2), **common)
        return
    rows = qkv2.shape[0]
    B = rows // S_src
    ct = torch.float64 if qkv2.dtype == torch.float64 else torch.float32
    x = qkv2.to(ct).view(B, S_src, -1)

    def take(off):
        return None if off < 0 else x[..., off:off + H * dh].reshape(B, S_src, H, dh)

    q, k, v = take(q_off), take(k_off), take(v_off)

    def norm(t, wn, which=0):
        if t is None or norm_mode == 0:
            return t
        if norm_mode == 3:
            ss = row_sumsq[:, which].to(ct).view(B, S_src, 1, 1)
            t = t * torch.rsqrt(ss / norm_total + eps)
            return t * wn.to(ct).view(H, dh) if wn is not None else t
        if norm_mode == 1:
            t = t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps)
            return t * wn.to(ct) if wn is not None else t
        tf = t.reshape(B, S_src, H * dh)
        tf = tf * torch.rsqrt(tf.pow(2).mean(-1, keepdim=True) + eps)
        if wn is not None:
            tf = tf * wn.to(ct)
        return tf.view(B, S_src, H, dh)

    q, k = norm(q, wq, 0), norm(k, wk, 1)
    q, k, v = (None if t is None else t.permute(0, 2, 1, 3) for t in (q, k, v))  # B, H, S, dh
    if cos is not None:
        c = cos[rope_pos_off:rope_pos_off + S_src].to(ct)
        s_ = sin[rope_pos_off:rope_pos_off + S_src].to(ct)
        if c.shape[-1] == H * (dh // 2) and H > 1:  # per-head tables [S, H, dh/2] -> over [B, H, S, dh/2]
            c = c.view(S_src, H, dh // 2).transpose(0, 1)
            s_ = s_.view(S_src, H, dh // 2).transpose(0, 1)
        R = 2 * c.shape[-1]
        if R < dh:  # partial rotary: the first R channels rotate, the rest pass through
            rot = lambda t: None if t is None else torch.cat([_rope_cpu(t[..., :R], c, s_, rope_half),  # noqa: E731
                                                              t[..., R:]], -1)
            q, k = rot(q), rot(k)
        else:
            q = None if q is None else _rope_cpu(q, c, s_, rope_half)
            k = None if k is None else _rope_cpu(k, c, s_, rope_half)
    if kv_replicate:
        if q is not None:
            q_dst[0][:, :, q_seq_off:q_seq_off + S_src] = q.to(q_dst[0].dtype)
        for r in range(world):
            for src, dst in ((k, k_dst[r]), (v, v_dst[r])):
                if src is not None:
                    dst[:, :, seq_off:seq_off + S_src] = src.to(dst.dtype)
        return
    for r in range(world):
        hs = slice(r * hpr, (r + 1) * hpr)
        for src, dst in ((q, q_dst[r]), (k, k_dst[r]), (v, v_dst[r])):
            if src is None:
                continue
            part = src[:, hs]
            if token_major:
                dst.view(B, S_dst, hpr, dh)[:, seq_off:seq_off + S_src] = part.permute(0, 2, 1, 3).to(dst.dtype)
            else:
                dst[:, :, seq_off:seq_off + S_src] = part.to(dst.dtype)


def _scatter_args(q_off, k_off, v_off, S_src, H, dh, q_dst, k_dst, v_dst, S_dst, seq_off, norm_mode, wq, wk, eps,
                  cos, sin, rope_pos_off, rope_half, hpr, token_major, kv_replicate, q_S_dst, q_seq_off, seg_rows=0,
                  seg1_seq_off=0, seg1_rope_off=0, row_sumsq=None, norm_total=0):
    """Positional arguments of the native head scatter (after the source rows)."""
    ptr = lambda ts: [0 if t is None else (t if isinstance(t, int) else t.data_ptr()) for t in ts]  # noqa: E731
    return (q_off, k_off, v_off, S_src, H, dh, norm_mode, wq, wk, eps, cos, sin, rope_pos_off, rope_half, hpr,
            ptr(q_dst), ptr(k_dst), ptr(v_dst), S_dst, seq_off, token_major, kv_replicate, q_S_dst, q_seq_off,
            seg_rows, seg1_seq_off, seg1_rope_off, row_sumsq, norm_total)


def row_sumsq(x, off0: int, off1: int, width: int) -> torch.Tensor:
    """f32 [rows, 2]: per-row sums of squares of columns [off_i, off_i + width) (0 for off_i < 0)."""
    x2 = _rows2d(x)
    if x2.is_cuda:
        return native().row_sumsq(x2, off0, off1, width)
    ct = torch.float64 if x2.dtype == torch.float64 else torch.float32
    cols = [x2[:, o:o + width].to(ct).pow(2).sum(1) if o >= 0 else torch.zeros(x2.shape[0], dtype=ct)
            for o in (off0, off1)]
    return torch.stack(cols, 1)


def _qkv_epilogue_ok(sc: dict, act) -> bool:
    """The GEMM epilogue covers per-head RMS (or none), full-width RoPE, dh 64 / 128 and
    head blocks aligned to dh; anything else runs the standalone scatter kernel."""
    if envs.DIFFLET_FUSE_QKV == "0" or envs.DIFFLET_KERNEL_GEMM == "cublas" or act not in (None, "none", "gelu"):
        return False
    dh, H = sc["dh"], sc["H"]
    if dh not in (64, 128) or sc.get("norm_mode", 1) not in (0, 1):
        return False
    if any(o >= 0 and o % dh for o in (sc["q_off"], sc["k_off"], sc["v_off"])):
        return False
    cos = sc.get("cos")
    return cos is None or cos.shape[-1] in (dh // 2, H * dh // 2)


def _qkv_plan(sc: dict) -> bytes:
    """The packed head-scatter description the GEMM's qkv epilogue reads."""
    world = len(next(d for d in (sc.get("q_dst"), sc.get("k_dst"), sc.get("v_dst")) if d is not None))
    kv_rep = sc.get("kv_replicate", False)
    hpr = sc["H"] if kv_rep else (sc.get("heads_per_rank") or sc["H"] // world)
    dst = [sc.get(k) if sc.get(k) is not None else [None] * world for k in ("q_dst", "k_dst", "v_dst")]
    return _lib().qkv_plan(*_scatter_args(
        sc["q_off"], sc["k_off"], sc["v_off"], sc["S_src"], sc["H"], sc["dh"], dst[0], dst[1], dst[2], sc["S_dst"],
        sc.get("seq_off", 0), sc.get("norm_mode", 1), sc.get("wq"), sc.get("wk"), sc.get("eps", 1e-6), sc.get("cos"),
        sc.get("sin"), sc.get("rope_pos_off", 0), sc.get("rope_half", False), hpr, sc.get("token_major", False),
        kv_rep, sc.get("q_S_dst", 0), sc.get("q_seq_off", 0), sc.get("seg_rows", 0), sc.get("seg1_seq_off", 0),
        sc.get("seg1_rope_off", 0)))


def linear_qkv(x, w, b=None, *, scatter: dict, out=None, act=None, act_lo=0, act_hi=None):
    """``linear`` whose q / k / v column blocks are consumed by ``qkv_scatter(**scatter)``.

    On the GPU the head scatter (per-head q/k RMSNorm, RoPE, store by head into every
    destination rank's buffer) runs in the GEMM epilogue straight from the tensor-memory
    accumulator; the other columns get ``act`` on [act_lo, act_hi) and land in the same
    columns of ``out`` (which may be None when q, k and v cover every column).  The
    qkv columns of ``out`` are left unwritten on that path.  Otherwise (CPU oracle,
    unsupported scatter options) the full projection is stored and scattered.
    """
    x2 = _rows2d(x)
    N = w.shape[0]
    act_hi = N if act_hi is None else act_hi
    if x2.is_cuda and _qkv_epilogue_ok(scatter, act) and not (isinstance(w, MXWeight) and w.compute != "mx"):
        plan = _qkv_plan(scatter)
        lo, hi = (act_lo, act_hi) if act == "gelu" else (0, 0)  # non-qkv columns: GELU window or identity
        if isinstance(w, MXWeight):
            xq, xs = mx_quantize(x2, blocked=True)
            native().gemm_mx(xq, xs, w.q, w.sf, b, out, EPI_QKV, lo, hi, None, 0, None, 1.0, False, qkv_plan=plan)
        else:
            native().gemm(x2, w, b, out, EPI_QKV, lo, hi, None, 0, None, 1.0, False, qkv_plan=plan)
        return out
    y = linear(x2, w, b, out=out, act=act, act_lo=act_lo, act_hi=act_hi)
    qkv_scatter(y, **scatter)
    return out if out is not None else y


def _group_epi(c: dict):
    """Epilogue kind of one grouped call, or None when it cannot join a grouped launch."""
    x, w = c["x"], c["w"]
    if not x.is_cuda or isinstance(w, MXWeight):
        return None
    if c.get("scatter") is not None:
        return EPI_QKV if _qkv_epilogue_ok(c["scatter"], c.get("act")) else None
    if c.get("gate") is not None:
        return EPI_GATE_RESID
    act = c.get("act")
    return None if act == "swiglu" else _ACT[act]


def linear_group(calls: list) -> list:
    """Two ``linear`` (or ``linear_qkv``, with a ``scatter`` entry) calls as ONE persistent
    GEMM launch whose grid covers both problems' tiles, e.g. the text- and image-stream
    projections of a dual block (the 512-row text GEMM alone fills a third of the SMs).

    Each call is a dict of ``linear`` keyword arguments plus ``x`` and ``w``; calls that do not
    share an epilogue kind (or use MXFP8 weights) run one after the other.  Returns the outputs.
    """
    epis = [_group_epi(c) for c in calls]
    if (len(calls) != 2 or None in epis or epis[0] != epis[1] or envs.DIFFLET_GEMM_GROUP == "0"
            or envs.DIFFLET_KERNEL_GEMM == "cublas"):
        outs = []
        for c in calls:
            kw = {k: v for k, v in c.items() if k not in ("x", "w", "b")}
            fn = linear_qkv if kw.get("scatter") is not None else linear
            if kw.get("scatter") is None:
                kw.pop("scatter", None)
            outs.append(fn(c["x"], c["w"], c.get("b"), **kw))
        return outs
    epi = epis[0]
    A, Bw, bias, out, lo, hi, gate, rpb, resid, plans = ([] for _ in range(10))
    for c in calls:
        N = c["w"].shape[0]
        A.append(_rows2d(c["x"]))
        Bw.append(c["w"])
        bias.append(c.get("b"))
        out.append(c.get("out"))
        act_lo, act_hi = c.get("act_lo", 0), c.get("act_hi")
        act_hi = N if act_hi is None else act_hi
        if epi == EPI_QKV:
            act_lo, act_hi = (act_lo, act_hi) if c.get("act") == "gelu" else (0, 0)
        lo.append(act_lo)
        hi.append(act_hi)
        gate.append(c.get("gate"))
        rpb.append(c.get("rows_per_batch", 0))
        resid.append(c.get("resid"))
        plans.append(_qkv_plan(c["scatter"]) if epi == EPI_QKV else b"")
    return native().gemm_group(A, Bw, bias, out, epi, lo, hi, gate, rpb, resid, plans)


def kv_split_mode() -> int:
    """Key-range split of the native attention: -1 lets the kernel's model choose (launches
    whose query blocks leave SMs idle run as several key chunks + a log-sum-exp combine)."""
    return -1 if envs.DIFFLET_ATTN_SPLIT != "0" else 1


def attention(q, k, v, scale, *, out=None, lse=None, kv_lo=None, kv_hi=None):
    """softmax(scale * q k^T) v over [B, H, S, dh]; key window [kv_lo[b], kv_hi[b])."""
    if q.is_cuda and envs.DIFFLET_KERNEL_ATTN != "sdpa" and q.shape[-1] == 128:
        return native().attention(q, k, v, float(scale), out, lse, kv_lo, kv_hi, kv_split=kv_split_mode())
    ct = torch.float64 if q.dtype == torch.float64 else torch.float32
    if q.is_cuda and lse is None and kv_lo is None:
        o = F.scaled_dot_product_attention(q, k, v, scale=float(scale))
        if out is not None:
            out.copy_(o)
            return out
        return o
    s = torch.einsum("bhqd,bhkd->bhqk", q.to(ct), k.to(ct)) * scale
    if kv_lo is not None or kv_hi is not None:
        Sk = k.shape[2]
        idx = torch.arange(Sk, device=q.device)
        lo = kv_lo if kv_lo is not None else torch.zeros(q.shape[0], dtype=torch.long, device=q.device)
        hi = kv_hi if kv_hi is not None else torch.full((q.shape[0],), Sk, dtype=torch.long, device=q.device)
        mask = (idx[None] >= lo[:, None].to(idx.dtype)) & (idx[None] < hi[:, None].to(idx.dtype))
        s = s.masked_fill(~mask[:, None, None, :], float("-inf"))
    m = torch.logsumexp(s, -1)
    p = torch.exp(s - m[..., None])
    p = torch.nan_to_num(p, nan=0.0)
    o = torch.einsum("bhqk,bhkd->bhqd", p, v.to(ct))
    if lse is not None:
        lse.copy_(m.to(lse.dtype))
    o = o.to(q.dtype)
    if out is not None:
        out.copy_(o)
        return out
    return o


# --------------------------------------------------------------------------- convolution
def conv_weight(w: torch.Tensor) -> torch.Tensor:
    """torch conv weight [Co, Ci, (kt,) kh, kw] -> the kernel's [Co, taps * Ci] (tap-major t, h, w)."""
    if w.dim() == 4:
        w = w[:, :, None]
    Co, Ci = w.shape[:2]
    return w.permute(0, 2, 3, 4, 1).reshape(Co, -1, Ci).reshape(Co, -1).contiguous()


def conv_cl(x, w2, b=None, *, kt=3, kh=3, kw=3, causal=True, resid=None, silu=False, out=None, valid_t=False,
            valid_h=False, valid_w=False):
    """Stride-1 convolution on channels-last x [N, T, H, W, Ci] with ``conv_weight`` weights;
    zero spatial padding k/2, temporal causal (kt - 1 in front) or symmetric padding;
    ``valid_t``: no temporal padding (x starts with its causal context: T_out = T - kt + 1);
    ``valid_h``: no padding along H (x carries halo rows: H_out = H - kh + 1); ``valid_w`` likewise
    along W (x carries its border columns, e.g. replicate padding: W_out = W - kw + 1).
    Optional bias, SiLU, residual add (y = resid + conv).  CUDA -> tcgen05 implicit GEMM."""
    if x.is_cuda:
        return native().conv3d(x, w2, b, kt, kh, kw, causal, resid, silu, out, valid_t, valid_h, valid_w)
    N, T, H, W, Ci = x.shape
    Co = w2.shape[0]
    ct = torch.float64 if x.dtype == torch.float64 else torch.float32
    w5 = w2.to(ct).view(Co, kt, kh, kw, Ci).permute(0, 4, 1, 2, 3)
    xc = x.to(ct).permute(0, 4, 1, 2, 3)
    pt0, pt1 = (0, 0) if valid_t else ((kt - 1, 0) if causal else (kt // 2, kt // 2))
    ph = 0 if valid_h else kh // 2
    pw = 0 if valid_w else kw // 2
    xc = F.pad(xc, (pw, pw, ph, ph, pt0, pt1))
    y = F.conv3d(xc, w5, None if b is None else b.to(ct))
    if silu:
        y = F.silu(y)
    y = y.permute(0, 2, 3, 4, 1)
    if resid is not None:
        y = y + resid.to(ct)
    if out is not None:
        out.copy_(y.to(out.dtype))
        return out
    return y.to(x.dtype)


def gn_stats(x, G: int, eps: float = 1e-6):
    """GroupNorm statistics of a channels-last clip x [N, T, H, W, C]: f32 [N, G, 2] = (mean,
    1 / sqrt(var + eps)) over every frame, row, column and the group's C / G channels."""
    if x.is_cuda:
        return native().gn_stats(x, int(G), float(eps))
    N, C = x.shape[0], x.shape[-1]
    ct = torch.float64 if x.dtype == torch.float64 else torch.float32
    v = x.to(ct).reshape(N, -1, G, C // G).transpose(1, 2).reshape(N, G, -1)
    mean = v.mean(-1)
    var = ((v - mean[..., None]) ** 2).mean(-1)
    return torch.stack([mean, torch.rsqrt(var + eps)], -1).to(torch.float32 if ct == torch.float32 else ct)


def gn_apply(x, stats, gamma, beta, G: int, *, silu: bool, y, offs=(0, 0, 0)):
    """y[:, ot:ot+T, oh:oh+H, ow:ow+W] = GroupNorm(x) * gamma + beta (+ SiLU) with ``gn_stats``;
    ``gamma`` / ``beta`` f32 [C]."""
    ot, oh, ow = offs
    if x.is_cuda:
        native().gn_apply(x, stats, gamma, beta, int(G), bool(silu), y, int(ot), int(oh), int(ow))
        return y
    N, T, H, W, C = x.shape
    ct = torch.float64 if x.dtype == torch.float64 else torch.float32
    st = stats.to(ct).repeat_interleave(C // G, 1)  # [N, C, 2]
    v = (x.to(ct) - st[:, None, None, None, :, 0]) * st[:, None, None, None, :, 1] * gamma.to(ct) + beta.to(ct)
    if silu:
        v = F.silu(v)
    y[:, ot:ot + T, oh:oh + H, ow:ow + W] = v.to(y.dtype)
    return y


def pad_replicate(y, interior, size):
    """Fill the border of y [N, Ty, Hy, Wy, C] around its interior box (offset ``interior`` =
    (pt, ph, pw), extent ``size`` = (T, H, W)) with the nearest interior element, per dimension."""
    (pt, ph, pw), (T, H, W) = interior, size
    if y.is_cuda:
        native().pad_replicate(y, int(pt), int(ph), int(pw), int(T), int(H), int(W))
        return y
    Ty, Hy, Wy = y.shape[1:4]
    it = torch.arange(Ty).clamp(pt, pt + T - 1)
    ih = torch.arange(Hy).clamp(ph, ph + H - 1)
    iw = torch.arange(Wy).clamp(pw, pw + W - 1)
    y.copy_(y[:, it][:, :, ih][:, :, :, iw])
    return y


def upsample_causal(x, up_t: bool, y, offs=(0, 0, 0)):
    """Nearest 2x along H and W of x [N, T, H, W, C]; with ``up_t`` frame 0 stays one frame and
    every later frame is repeated twice (T_out = 2 T - 1); written into y at offset ``offs``."""
    ot, oh, ow = offs
    if x.is_cuda:
        native().upsample_causal(x, bool(up_t), y, int(ot), int(oh), int(ow))
        return y
    v = x.repeat_interleave(2, 2).repeat_interleave(2, 3)
    if up_t and x.shape[1] > 1:
        v = torch.cat([v[:, :1], v[:, 1:].repeat_interleave(2, 1)], 1)
    y[:, ot:ot + v.shape[1], oh:oh + v.shape[2], ow:ow + v.shape[3]] = v
    return y


def vae_chan_norm(x, gamma, y, *, silu=True, halo=0, up=0, up_rows=0, down=0, down_rows=0):
    """Channels-last RMS over the channels of each pixel (``x / max(|x|, 1e-12) * sqrt(C) * gamma``,
    optional SiLU) of x [F, Hl, W, C] into y [F, Hl + 2 halo, W, C] at row offset ``halo``; on CUDA
    the first / last rows also go to the slabs above / below (``up`` / ``down``: peer pointers of
    their y, 0 = none) -- the halo exchange of a spatially split decode."""
    if x.is_cuda:
        native().vae_chan_norm(x, gamma, y, bool(silu), bool(halo), int(up), int(up_rows), int(down),
                               int(down_rows))
        return y
    ct = torch.float64 if x.dtype == torch.float64 else torch.float32
    xf = x.to(ct)
    v = xf / xf.norm(dim=-1, keepdim=True).clamp_min(1e-12) * (x.shape[-1] ** 0.5) * gamma.to(ct)
    if silu:
        v = F.silu(v)
    y[:, halo:halo + x.shape[1]] = v.to(y.dtype)
    return y


def vae_upsample2x(x, y, *, halo=0, up=0, up_rows=0, down=0, down_rows=0):
    """Nearest 2x (H, W) upsample of channels-last x [F, Hl, W, C] into y [F, 2 Hl + 2 halo, 2 W, C]
    (halo rows to the neighbouring slabs as in ``vae_chan_norm``)."""
    if x.is_cuda:
        native().vae_upsample2x(x, y, bool(halo), int(up), int(up_rows), int(down), int(down_rows))
        return y
    v = x.repeat_interleave(2, dim=1).repeat_interleave(2, dim=2)
    y[:, halo:halo + v.shape[1]] = v.to(y.dtype)
    return y


# --------------------------------------------------------------------------- MXFP8
def block_scales(s_plain: torch.Tensor) -> torch.Tensor:
    """Plain E8M0 scales [R, K/32] -> the tensor-core blocked layout (flat uint8): one
    512-byte atom per (128 rows, 128 K), atoms K-fastest, inside an atom byte
    (r%32)*16 + ((r%128)/32)*4 + (k/32)%4; rows padded to 256 with zeros."""
    R, KB = s_plain.shape
    if KB % 4:
        raise ValueError("blocked MX scales need K to be a multiple of 128")
    Rp = -(-R // 256) * 256
    sp = torch.zeros(Rp, KB, dtype=torch.uint8, device=s_plain.device)
    sp[:R] = s_plain
    return sp.view(Rp // 128, 4, 32, KB // 4, 4).permute(0, 3, 2, 1, 4).contiguous().view(-1)


def unblock_scales(s_blocked: torch.Tensor, R: int, K: int) -> torch.Tensor:
    """Inverse of ``block_scales``: the plain [R, K/32] scales."""
    KB = K // 32
    Rp = s_blocked.numel() // KB
    t = s_blocked.view(Rp // 128, KB // 4, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(Rp, KB)
    return t[:R].contiguous()


def mx_quantize(x: torch.Tensor, blocked: bool = True):
    """bf16 [R, K] -> (FP8 E4M3 [R, K], E8M0 scales: blocked flat, or plain [R, K/32])."""
    x2 = _rows2d(x)
    if x2.is_cuda:
        return native().mx_quantize(x2.contiguous(), blocked)
    from difflet_b200.ops.mx import quantize_mx

    q, s = quantize_mx(x2)
    return q, (block_scales(s) if blocked else s)


def linear_mx(aq, a_sf, bq, b_sf, bias=None, *, out=None, act=None, act_lo=0, act_hi=None, gate=None, resid=None,
              rows_per_batch=0, alpha=1.0, out_f32=False, accumulate=False, out_dtype=None):
    """``act(A B^T + b)`` (or ``resid + gate * (...)``) from MXFP8 operands with blocked
    scales: A [M, K] activations, B [N, K] weights (``mx_quantize(..., blocked=True)``)."""
    M, N = aq.shape[0], bq.shape[0]
    if out_dtype is not None:
        out_f32 = out_dtype == torch.float32
    if aq.is_cuda:
        act_hi = N if act_hi is None else act_hi
        epi = EPI_GATE_RESID if gate is not None else _ACT[act]
        if accumulate:
            y = native().gemm_mx(aq, a_sf, bq, b_sf, bias, None, epi, act_lo, act_hi, gate, rows_per_batch, resid,
                                 alpha, True)
            out.add_(y.to(out.dtype))
            return out
        return native().gemm_mx(aq, a_sf, bq, b_sf, bias, out, epi, act_lo, act_hi, gate, rows_per_batch, resid,
                                alpha, out_f32)
    from difflet_b200.ops.mx import dequantize_mx

    K = aq.shape[1]
    a = dequantize_mx(aq, unblock_scales(a_sf, M, K), output_dtype=torch.float32)
    b = dequantize_mx(bq, unblock_scales(b_sf, N, K), output_dtype=torch.float32)
    y = linear(a, b, bias.float() if bias is not None else None, act=act, act_lo=act_lo, act_hi=act_hi,
               gate=gate, resid=resid.float() if resid is not None else None, rows_per_batch=rows_per_batch,
               alpha=alpha)
    if accumulate:
        out.add_(y.to(out.dtype))
        return out
    if out is not None:
        out.copy_(y.to(out.dtype))
        return out
    return y.to(torch.float32 if out_f32 else torch.bfloat16)


MERGE_FIRST, MERGE_MID, MERGE_LAST = 1, 2, 3


def attention_partial(q, k, v, scale, acc_o, acc_lse, mode, *, out=None, lse=None, kv_lo=None, kv_hi=None):
    """Attention over one key block, merged by log-sum-exp into a running result.

    ``acc_o`` f32 [B, H, Sq, dh], ``acc_lse`` f32 [B, H, Sq].  ``mode`` 1 stores this
    block's normalised output and LSE, 2 merges into them, 3 merges and writes the
    final output to ``out`` (bf16, [B, H, Sq, dh] or any strided view).  Running the
    blocks of a key sequence through modes 1, 2, ..., 3 equals attention over the
    whole sequence (ring attention's online merge,
    difflet/backends/neuron/ops_impl/attention.py:280-301)."""
    if q.is_cuda and q.shape[-1] == 128:
        if mode == MERGE_LAST and out is None:
            out = torch.empty_like(q)
        native().attention(q, k, v, float(scale), out if mode == MERGE_LAST else None, lse, kv_lo, kv_hi,
                           acc_o=acc_o, acc_lse=acc_lse, merge_mode=int(mode))
        return out if mode == MERGE_LAST else acc_o
    ct = torch.float64 if q.dtype == torch.float64 else torch.float32
    B, H, Sq, dh = q.shape
    part_lse = torch.empty(B, H, Sq, dtype=ct, device=q.device)
    o = attention(q.to(ct), k.to(ct), v.to(ct), scale, lse=part_lse, kv_lo=kv_lo, kv_hi=kv_hi).to(ct)
    if mode == MERGE_FIRST:
        new_o, new_lse = o, part_lse
    else:
        prev = acc_lse.to(ct)
        mx = torch.maximum(prev, part_lse)
        safe = torch.where(torch.isinf(mx), torch.zeros_like(mx), mx)
        wp, wc = torch.exp(prev - safe), torch.exp(part_lse - safe)
        s = wp + wc
        new_lse = torch.where(s > 0, safe + torch.log(s), torch.full_like(s, float("-inf")))
        s = torch.where(s > 0, s, torch.ones_like(s))
        new_o = (wp / s)[..., None] * acc_o.to(ct) + (wc / s)[..., None] * o
    if lse is not None:
        lse.copy_(new_lse.to(lse.dtype))
    if mode == MERGE_LAST:
        if out is None:
            return new_o.to(q.dtype)
        out.copy_(new_o.to(out.dtype))
        return out
    acc_o.copy_(new_o.to(acc_o.dtype))
    acc_lse.copy_(new_lse.to(acc_lse.dtype))
    return acc_o


def gemv(W, x, bias=None, *, silu_in=False, silu_out=False, out=None):
    if W.is_cuda:
        x = x.float().contiguous()
        if x.shape[0] <= 8:
            return native().gemv(W, x, bias, out, silu_in, silu_out)
        # the kernel stages at most 8 input rows in shared memory: chunk larger batches
        y = out if out is not None else torch.empty(x.shape[0], W.shape[0], device=x.device)
        for i in range(0, x.shape[0], 8):
            native().gemv(W, x[i:i + 8], bias, y[i:i + 8], silu_in, silu_out)
        return y
    ct = torch.float64 if x.dtype == torch.float64 else torch.float32
    xx = F.silu(x.to(ct)) if silu_in else x.to(ct)
    y = xx @ W.to(ct).t()
    if bias is not None:
        y = y + bias.to(ct)
    if silu_out:
        y = F.silu(y)
    if out is not None:
        out.copy_(y)
        return out
    return y


def euler_step(x32, v, dt, *, x16=None, cond=None, guidance=1.0):
    """x32 += dt * pred, pred = v or v + guidance * (cond - v) (CFG); optional bf16 mirror."""
    if x32.is_cuda:
        native().euler_step(x32, x16, v, cond, float(dt), float(guidance))
        return x32
    pred = v.to(x32.dtype)
    if cond is not None:
        pred = pred + guidance * (cond.to(x32.dtype) - pred)
    x32.add_(pred, alpha=dt)
    if x16 is not None:
        x16.copy_(x32.to(x16.dtype))
    return x32


def guided_step(a, b=None, *, scale=1.0, x, x16=None, last=None, m1=None, m2=None, m_out=None, k_v=0.0,
                e=(1.0, 0.0, 0.0, 0.0, 0.0), g=(1.0, 0.0, 0.0, 0.0, 0.0, 0.0), store_last=False, b_ptr=None,
                swap=False):
    """Guidance combine + sampler update in one pass (``csrc/sched.cu``): v = a + scale (b - a)
    (v = a without b; ``swap``: b is the uncond branch, v = b + scale (a - b)), m = x + k_v v, xc = e . (x, last, m1, m2, m), xn = g . (x, last, m1, m2, m, v);
    x <- xn (f32, in place), x16 <- bf16(xn), last <- xc (``store_last``), m_out <- m.
    On CUDA, ``b_ptr`` (a raw device pointer, e.g. the CFG partner's buffer) replaces ``b``."""
    coeffs = [float(k_v)] + [float(c) for c in e] + [float(c) for c in g]
    if x.is_cuda:
        ptr = int(b_ptr) if b_ptr is not None else (b.data_ptr() if b is not None else 0)
        native().guided_step(a, ptr, float(scale), x, x16, last, m1, m2, m_out, coeffs, bool(store_last),
                             bool(swap))
        return x
    ct = x.dtype
    if b is None:
        v = a.to(ct)
    else:
        u_, c_ = (b, a) if swap else (a, b)
        v = u_.to(ct) + scale * (c_.to(ct) - u_.to(ct))
    m = x + coeffs[0] * v
    z = torch.zeros_like(x)
    u = [x, last if last is not None else z, m1 if m1 is not None else z, m2 if m2 is not None else z, m]
    xc = sum(c * t for c, t in zip(coeffs[1:6], u))
    xn = sum(c * t for c, t in zip(coeffs[6:11], u)) + coeffs[11] * v
    if store_last:
        last.copy_(xc)
    if m_out is not None:
        m_out.copy_(m)
    x.copy_(xn)
    if x16 is not None:
        x16.copy_(xn.to(x16.dtype))
    return x


def timestep_embed(t, dim, *, max_period=10000.0, flip_sin_to_cos=True, downscale_freq_shift=0.0,
                   scale=1.0):
    """Sinusoidal timestep features (diffusers ``get_timestep_embedding`` semantics)."""
    if t.is_cuda:
        return native().timestep_embed(t.float().contiguous(), dim, max_period, flip_sin_to_cos,
                                       downscale_freq_shift, scale)
    ct = torch.float64 if t.dtype == torch.float64 else torch.float32
    half = dim // 2
    ex = -math.log(max_period) * torch.arange(half, dtype=ct) / (half - downscale_freq_shift)
    arg = scale * t.to(ct)[:, None] * torch.exp(ex)[None]
    emb = torch.cat([torch.sin(arg), torch.cos(arg)], -1)
    if flip_sin_to_cos:
        emb = torch.cat([emb[:, half:], emb[:, :half]], -1)
    return emb


def rel_l1(a, b) -> torch.Tensor:
    """sum|a - b| / sum|b| as a 1-element f32 tensor on the device (TeaCache probe)."""
    if a.is_cuda:
        return native().rel_l1(a.contiguous(), b.contiguous())
    ct = torch.float64 if a.dtype == torch.float64 else torch.float32
    den = b.to(ct).abs().sum()
    return ((a.to(ct) - b.to(ct)).abs().sum() / den if den > 0 else den * 0).reshape(1)
