// Memory-bound fused kernels for sm_100a:
//   * adaLN LayerNorm / RMSNorm with optional affine and (1 + scale) / shift
//     modulation (fp32 statistics, one warp per row, 16-byte vector IO)
//   * q/k RMSNorm (per head or across heads) + RoPE + scatter of q/k/v to a
//     head-major layout; with a table of per-rank destination pointers the
//     same pass is the Ulysses sequence->head all-to-all (NVLink stores)
//   * GEMV for adaLN / timestep-embedding linears (M <= 8)
//   * flow-matching Euler update with optional CFG combine
//   * sinusoidal timestep features
//
// Reference parity: adaLN-Zero / Single / Continuous
// (difflet/layers/normalization.py:38-190), q/k CustomRMSNorm + RoPE
// (difflet/models/flux/modeling_flux.py:1083-1084,1249-1252;
// difflet/backends/_torch_megatron/embeddings.py:13-33), Wan across-heads RMS
// (difflet/models/wan/modeling_wan.py:564-590), Ulysses seq_to_heads
// (difflet/backends/neuron/ops_impl/collectives.py:276-289), timestep
// projection (difflet/layers/embeddings.py:247-420), Euler / CFG combine
// (difflet/models/flux/pipeline.py:370-420).
#include "common.cuh"
#include "kernels.h"

namespace {
using namespace dfl;

// ---------------------------------------------------------------------------
// LayerNorm / RMSNorm + modulation.  One warp per row; D <= 32 * 8 * kMaxVec.
// ---------------------------------------------------------------------------
constexpr int kMaxVec = 24;  // 24 x 8 bf16 per lane -> D <= 6144

__device__ __forceinline__ void unpack_bf16x8(const uint4& w, float (&f)[8]) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const float2 t = unpack_bf16x2(ws[h]);
    f[2 * h] = t.x;
    f[2 * h + 1] = t.y;
  }
}

// One 8-value output vector: (x - mean) * rstd [* w + b] [* (1 + scale) + shift], stored
// locally or (sequence-parallel all-gather) into every rank's buffer.
__device__ __forceinline__ void ln_store_vec(const LnModArgs& a, int row, int vi, const uint4& raw, float mean,
                                             float rstd, const float* sh, const float* sc, const __nv_bfloat16* w,
                                             const __nv_bfloat16* bb, uint4* y4) {
  const int c0 = vi * 8;
  float o[8];
  unpack_bf16x8(raw, o);
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j] = (o[j] - mean) * rstd;
  if (w) {
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] *= __bfloat162float(w[c0 + j]);
  }
  if (bb) {
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] += __bfloat162float(bb[c0 + j]);
  }
  if (sc) {
    float4 s0 = *reinterpret_cast<const float4*>(sc + c0);
    float4 s1 = *reinterpret_cast<const float4*>(sc + c0 + 4);
    float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] *= (1.f + s[j]);
  }
  if (sh) {
    float4 s0 = *reinterpret_cast<const float4*>(sh + c0);
    float4 s1 = *reinterpret_cast<const float4*>(sh + c0 + 4);
    float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] += s[j];
  }
  uint4 out;
  out.x = pack_bf16x2(o[0], o[1]);
  out.y = pack_bf16x2(o[2], o[3]);
  out.z = pack_bf16x2(o[4], o[5]);
  out.w = pack_bf16x2(o[6], o[7]);
  if (a.y_world > 0) {  // sequence-parallel all-gather: this row into every rank's buffer
    for (int d = 0; d < a.y_world; ++d)
      reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.y_peer[d]) + (long long)row * a.ldy)[vi] = out;
  } else {
    y4[vi] = out;
  }
}

template <int kMaxVec>
__global__ void __launch_bounds__(256) ln_modulate_kernel(LnModArgs a) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (warp >= a.M) return;
  const int row = (int)(a.row0 + warp);
  const int nvec = a.D / 8;  // 16-byte vectors per row
  const uint4* x4 = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.x) +
                                                   (long long)row * a.ldx);
  // the row stays in registers as packed bf16 (4 registers per 8 values): low register
  // count, so more rows per SM are in flight
  uint4 raw[kMaxVec];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    int vi = lane + 32 * i;
    raw[i] = vi < nvec ? x4[vi] : make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    float f[8];
    unpack_bf16x8(raw[i], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) sum += f[j];
  }
  float mean = 0.f;
  if (!a.rms) mean = warp_sum(sum) / (float)a.D;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    int vi = lane + 32 * i;
    if (vi < nvec) {
      float f[8];
      unpack_bf16x8(raw[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float d = f[j] - mean;
        sq += d * d;
      }
    }
  }
  const float rstd = rsqrtf(warp_sum(sq) / (float)a.D + a.eps);
  const int b = a.row_map ? a.row_map[row] : row / a.rows_per_batch;
  const float* sh = a.shift ? a.shift + (long long)b * a.mod_bstride : nullptr;
  const float* sc = a.scale ? a.scale + (long long)b * a.mod_bstride : nullptr;
  const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(a.w);
  const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(a.b);
  uint4* y4 = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.y) + (long long)row * a.ldy);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    int vi = lane + 32 * i;
    if (vi < nvec) ln_store_vec(a, row, vi, raw[i], mean, rstd, sh, sc, w, bb, y4);
  }
}

// Block-per-row variant for wide rows (D >= 1024): 128 threads share a row, each holding
// VPT 16-byte vectors, so registers stay low and many rows per SM are in flight.
template <int VPT>
__global__ void __launch_bounds__(128) ln_modulate_row_kernel(LnModArgs a) {
  __shared__ float red[2][4];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int row = (int)(a.row0 + blockIdx.x);
  const int nvec = a.D / 8;
  const uint4* x4 = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.x) +
                                                   (long long)row * a.ldx);
  uint4 raw[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = t + 128 * i;
    raw[i] = vi < nvec ? x4[vi] : make_uint4(0u, 0u, 0u, 0u);
  }
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    float f[8];
    unpack_bf16x8(raw[i], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) sum += f[j];
  }
  sum = warp_sum(sum);
  if (lane == 0) red[0][warp] = sum;
  __syncthreads();
  const float mean = a.rms ? 0.f : (red[0][0] + red[0][1] + red[0][2] + red[0][3]) / (float)a.D;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    if (t + 128 * i < nvec) {
      float f[8];
      unpack_bf16x8(raw[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = f[j] - mean;
        sq += d * d;
      }
    }
  }
  sq = warp_sum(sq);
  if (lane == 0) red[1][warp] = sq;
  __syncthreads();
  const float rstd = rsqrtf((red[1][0] + red[1][1] + red[1][2] + red[1][3]) / (float)a.D + a.eps);
  const int b = a.row_map ? a.row_map[row] : row / a.rows_per_batch;
  const float* sh = a.shift ? a.shift + (long long)b * a.mod_bstride : nullptr;
  const float* sc = a.scale ? a.scale + (long long)b * a.mod_bstride : nullptr;
  const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(a.w);
  const __nv_bfloat16* bb = reinterpret_cast<const __nv_bfloat16*>(a.b);
  uint4* y4 = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.y) + (long long)row * a.ldy);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int vi = t + 128 * i;
    if (vi < nvec) ln_store_vec(a, row, vi, raw[i], mean, rstd, sh, sc, w, bb, y4);
  }
}

// ---------------------------------------------------------------------------
// q/k norm + RoPE + head-major scatter.  One block of 128 threads per token;
// warp w handles heads w, w + 4, ...; lane holds DH/32 consecutive elements.
// ---------------------------------------------------------------------------
template <int DH>
__device__ __forceinline__ void load_head(const __nv_bfloat16* src, int lane, float (&x)[DH / 32]) {
  constexpr int E = DH / 32;
  if constexpr (E == 4) {
    uint2 w = *reinterpret_cast<const uint2*>(src + lane * 4);
    float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y);
    x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
  } else {
    uint32_t w = *reinterpret_cast<const uint32_t*>(src + lane * 2);
    float2 a = unpack_bf16x2(w);
    x[0] = a.x; x[1] = a.y;
  }
}

template <int DH>
__device__ __forceinline__ void store_head(__nv_bfloat16* dst, int lane, const float (&x)[DH / 32]) {
  constexpr int E = DH / 32;
  if constexpr (E == 4) {
    uint2 w;
    w.x = pack_bf16x2(x[0], x[1]);
    w.y = pack_bf16x2(x[2], x[3]);
    *reinterpret_cast<uint2*>(dst + lane * 4) = w;
  } else {
    *reinterpret_cast<uint32_t*>(dst + lane * 2) = pack_bf16x2(x[0], x[1]);
  }
}

template <int DH>
__device__ __forceinline__ void rope_apply(float (&x)[DH / 32], int lane, const float* cos_row,
                                           const float* sin_row, int half, int rope_dims) {
  constexpr int E = DH / 32;
  if (half && rope_dims > 0 && rope_dims < DH) {
    // partial half-split rotary: channel i < R pairs with i +- R/2 (R/2 a multiple of E,
    // so the partner sits at the same slot e of lane +- R/(2E)); channels >= R pass
    const int R2 = rope_dims / 2;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int i = lane * E + e;
      const int j = i < R2 ? i + R2 : (i < rope_dims ? i - R2 : i);
      const float other = __shfl_sync(0xffffffffu, x[e], j / E);
      if (i < rope_dims) {
        const int fi = i < R2 ? i : i - R2;
        const float c = cos_row[fi], s = sin_row[fi];
        x[e] = (i < R2) ? (x[e] * c - other * s) : (x[e] * c + other * s);
      }
    }
    return;
  }
  if (!half) {
    // interleaved pairs (2i, 2i+1) live in one lane
#pragma unroll
    for (int p = 0; p < E / 2; ++p) {
      int fi = lane * (E / 2) + p;
      float c = cos_row[fi], s = sin_row[fi];
      float x0 = x[2 * p], x1 = x[2 * p + 1];
      x[2 * p] = x0 * c - x1 * s;
      x[2 * p + 1] = x1 * c + x0 * s;
    }
  } else {
    // half-split: element i pairs with i + DH/2, which sits in lane ^ 16
#pragma unroll
    for (int e = 0; e < E; ++e) {
      float other = __shfl_xor_sync(0xffffffffu, x[e], 16);
      int i = lane * E + e;
      int fi = i % (DH / 2);
      float c = cos_row[fi], s = sin_row[fi];
      x[e] = (i < DH / 2) ? (x[e] * c - other * s) : (x[e] * c + other * s);
    }
  }
}

template <int DH>
__global__ void __launch_bounds__(128) qkv_scatter_kernel(QkvScatterArgs a) {
  constexpr int E = DH / 32;
  const int row = blockIdx.x;
  if (row >= a.rows) return;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int b = row / a.S_src;
  const int s = row % a.S_src;
  const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(a.qkv) + (long long)row * a.ld;
  const int H_local = a.heads_per_rank;
  const bool seg1 = a.seg_rows > 0 && s >= a.seg_rows;
  const int dpos = seg1 ? a.seg1_seq_off + (s - a.seg_rows) : a.seq_off + s;
  const int rpos = seg1 ? a.seg1_rope_off + (s - a.seg_rows) : a.rope_pos_off + s;
  const int rope_row = (a.rope_heads > 0 ? a.rope_heads : 1) * ((a.rope_dims > 0 ? a.rope_dims : DH) / 2);
  const float* cos_row = a.cos_t ? a.cos_t + (long long)rpos * rope_row : nullptr;
  const float* sin_row = a.sin_t ? a.sin_t + (long long)rpos * rope_row : nullptr;
  __shared__ float red[2][4];

  // Across-heads RMS (mode 2): sum of squares over the whole q (and k) row.
  float rq = 1.f, rk = 1.f;
  if (a.norm_mode == 2) {
    float sq = 0.f, sk = 0.f;
    for (int h = warp; h < a.H; h += 4) {
      float xq[E], xk[E];
      if (a.q_off >= 0) {
        load_head<DH>(src + a.q_off + h * DH, lane, xq);
#pragma unroll
        for (int e = 0; e < E; ++e) sq += xq[e] * xq[e];
      }
      if (a.k_off >= 0) {
        load_head<DH>(src + a.k_off + h * DH, lane, xk);
#pragma unroll
        for (int e = 0; e < E; ++e) sk += xk[e] * xk[e];
      }
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    if (lane == 0) red[0][warp] = sq, red[1][warp] = sk;
    __syncthreads();
    float tq = red[0][0] + red[0][1] + red[0][2] + red[0][3];
    float tk = red[1][0] + red[1][1] + red[1][2] + red[1][3];
    rq = rsqrtf(tq / (float)(a.H * DH) + a.eps);
    rk = rsqrtf(tk / (float)(a.H * DH) + a.eps);
  } else if (a.norm_mode == 3) {  // sums over all heads, reduced across tensor-parallel ranks
    rq = rsqrtf(a.row_sumsq[2 * row] / (float)a.norm_total + a.eps);
    rk = rsqrtf(a.row_sumsq[2 * row + 1] / (float)a.norm_total + a.eps);
  }

  for (int h = warp; h < a.H; h += 4) {
    const int r = a.kv_replicate ? 0 : h / H_local;
    const int hl = a.kv_replicate ? h : h % H_local;
    const long long dst_off =
        a.out_token_major
            ? ((long long)b * a.S_dst + dpos) * (long long)(H_local * DH) + (long long)hl * DH
            : (((long long)b * H_local + hl) * a.S_dst + dpos) * DH;
    // replicate mode: q rows live in a local buffer of q_S_dst rows at q_seq_off
    const long long q_off_rows =
        a.kv_replicate ? (((long long)b * H_local + hl) * a.q_S_dst + a.q_seq_off + s) * DH : dst_off;
    // q and k
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      float x[E];
      const int off = which == 0 ? a.q_off : a.k_off;
      if (off < 0) continue;  // stream not present (q-only / k,v-only passes)
      load_head<DH>(src + off + h * DH, lane, x);
      const __nv_bfloat16* wn = reinterpret_cast<const __nv_bfloat16*>(which == 0 ? a.wq : a.wk);
      if (a.norm_mode == 1) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) ss += x[e] * x[e];
        float rr = rsqrtf(warp_sum(ss) / (float)DH + a.eps);
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] *= rr;
        if (wn) {
#pragma unroll
          for (int e = 0; e < E; ++e) x[e] *= __bfloat162float(wn[lane * E + e]);
        }
      } else if (a.norm_mode >= 2) {
        float rr = which == 0 ? rq : rk;
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] *= rr;
        if (wn) {
#pragma unroll
          for (int e = 0; e < E; ++e) x[e] *= __bfloat162float(wn[h * DH + lane * E + e]);
        }
      }
      if (cos_row) {
        const int ho = a.rope_heads > 0 ? h * (DH / 2) : 0;
        rope_apply<DH>(x, lane, cos_row + ho, sin_row + ho, a.rope_half, a.rope_dims);
      }
      if (which == 0) {
        store_head<DH>(reinterpret_cast<__nv_bfloat16*>(a.q_dst[r]) + q_off_rows, lane, x);
      } else if (a.kv_replicate) {
        for (int d = 0; d < a.world; ++d) store_head<DH>(reinterpret_cast<__nv_bfloat16*>(a.k_dst[d]) + dst_off, lane, x);
      } else {
        store_head<DH>(reinterpret_cast<__nv_bfloat16*>(a.k_dst[r]) + dst_off, lane, x);
      }
    }
    // v: plain copy into the destination layout
    if (a.v_off >= 0) {
      float x[E];
      load_head<DH>(src + a.v_off + h * DH, lane, x);
      if (a.kv_replicate) {
        for (int d = 0; d < a.world; ++d) store_head<DH>(reinterpret_cast<__nv_bfloat16*>(a.v_dst[d]) + dst_off, lane, x);
      } else {
        store_head<DH>(reinterpret_cast<__nv_bfloat16*>(a.v_dst[r]) + dst_off, lane, x);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// GEMV: one warp per output row, x staged in shared memory (f32).
// ---------------------------------------------------------------------------
// Streaming 16-byte weight load (read once: no L1 allocation).
__device__ __forceinline__ uint4 ld_stream16(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void gemv_accum(const uint4& w, const float* xs, int v, int K, int batch,
                                           float (&acc)[8]) {
  float wf[8];
  unpack_bf16x8(w, wf);
#pragma unroll
  for (int bi = 0; bi < 8; ++bi) {
    if (bi < batch) {
      const float4* xr = reinterpret_cast<const float4*>(xs + bi * K + v * 8);
      float4 x0 = xr[0], x1 = xr[1];
      acc[bi] += wf[0] * x0.x + wf[1] * x0.y + wf[2] * x0.z + wf[3] * x0.w + wf[4] * x1.x + wf[5] * x1.y +
                 wf[6] * x1.z + wf[7] * x1.w;
    }
  }
}

constexpr int kGemvU = 6;  // 16-byte weight loads in flight per lane (memory-level parallelism)

__global__ void __launch_bounds__(256) gemv_kernel(GemvArgs a) {
  extern __shared__ float xs[];  // [batch, K]
  for (int i = threadIdx.x; i < a.batch * a.K; i += blockDim.x) {
    float v = a.x[i];
    xs[i] = a.silu_in ? silu(v) : v;
  }
  __syncthreads();
  const int warps = blockDim.x / 32;
  const int lane = threadIdx.x % 32;
  const int nv = a.K / 8;
  const __nv_bfloat16* bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  for (int n = blockIdx.x * warps + threadIdx.x / 32; n < a.N; n += gridDim.x * warps) {
    const uint4* w4 = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.W) +
                                                     (long long)n * a.ldw);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int v = lane;
    for (; v + 32 * (kGemvU - 1) < nv; v += 32 * kGemvU) {
      uint4 w[kGemvU];
#pragma unroll
      for (int u = 0; u < kGemvU; ++u) w[u] = ld_stream16(w4 + v + 32 * u);
#pragma unroll
      for (int u = 0; u < kGemvU; ++u) gemv_accum(w[u], xs, v + 32 * u, a.K, a.batch, acc);
    }
    for (; v < nv; v += 32) gemv_accum(ld_stream16(w4 + v), xs, v, a.K, a.batch, acc);
#pragma unroll
    for (int bi = 0; bi < 8; ++bi) {
      if (bi >= a.batch) break;
      float s = warp_sum(acc[bi]);
      if (lane == 0) {
        if (bias) s += __bfloat162float(bias[n]);
        if (a.silu_out) s = silu(s);
        a.y[(long long)bi * a.ldy + n] = s;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Euler / CFG
// ---------------------------------------------------------------------------
__global__ void euler_kernel(SchedArgs a) {
  long long i0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  long long stride = (long long)gridDim.x * blockDim.x * 4;
  const __nv_bfloat16* v = reinterpret_cast<const __nv_bfloat16*>(a.v);
  const __nv_bfloat16* c = reinterpret_cast<const __nv_bfloat16*>(a.cond);
  __nv_bfloat16* x16 = reinterpret_cast<__nv_bfloat16*>(a.x16);
  for (long long i = i0; i < a.n; i += stride) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      long long k = i + j;
      if (k < a.n) {
        float pred = __bfloat162float(v[k]);
        if (c) pred = pred + a.guidance * (__bfloat162float(c[k]) - pred);
        float x = a.x32[k] + a.dt * pred;
        a.x32[k] = x;
        if (x16) x16[k] = __float2bfloat16(x);
      }
    }
  }
}

__global__ void timestep_kernel(const float* t, int batch, int dim, float max_period, int flip,
                                float shift, float scale, float* out) {
  int half = dim / 2;
  int b = blockIdx.x;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float expo = -logf(max_period) * (float)i / ((float)half - shift);
    float f = expf(expo);
    float arg = scale * t[b] * f;
    float s = sinf(arg), c = cosf(arg);
    if (flip) {
      out[(long long)b * dim + i] = c;
      out[(long long)b * dim + half + i] = s;
    } else {
      out[(long long)b * dim + i] = s;
      out[(long long)b * dim + half + i] = c;
    }
  }
}

}  // namespace

extern "C" int dfl_ln_modulate(const LnModArgs* a, cudaStream_t stream) {
  if (a->D % 8 || a->D > 32 * 8 * kMaxVec) return -2;
  if ((a->ldx % 8) || (a->ldy % 8)) return -3;
  if ((a->shift || a->scale) && (a->mod_bstride % 4)) return -4;
  if (a->M == 0) return 0;
  if (a->y_world < 0 || a->y_world > DFL_MAX_PEERS) return -5;
  LnModArgs c = *a;
  if (c.rows_per_batch <= 0) c.rows_per_batch = c.M;
  const int nvec = c.D / 8;
  if (nvec >= 128) {  // wide rows: one 128-thread block per row
    const int vpt = (nvec + 127) / 128;
    switch (vpt) {
      case 1: ln_modulate_row_kernel<1><<<c.M, 128, 0, stream>>>(c); break;
      case 2: ln_modulate_row_kernel<2><<<c.M, 128, 0, stream>>>(c); break;
      case 3: ln_modulate_row_kernel<3><<<c.M, 128, 0, stream>>>(c); break;
      case 4: ln_modulate_row_kernel<4><<<c.M, 128, 0, stream>>>(c); break;
      case 5: ln_modulate_row_kernel<5><<<c.M, 128, 0, stream>>>(c); break;
      default: ln_modulate_row_kernel<6><<<c.M, 128, 0, stream>>>(c); break;
    }
    return (int)cudaGetLastError();
  }
  int threads = 256;
  int blocks = (int)((c.M * 32LL + threads - 1) / threads);
  int nv = (c.D / 8 + 31) / 32;
  if (nv <= 1) ln_modulate_kernel<1><<<blocks, threads, 0, stream>>>(c);
  else if (nv <= 2) ln_modulate_kernel<2><<<blocks, threads, 0, stream>>>(c);
  else if (nv <= 4) ln_modulate_kernel<4><<<blocks, threads, 0, stream>>>(c);
  else if (nv <= 8) ln_modulate_kernel<8><<<blocks, threads, 0, stream>>>(c);
  else if (nv <= 12) ln_modulate_kernel<12><<<blocks, threads, 0, stream>>>(c);
  else if (nv <= 16) ln_modulate_kernel<16><<<blocks, threads, 0, stream>>>(c);
  else if (nv <= 20) ln_modulate_kernel<20><<<blocks, threads, 0, stream>>>(c);
  else ln_modulate_kernel<24><<<blocks, threads, 0, stream>>>(c);
  return (int)cudaGetLastError();
}

// One warp per row: sums of squares of two column blocks (16-byte loads).
__global__ void __launch_bounds__(256) row_sumsq_kernel(const __nv_bfloat16* x, long long ld, int rows, int off0,
                                                        int off1, int width, float* out) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int off = i == 0 ? off0 : off1;
    float ss = 0.f;
    if (off >= 0) {
      const uint4* p = reinterpret_cast<const uint4*>(x + (long long)row * ld + off);
      for (int v = lane; v < width / 8; v += 32) {
        float f[8];
        unpack_bf16x8(p[v], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) out[2 * row + i] = ss;
  }
}

extern "C" int dfl_row_sumsq(const void* x, long long ld, int rows, int off0, int off1, int width, float* out,
                             cudaStream_t stream) {
  if (rows == 0) return 0;
  if (width % 8 || ld % 8 || (off0 > 0 && off0 % 8) || (off1 > 0 && off1 % 8)) return -2;
  if (reinterpret_cast<uintptr_t>(x) & 15) return -3;
  const int blocks = (rows * 32 + 255) / 256;
  row_sumsq_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x), ld, rows, off0, off1,
                                                width, out);
  return (int)cudaGetLastError();
}

extern "C" int dfl_qkv_scatter(const QkvScatterArgs* a, cudaStream_t stream) {
  if (a->rows == 0) return 0;
  if (a->world < 1 || a->world > DFL_MAX_PEERS) return -2;
  if (a->kv_replicate ? (a->heads_per_rank != a->H || a->out_token_major) : a->heads_per_rank * a->world != a->H)
    return -3;
  if (a->ld % 8) return -4;
  if (a->norm_mode == 3 && (!a->row_sumsq || a->norm_total <= 0)) return -7;
  if (a->rope_dims && (a->rope_dims > a->dh || (a->rope_dims / 2) % (a->dh / 32) || !a->rope_half || a->rope_heads))
    return -6;
  if (a->dh == 128)
    qkv_scatter_kernel<128><<<a->rows, 128, 0, stream>>>(*a);
  else if (a->dh == 64)
    qkv_scatter_kernel<64><<<a->rows, 128, 0, stream>>>(*a);
  else
    return -5;
  return (int)cudaGetLastError();
}

extern "C" int dfl_gemv(const GemvArgs* a, cudaStream_t stream) {
  if (a->batch < 1 || a->batch > 8) return -2;
  if (a->K % 8 || a->ldw % 8) return -3;
  size_t smem = (size_t)a->batch * a->K * sizeof(float);
  if (smem > 200 * 1024) return -4;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attr = true;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  int blocks = (a->N + 7) / 8;
  int cap = dfl_host::num_sms(dev) * 4;
  if (blocks > cap) blocks = cap;
  gemv_kernel<<<blocks, 256, smem, stream>>>(*a);
  return (int)cudaGetLastError();
}

extern "C" int dfl_euler_step(const SchedArgs* a, cudaStream_t stream) {
  if (a->n == 0) return 0;
  long long blocks = (a->n / 4 + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  euler_kernel<<<(int)blocks, 256, 0, stream>>>(*a);
  return (int)cudaGetLastError();
}

extern "C" int dfl_timestep_embed(const float* t, int batch, int dim, float max_period,
                                  int flip_sin_to_cos, float downscale_freq_shift, float scale,
                                  float* out, cudaStream_t stream) {
  if (dim % 2) return -2;
  timestep_kernel<<<batch, 128, 0, stream>>>(t, batch, dim, max_period, flip_sin_to_cos,
                                             downscale_freq_shift, scale, out);
  return (int)cudaGetLastError();
}
