// Shared GEMM epilogue for the tcgen05 GEMMs (bf16 and MXFP8): tile raster,
// bias, GELU-tanh / SiLU on a column window, residual + gate * y, SwiGLU, bf16 /
// f32 stores, an optional row scatter into peer ranks' buffers (tensor-parallel
// partial sums land directly at the rank that owns each row), and the q/k/v head
// scatter (per-head RMSNorm + RoPE + store into head-major buffers, one per rank:
// the Ulysses sequence->head all-to-all fused into the projection that feeds it).
#pragma once
#include <cstring>

#include "common.cuh"
#include "kernels.h"

namespace dfl {

constexpr int kGroupM = 16;  // tile raster: 16 M-blocks per group for L2 reuse

struct EpiParams {
  void* D;
  long long ldd;
  const __nv_bfloat16* bias;
  int act_lo, act_hi;
  const float* gate;
  long long gate_bstride;
  int rows_per_batch;
  const int* gate_row_map;
  const __nv_bfloat16* resid;
  long long ldr;
  float alpha;
  // Row scatter (out_world > 0): row r goes to out_peer[r / rows_per_rank] at row
  // peer_row_off + r % rows_per_rank (stride ldd); D is unused then.
  void* out_peer[8];
  int out_world;
  int rows_per_rank;
  long long peer_row_off;
  // kEpiQkv: head scatter of the q / k / v column blocks (source rows = GEMM rows)
  QkvScatterArgs qs;
  int* err;  // device error word (bounds-check builds record guard failures here)
};

// Grouped launch: up to kMaxGroup independent GEMMs (same epilogue kind) share one
// persistent grid; their tiles are numbered one problem after the other, so the
// tiles of a small problem (the 512-row text stream of a dual block) fill the
// last wave of a large one instead of running as a mostly idle launch of its own.
constexpr int kMaxGroup = 2;

struct alignas(64) GemmProblem {
  CUtensorMap ta, tb;
  EpiParams ep;
  int M, N, K;
  int num_m, num_n, tiles;  // tiles counts split items (num_m * num_n * splits)
  // Serial split-K (small-M GEMMs that leave SMs idle): the K range of an output tile is
  // cut into `splits` items, adjacent in the tile order so they run concurrently on
  // different SMs.  Item s > 0 waits for sem[tile] == s, adds the f32 partial in ws,
  // and either stores the sum back (sem = s + 1) or, the last item, runs the real
  // epilogue (sem back to 0).  Items of one tile complete in order: the lowest unfinished
  // item never waits, so the persistent grid (every CTA resident) always progresses.
  int splits;
  float* ws;  // f32 [num_m * num_n][128][BN] partial tiles
  int* sem;   // [num_m * num_n] split counters, 0 between launches
};

struct alignas(64) GemmGroup {
  GemmProblem p[kMaxGroup];
  int count, total_tiles;
};

// Problem owning grouped tile t, and the tile's index inside it.
DFL_DEVICE const GemmProblem& group_tile(const GemmGroup& g, int t, int& local) {
  int i = 0;
  while (i + 1 < g.count && t >= g.p[i].tiles) {
    t -= g.p[i].tiles;
    ++i;
  }
  local = t;
  return g.p[i];
}

// K blocks [kb0, kb1) of split item `split` (every item gets at least one block).
DFL_DEVICE void split_k_range(const GemmProblem& P, int split, int BK, int& kb0, int& kb1) {
  const int num_k = (P.K + BK - 1) / BK;
  const int per = (num_k + P.splits - 1) / P.splits;
  kb0 = split * per;
  kb1 = min(num_k, kb0 + per);
}

DFL_DEVICE void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  int group_tiles = kGroupM * num_n;
  int g = t / group_tiles;
  int first_m = g * kGroupM;
  int gm = min(kGroupM, num_m - first_m);
  int r = t - g * group_tiles;
  mb = first_m + (r % gm);
  nb = r / gm;
}

// LIN = false: r already holds the finished linear output (alpha and bias applied).
template <int EPI, bool OUT_F32, bool LIN = true>
DFL_DEVICE void epilogue_chunk(const uint32_t (&r)[32], int row, int col0, int M, int N,
                               const EpiParams& p) {
  if (row >= M) return;
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = LIN ? __uint_as_float(r[j]) * p.alpha : __uint_as_float(r[j]);
  const bool full = (col0 + 32 <= N);
  if (LIN && p.bias != nullptr) {
    if (full) {
      const uint4* b4 = reinterpret_cast<const uint4*>(p.bias + col0);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w = __ldg(b4 + q);
        uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          float2 f = unpack_bf16x2(ws[h]);
          v[q * 8 + 2 * h] += f.x;
          v[q * 8 + 2 * h + 1] += f.y;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) v[j] += __bfloat162float(p.bias[col0 + j]);
    }
  }
  if constexpr (EPI == kEpiGelu || EPI == kEpiSilu) {
    if (col0 + 32 > p.act_lo && col0 < p.act_hi) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        int c = col0 + j;
        if (c >= p.act_lo && c < p.act_hi) v[j] = (EPI == kEpiGelu) ? gelu_tanh(v[j]) : silu(v[j]);
      }
    }
  }
  if constexpr (EPI == kEpiGateResid) {
    int b = p.gate_row_map ? p.gate_row_map[row] : row / p.rows_per_batch;
    if (!DFL_GUARD(b >= 0, p.err, kKidGemm, 71, row)) return;
    const float* g = p.gate + (long long)b * p.gate_bstride;
    const __nv_bfloat16* rs = p.resid + (long long)row * p.ldr;
    if (full) {
      const float4* g4 = reinterpret_cast<const float4*>(g + col0);
      const uint4* r4 = reinterpret_cast<const uint4*>(rs + col0);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float4 ga = __ldg(g4 + 2 * q);
        float4 gb = __ldg(g4 + 2 * q + 1);
        float gs[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
        uint4 rw = r4[q];
        uint32_t rr[4] = {rw.x, rw.y, rw.z, rw.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          float2 rf = unpack_bf16x2(rr[h]);
          v[q * 8 + 2 * h] = rf.x + gs[2 * h] * v[q * 8 + 2 * h];
          v[q * 8 + 2 * h + 1] = rf.y + gs[2 * h + 1] * v[q * 8 + 2 * h + 1];
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) v[j] = __bfloat162float(rs[col0 + j]) + g[col0 + j] * v[j];
    }
  }
  void* dbase = p.D;
  long long drow = row;
  if (p.out_world > 0) {
    const int owner = row / p.rows_per_rank;
    if (!DFL_GUARD(owner < p.out_world, p.err, kKidGemm, 70, row)) return;
    dbase = p.out_peer[owner];
    drow = p.peer_row_off + (row - owner * p.rows_per_rank);
  }
  if constexpr (OUT_F32) {
    float* d = reinterpret_cast<float*>(dbase) + drow * p.ldd + col0;
    if (full) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        reinterpret_cast<float4*>(d)[q] =
            make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) d[j] = v[j];
    }
  } else {
    __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(dbase) + drow * p.ldd + col0;
    if (full) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
        w.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
        w.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
        w.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
        reinterpret_cast<uint4*>(d)[q] = w;
      }
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) d[j] = __float2bfloat16(v[j]);
    }
  }
}

// ---------------------------------------------------------------------------
// q/k/v head scatter.  One thread owns one row of the 128-row tile; a head is
// dh / 32 TMEM chunks of that row.  The linear output is rounded to bf16 first
// (the value the unfused path stores and re-reads), then per-head RMS, the norm
// weight, RoPE (interleaved pairs (2i, 2i+1), or half-split pairs (i, i + dh/2) =
// chunks c and c + dh/64), and a bf16 store to every destination of the head.
DFL_DEVICE void qkv_linear_chunk(const uint32_t (&r)[32], float (&x)[32], const __nv_bfloat16* bias, float alpha) {
#pragma unroll
  for (int j = 0; j < 32; ++j) x[j] = __uint_as_float(r[j]) * alpha;
  if (bias != nullptr) {
    const uint4* b4 = reinterpret_cast<const uint4*>(bias);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w = __ldg(b4 + q);
      uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        float2 f = unpack_bf16x2(ws[h]);
        x[q * 8 + 2 * h] += f.x;
        x[q * 8 + 2 * h + 1] += f.y;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) x[j] = __bfloat162float(__float2bfloat16(x[j]));
}

DFL_DEVICE void qkv_scale_chunk(float (&x)[32], float rr, const __nv_bfloat16* w) {
#pragma unroll
  for (int j = 0; j < 32; ++j) x[j] *= rr;
  if (w != nullptr) {
    const uint4* w4 = reinterpret_cast<const uint4*>(w);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 u = __ldg(w4 + q);
      uint32_t us[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        float2 f = unpack_bf16x2(us[h]);
        x[q * 8 + 2 * h] *= f.x;
        x[q * 8 + 2 * h + 1] *= f.y;
      }
    }
  }
}

DFL_DEVICE void store_bf16x32(__nv_bfloat16* d, const float (&x)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    w.x = pack_bf16x2(x[8 * q + 0], x[8 * q + 1]);
    w.y = pack_bf16x2(x[8 * q + 2], x[8 * q + 3]);
    w.z = pack_bf16x2(x[8 * q + 4], x[8 * q + 5]);
    w.w = pack_bf16x2(x[8 * q + 6], x[8 * q + 7]);
    reinterpret_cast<uint4*>(d)[q] = w;
  }
}

DFL_DEVICE void load_f32x16(const float* p, float (&x)[16]) {
  const float4* p4 = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float4 f = __ldg(p4 + q);
    x[4 * q] = f.x, x[4 * q + 1] = f.y, x[4 * q + 2] = f.z, x[4 * q + 3] = f.w;
  }
}

// Which block (0 q, 1 k, 2 v) and head the column col0 starts, or false for other columns.
DFL_DEVICE bool qkv_locate(const QkvScatterArgs& a, int col0, int& which, int& h) {
  const int offs[3] = {a.q_off, a.k_off, a.v_off};
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    if (offs[i] >= 0 && col0 >= offs[i] && col0 < offs[i] + a.H * a.dh) {
      which = i;
      h = (col0 - offs[i]) / a.dh;
      return true;
    }
  }
  return false;
}

// Per-warp staging for the head scatter: 32 rows of one head, 256 B per row, 16-byte pieces
// stored at piece ^ (row % pieces_per_row) (an XOR swizzle: the 32 rows' stores of one piece
// spread over the banks, and every access stays 16-byte aligned).  A head of 32 consecutive
// rows is then written as whole rows by the warp together (512 contiguous bytes per store
// instruction) instead of 32 scattered 16-byte pieces: full-sized NVLink packets for peer
// destinations, full L2 lines locally.
constexpr int kHeadStageRow = 256;
constexpr int kHeadStageWarp = 32 * kHeadStageRow;
constexpr int kHeadStageBytes = 4 * kHeadStageWarp;  // the four epilogue warps
static_assert(kHeadStageRow % 16 == 0 && kHeadStageWarp % 16 == 0, "16-byte aligned staging rows");

// The epilogue thread of a row is lane (row % 32) of its warp (tiles start at multiples of 32 rows).
DFL_DEVICE int lane_of_row(int row) { return row & 31; }

// 32 values = 4 pieces starting at piece p0 of staging row `lane` (swizzle mask `swz`).
DFL_DEVICE void stage_bf16x32(uint8_t* stage, int lane, int p0, int swz, const float (&x)[32]) {
  uint8_t* row = stage + lane * kHeadStageRow;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    w.x = pack_bf16x2(x[8 * q + 0], x[8 * q + 1]);
    w.y = pack_bf16x2(x[8 * q + 2], x[8 * q + 3]);
    w.z = pack_bf16x2(x[8 * q + 4], x[8 * q + 5]);
    w.w = pack_bf16x2(x[8 * q + 6], x[8 * q + 7]);
    *reinterpret_cast<uint4*>(row + 16 * ((p0 + q) ^ swz)) = w;
  }
}

// RoPE of one 32-column chunk c of interleaved pairs (2p, 2p+1): frequencies c*16 + p.
DFL_DEVICE void rope_interleaved_chunk(float (&x)[32], const float* cs, const float* sn, int c) {
  float cv[16], sv[16];
  load_f32x16(cs + c * 16, cv);
  load_f32x16(sn + c * 16, sv);
#pragma unroll
  for (int p = 0; p < 16; ++p) {
    const float x0 = x[2 * p], x1 = x[2 * p + 1];
    x[2 * p] = x0 * cv[p] - x1 * sv[p];
    x[2 * p + 1] = x1 * cv[p] + x0 * sv[p];
  }
}

// RoPE of half-split pairs: column i of chunk c (first half) with the same column of chunk
// c + dh/64 (second half), frequency c*32 + i.
DFL_DEVICE void rope_half_chunks(float (&x1)[32], float (&x2)[32], const float* cs, const float* sn, int c) {
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    float cv[16], sv[16];
    load_f32x16(cs + c * 32 + hh * 16, cv);
    load_f32x16(sn + c * 32 + hh * 16, sv);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float a1 = x1[hh * 16 + j], a2 = x2[hh * 16 + j];
      x1[hh * 16 + j] = a1 * cv[j] - a2 * sv[j];
      x2[hh * 16 + j] = a2 * cv[j] + a1 * sv[j];
    }
  }
}

template <int DH, class Rel>
DFL_DEVICE void qkv_head_epilogue(uint32_t taddr, int row, int M, int hcol, int which, int h, const EpiParams& ep,
                                  bool last, Rel& release, uint8_t* stage) {
  constexpr int NC = DH / 32;
  const QkvScatterArgs& a = ep.qs;
  const bool row_ok = row < M;
  const int b = row_ok ? row / a.S_src : 0;
  const int s = row_ok ? row - b * a.S_src : 0;
  const __nv_bfloat16* bias = ep.bias ? ep.bias + hcol : nullptr;
  const bool norm = which < 2 && a.norm_mode == 1;
  const __nv_bfloat16* wn =
      norm ? reinterpret_cast<const __nv_bfloat16*>(which == 0 ? a.wq : a.wk) : nullptr;
  // destinations (same addressing as dfl_qkv_scatter)
  const int Hl = a.heads_per_rank;
  const bool seg1 = a.seg_rows > 0 && s >= a.seg_rows;
  const int dpos = seg1 ? a.seg1_seq_off + (s - a.seg_rows) : a.seq_off + s;
  const int rpos = seg1 ? a.seg1_rope_off + (s - a.seg_rows) : a.rope_pos_off + s;
  const int owner = a.kv_replicate ? 0 : h / Hl;
  const int hl = a.kv_replicate ? h : h % Hl;
  const bool valid = row_ok && DFL_GUARD(owner < a.world, ep.err, kKidGemm, 72, h);
  const long long dst_off = a.out_token_major
                                ? ((long long)b * a.S_dst + dpos) * (long long)(Hl * DH) + (long long)hl * DH
                                : (((long long)b * Hl + hl) * a.S_dst + dpos) * DH;
  const long long q_off_rows =
      a.kv_replicate ? (((long long)b * Hl + hl) * a.q_S_dst + a.q_seq_off + s) * DH : dst_off;
  const int ndst = (which > 0 && a.kv_replicate) ? a.world : 1;
  auto dst = [&](int d) -> __nv_bfloat16* {
    if (which == 0) return reinterpret_cast<__nv_bfloat16*>(a.q_dst[owner]) + q_off_rows;
    void* base = which == 1 ? (a.kv_replicate ? a.k_dst[d] : a.k_dst[owner])
                            : (a.kv_replicate ? a.v_dst[d] : a.v_dst[owner]);
    return reinterpret_cast<__nv_bfloat16*>(base) + dst_off;
  };
  const float* cs = nullptr;
  const float* sn = nullptr;
  if (which < 2 && a.cos_t != nullptr && valid) {
    const long long rope_row = (long long)(a.rope_heads > 0 ? a.rope_heads : 1) * (DH / 2);
    const long long o = (long long)rpos * rope_row + (a.rope_heads > 0 ? h * (DH / 2) : 0);
    cs = a.cos_t + o;
    sn = a.sin_t + o;
  }
  const bool half = which < 2 && a.cos_t != nullptr && a.rope_half;  // warp-uniform (cs may be null)
  // chunk c's 32 finished values -> staging row or every destination
  auto emit = [&](int c, const float (&x)[32]) {
    if (stage != nullptr)
      stage_bf16x32(stage, lane_of_row(row), 4 * c, lane_of_row(row) & (DH / 8 - 1), x);
    else if (valid)
      for (int d = 0; d < ndst; ++d) store_bf16x32(dst(d) + c * 32, x);
  };
  if (norm) {
    // One pass over tensor memory: the head's bf16 values (bias, alpha and the bf16 rounding
    // of the unfused projection applied) stay in registers, packed two per word, while the
    // sum of squares accumulates; the accumulator is released after the last load.
    uint32_t hp[DH / 2];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      uint32_t r[32];
      float x[32];
      tmem_ld_32x32b_x32(taddr + c * 32, r);
      tmem_wait_ld();
      if (last && c == NC - 1) release();
      qkv_linear_chunk(r, x, bias ? bias + c * 32 : nullptr, ep.alpha);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        ss += x[2 * j] * x[2 * j] + x[2 * j + 1] * x[2 * j + 1];
        hp[c * 16 + j] = pack_bf16x2(x[2 * j], x[2 * j + 1]);  // exact: x is bf16-rounded
      }
    }
    const float rr = rsqrtf(ss / (float)DH + a.eps);
    auto unpack = [&](int c, float (&x)[32]) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float2 f = unpack_bf16x2(hp[c * 16 + j]);
        x[2 * j] = f.x;
        x[2 * j + 1] = f.y;
      }
    };
    if (!half) {
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        float x[32];
        unpack(c, x);
        qkv_scale_chunk(x, rr, wn ? wn + c * 32 : nullptr);
        if (cs != nullptr) rope_interleaved_chunk(x, cs, sn, c);
        emit(c, x);
      }
    } else {
#pragma unroll
      for (int c = 0; c < NC / 2; ++c) {
        float x1[32], x2[32];
        unpack(c, x1);
        unpack(c + NC / 2, x2);
        qkv_scale_chunk(x1, rr, wn ? wn + c * 32 : nullptr);
        qkv_scale_chunk(x2, rr, wn ? wn + (c + NC / 2) * 32 : nullptr);
        if (cs != nullptr) rope_half_chunks(x1, x2, cs, sn, c);
        emit(c, x1);
        emit(c + NC / 2, x2);
      }
    }
  } else if (!half) {
#pragma unroll 1
    for (int c = 0; c < NC; ++c) {
      uint32_t r[32];
      float x[32];
      tmem_ld_32x32b_x32(taddr + c * 32, r);
      tmem_wait_ld();
      if (last && c == NC - 1) release();
      qkv_linear_chunk(r, x, bias ? bias + c * 32 : nullptr, ep.alpha);
      if (cs != nullptr) rope_interleaved_chunk(x, cs, sn, c);
      emit(c, x);
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < NC / 2; ++c) {
      uint32_t r1[32], r2[32];
      float x1[32], x2[32];
      tmem_ld_32x32b_x32(taddr + c * 32, r1);
      tmem_ld_32x32b_x32(taddr + (c + NC / 2) * 32, r2);
      tmem_wait_ld();
      if (last && c == NC / 2 - 1) release();
      qkv_linear_chunk(r1, x1, bias ? bias + c * 32 : nullptr, ep.alpha);
      qkv_linear_chunk(r2, x2, bias ? bias + (c + NC / 2) * 32 : nullptr, ep.alpha);
      if (cs != nullptr) rope_half_chunks(x1, x2, cs, sn, c);
      emit(c, x1);
      emit(c + NC / 2, x2);
    }
  }
  if (stage != nullptr) {
    // the warp writes its 32 rows of this head: row r's destination comes from lane r
    constexpr int kPieces = DH / 8;  // 16-byte pieces per row
    constexpr int kRowsPerStep = 32 / kPieces;
    const int piece = lane_of_row(row) % kPieces;
    __syncwarp();
    for (int d = 0; d < ndst; ++d) {
      const unsigned long long mine = valid ? reinterpret_cast<unsigned long long>(dst(d)) : 0ull;
#pragma unroll 4
      for (int it = 0; it < 32 / kRowsPerStep; ++it) {
        const int r = it * kRowsPerStep + lane_of_row(row) / kPieces;
        const unsigned long long pr = __shfl_sync(0xffffffffu, mine, r);
        if (pr != 0ull)
          reinterpret_cast<uint4*>(pr)[piece] =
              *reinterpret_cast<const uint4*>(stage + r * kHeadStageRow + 16 * (piece ^ (r & (kPieces - 1))));
      }
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// One accumulator tile row (BN columns starting at col_base) of one thread:
// TMEM -> registers -> epilogue.  `release()` runs once, right after the tile's
// last TMEM load has completed (the accumulator may then be overwritten).
template <int EPI, bool OUT_F32, int BN, class Rel>
DFL_DEVICE void epilogue_tile(uint32_t tbase, int row, int col_base, int M, int N, const EpiParams& ep,
                              Rel&& release, uint8_t* stage = nullptr) {
  const int ncols = min(BN, N - col_base);
  const int nch = (ncols + 31) / 32;  // warp-uniform
  if (nch <= 0) {  // a column slice past N (pair kernel with two slices per tile)
    release();
    return;
  }
  if constexpr (EPI == kEpiSwiGLU) {
    // chunk pairs (h, g) of interleaved 32-column groups -> 32 output columns
#pragma unroll 1
    for (int c = 0; c < nch; c += 2) {
      const int col0 = col_base + c * 32;
      uint32_t rh[32], rg[32];
      tmem_ld_32x32b_x32(tbase + c * 32, rh);
      tmem_ld_32x32b_x32(tbase + (c + 1) * 32, rg);
      tmem_wait_ld();
      if (c + 2 >= nch) release();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float hv = __uint_as_float(rh[j]) * ep.alpha, gv = __uint_as_float(rg[j]) * ep.alpha;
        if (ep.bias) {
          hv += __bfloat162float(ep.bias[col0 + j]);
          gv += __bfloat162float(ep.bias[col0 + 32 + j]);
        }
        rh[j] = __float_as_uint(hv * silu(gv));
      }
      epilogue_chunk<kEpiNone, OUT_F32, false>(rh, row, col0 / 2, M, N / 2, ep);
    }
  } else if constexpr (EPI == kEpiQkv) {
#pragma unroll 1
    for (int c = 0; c < nch;) {
      const int col0 = col_base + c * 32;
      int which = 0, h = 0;
      if (qkv_locate(ep.qs, col0, which, h)) {
        const int hc = ep.qs.dh / 32;
        const bool last = c + hc >= nch;
        if (hc == 4)
          qkv_head_epilogue<128>(tbase + c * 32, row, M, col0, which, h, ep, last, release, stage);
        else
          qkv_head_epilogue<64>(tbase + c * 32, row, M, col0, which, h, ep, last, release, stage);
        c += hc;
      } else {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tbase + c * 32, r);
        tmem_wait_ld();
        if (c + 1 >= nch) release();
        epilogue_chunk<kEpiGelu, false>(r, row, col0, M, N, ep);
        ++c;
      }
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < nch; ++c) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(tbase + c * 32, r);
      tmem_wait_ld();
      if (c + 1 >= nch) release();
      epilogue_chunk<EPI, OUT_F32>(r, row, col_base + c * 32, M, N, ep);
    }
  }
}

// ---------------------------------------------------------------------------
// Split-K item epilogue (the four epilogue warps, 128 threads, named barrier 1).
DFL_DEVICE void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

DFL_DEVICE int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <int EPI, bool OUT_F32, int BN, class Rel>
DFL_DEVICE void epilogue_tile_split(uint32_t tbase, int trow, int row, int col_base, const GemmProblem& P, int tile,
                                    int split, Rel&& release, int* err, volatile int* abort_flag,
                                    volatile int* split_ok) {
  const bool first_thread = trow == 0;
  const bool last = split == P.splits - 1;
  int* sem = P.sem + tile;
  if (split > 0) {  // the previous item's partial must be in ws
    if (first_thread) {
      int ok = 1;
      const long long t0 = clock64();
      while (ld_acquire_gpu(sem) != split) {
        if (*abort_flag || clock64() - t0 > kLocalWaitCycles) {
          record_error(err, kErrMbarTimeout, kKidGemm, 60, split);
          *abort_flag = 1;
          ok = 0;
          break;
        }
      }
      *split_ok = ok;
    }
    epi_bar();
    if (!*split_ok) {  // one shared decision: the TMEM loads below are warp-collective
      release();
      return;
    }
  }
  // The partial tile is stored thread-major: float4 q of chunk c of epilogue thread trow sits at
  // ((c * 8 + q) * 128 + trow), so the 32 lanes of a warp touch 512 consecutive bytes per access
  // (a row-major tile would give each lane its own 32-byte sector).  Loads bypass L1 (the data
  // was written by another SM) and the next chunk's partial is loaded while this one is added.
  float4* const wt = reinterpret_cast<float4*>(P.ws + (size_t)tile * 128 * BN) + trow;
  const int ncols = min(BN, P.N - col_base);
  const int nch = (ncols + 31) / 32;
  float4 nxt[8];
  if (split > 0) {
#pragma unroll
    for (int q = 0; q < 8; ++q) nxt[q] = __ldcg(wt + q * 128);
  }
#pragma unroll 1
  for (int c = 0; c < nch; ++c) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(tbase + c * 32, r);
    tmem_wait_ld();
    if (c + 1 >= nch) release();
    float4* const w4 = wt + (size_t)c * 8 * 128;
    if (split > 0) {
      float4 cur[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) cur[q] = nxt[q];
      if (c + 1 < nch) {
#pragma unroll
        for (int q = 0; q < 8; ++q) nxt[q] = __ldcg(w4 + (8 + q) * 128);
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        r[4 * q] = __float_as_uint(__uint_as_float(r[4 * q]) + cur[q].x);
        r[4 * q + 1] = __float_as_uint(__uint_as_float(r[4 * q + 1]) + cur[q].y);
        r[4 * q + 2] = __float_as_uint(__uint_as_float(r[4 * q + 2]) + cur[q].z);
        r[4 * q + 3] = __float_as_uint(__uint_as_float(r[4 * q + 3]) + cur[q].w);
      }
    }
    if (!last) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        __stcg(w4 + q * 128, make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                         __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3])));
    } else {
      epilogue_chunk<EPI, OUT_F32>(r, row, col_base + c * 32, P.M, P.N, P.ep);
    }
  }
  __threadfence();
  epi_bar();  // every thread's partial (or final rows) is written
  if (first_thread) atomicExch(sem, last ? 0 : split + 1);
}

}  // namespace dfl

// ---------------------------------------------------------------------------
// Host: GemmArgs -> EpiParams with the argument checks shared by every GEMM.
namespace dfl_host {

inline bool misaligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; }

// kEpiQkv plan checks: the fused head scatter covers per-head RMS (or none), full-width
// RoPE, dh 64 / 128, head blocks aligned to dh inside [0, N), bf16 output, no row scatter.
inline int check_qkv_plan(const GemmArgs& a) {
  const QkvScatterArgs* q = a.qkv;
  if (q == nullptr || a.out_f32 || a.out_world > 0) return -20;
  if (q->dh != 64 && q->dh != 128) return -21;
  if (q->norm_mode != 0 && q->norm_mode != 1) return -22;
  if (q->rope_dims != 0 && q->rope_dims != q->dh) return -23;
  if ((q->cos_t == nullptr) != (q->sin_t == nullptr)) return -23;
  if (q->cos_t && (misaligned16(q->cos_t) || misaligned16(q->sin_t))) return -23;
  if (q->S_src <= 0 || q->H <= 0 || q->heads_per_rank <= 0 || q->world < 1 || q->world > DFL_MAX_PEERS) return -24;
  if (q->norm_mode == 1 && ((q->wq && misaligned16(q->wq)) || (q->wk && misaligned16(q->wk)))) return -25;
  const int offs[3] = {q->q_off, q->k_off, q->v_off};
  void* const* dsts[3] = {q->q_dst, q->k_dst, q->v_dst};
  long long covered = 0;
  for (int i = 0; i < 3; ++i) {
    if (offs[i] < 0) continue;
    if (offs[i] % q->dh || (long long)offs[i] + (long long)q->H * q->dh > a.N) return -26;
    covered += (long long)q->H * q->dh;
    // destinations written: q_dst[0] / all ranks (gather-KV replication), else one per head owner
    const int nd = q->kv_replicate ? (i == 0 ? 1 : q->world) : (q->H + q->heads_per_rank - 1) / q->heads_per_rank;
    if (nd > q->world) return -24;
    for (int d = 0; d < nd; ++d)
      if (dsts[i][d] == nullptr || misaligned16(dsts[i][d])) return -27;
  }
  if (a.D == nullptr && covered != a.N) return -28;  // columns outside q / k / v need D
  return 0;
}

inline int fill_epi_params(const GemmArgs& a, dfl::EpiParams& ep) {
  std::memset(&ep, 0, sizeof(ep));
  ep.D = a.D;
  ep.ldd = a.ldd;
  ep.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  ep.act_lo = a.act_lo;
  ep.act_hi = a.act_hi;
  ep.gate = a.gate;
  ep.gate_bstride = a.gate_bstride;
  ep.rows_per_batch = a.rows_per_batch > 0 ? a.rows_per_batch : a.M;
  ep.gate_row_map = a.gate_row_map;
  ep.resid = reinterpret_cast<const __nv_bfloat16*>(a.resid);
  ep.ldr = a.ldr;
  ep.alpha = a.alpha;
  ep.err = a.err;
  if (a.out_world < 0 || a.out_world > DFL_MAX_PEERS) return -9;
  ep.out_world = a.out_world;
  ep.rows_per_rank = a.rows_per_rank > 0 ? a.rows_per_rank : a.M;
  ep.peer_row_off = a.peer_row_off;
  for (int r = 0; r < DFL_MAX_PEERS; ++r) ep.out_peer[r] = r < a.out_world ? a.out_peer[r] : nullptr;
  if (a.out_world > 0) {  // every row needs an owner (the device side does not check in release builds)
    if ((long long)ep.rows_per_rank * a.out_world < a.M) return -10;
    for (int r = 0; r < a.out_world; ++r)
      if (!a.out_peer[r]) return -10;
  }
  if (a.epi == kEpiSwiGLU && (a.N % 64 || a.out_world > 0)) return -11;
  if (a.epi == kEpiQkv) {
    const int rc = check_qkv_plan(a);
    if (rc) return rc;
    ep.qs = *a.qkv;
  }
  return 0;
}

}  // namespace dfl_host
