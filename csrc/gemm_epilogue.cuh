// Shared GEMM epilogue for the tcgen05 GEMMs (bf16 and MXFP8): tile raster,
// bias, GELU-tanh / SiLU on a column window, residual + gate * y, bf16 / f32
// stores, and an optional row scatter into peer ranks' buffers (tensor-parallel
// partial sums land directly at the rank that owns each row).
#pragma once
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
};

DFL_DEVICE void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  int group_tiles = kGroupM * num_n;
  int g = t / group_tiles;
  int first_m = g * kGroupM;
  int gm = min(kGroupM, num_m - first_m);
  int r = t - g * group_tiles;
  mb = first_m + (r % gm);
  nb = r / gm;
}

template <int EPI, bool OUT_F32>
DFL_DEVICE void epilogue_chunk(const uint32_t (&r)[32], int row, int col0, int M, int N,
                               const EpiParams& p) {
  if (row >= M) return;
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * p.alpha;
  const bool full = (col0 + 32 <= N);
  if (p.bias != nullptr) {
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

}  // namespace dfl
