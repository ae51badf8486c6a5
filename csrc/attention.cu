// Flash attention forward for sm_100a (head_dim 128, bf16 in/out, fp32 softmax).
//
// One CTA per (256-query block, head, batch), two 128-row Q tiles in ping-pong:
//   warp 8      TMA producer: Q0/Q1 once, then K_j / V_j tiles (2-stage ring,
//               shared by both Q tiles)
//   warp 9      MMA issuer, in the order  PV0(j-1), QK0(j), PV1(j-1), QK1(j):
//               S_g = Q_g K_j^T into TMEM; P_g (bf16) is written back over S_g
//               by the softmax warps and consumed as the A operand straight
//               from TMEM (tcgen05.mma ... [a_tmem]); O_g += P_g V (V read from
//               smem as an MN-major operand).  tcgen05 operations of one thread
//               complete in order, so when S_g(j) is ready the previous PV_g
//               has finished: no extra barrier guards P reuse or O rescaling.
//   warps 0..3  softmax for Q tile 0; warps 4..7 for Q tile 1 (216 registers each
//               after the setmaxnreg split): one query row per thread, running
//               max in log2 units, exp2 on the SFU, P packed to bf16x2 and
//               stored to TMEM; O_g is rescaled in TMEM only when the
//               max grew by more than 2^8 (a stale max keeps P <= 256, exact
//               after the final 1/l); epilogue normalises and stores rows.
// Optional per-batch key window [kv_lo, kv_hi), natural-log LSE output (ring /
// context-parallel merges), and an output-row scatter into peer ranks' buffers
// (the Ulysses head->sequence all-to-all done by the epilogue's stores).
//
// Reference parity: attention contract of difflet/ops/attention.py:4-128 and
// the CUDA SDPA path difflet/backends/cuda/ops_impl/attention.py:41-86 (scale
// given explicitly, bounded key windows as in
// difflet/backends/neuron/ops_impl/attention.py:212-249, LSE as in :280-301).
#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace {
using namespace dfl;

constexpr int kBM = 128;   // queries per Q tile
constexpr int kBN = 128;   // keys per tile
constexpr int kD = 128;    // head dim
// K and V tiles share one FIFO ring of shared-memory slots, loaded in the order
// K0, V0, K1, V1, ... and freed in the same order (K_j after QK_1(j), V_j after PV_1(j)),
// so a slot is refilled as soon as the tile loaded kRing loads earlier is consumed.
constexpr int kTileBytes = 128 * kD * 2;  // 32 KB (two 16 KB swizzle chunks)
constexpr int kChunk = 16384;

// QT = Q tiles per CTA: 2 (ping-pong, default) or 1 (small grids: twice the CTAs)
template <int QT>
struct AttnSmem {
  // warpgroups 0..QT-1: softmax of Q tile g; last warpgroup: TMA warp, MMA warp, 2 idle warps
  static constexpr int kThreads = 128 * QT + 128;
  static constexpr int kProducerWarp = 4 * QT;
  static constexpr int kMmaWarp = 4 * QT + 1;
  static constexpr uint32_t kTmemCols = QT == 2 ? 512 : 256;
  static constexpr int kQ = 0;                              // QT tiles
  static constexpr int kRing = QT == 2 ? 5 : 6;             // K/V slots (224 KB of smem with Q)
  static constexpr int kKV = kQ + QT * kTileBytes;
  static constexpr int kBar = kKV + kRing * kTileBytes;
  // q_full, kv_full[R], kv_empty[R], s_full[2], p_full[2][2], o_full
  static constexpr int kNumBars = 1 + 2 * kRing + 2 + 4 + 1;
  static constexpr int kTotal = kBar + kNumBars * 8 + 16 + 1024;
};

// TMEM columns: S_g/P_g at [128 g, 128 g + 128), O_g after all S tiles
// (QT=2: S0 0, S1 128, O0 256, O1 384; QT=1: S0 0, O0 128)
__device__ __forceinline__ uint32_t tmem_s_col(int g) { return 128u * g; }
template <int QT>
__device__ __forceinline__ uint32_t tmem_o_col(int g) { return 128u * (QT + g); }

// 2^x on the SFU (PTX ex2.approx.ftz.f32); inputs here are <= 8 after the max shift.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void regs_dec_64() { asm volatile("setmaxnreg.dec.sync.aligned.u32 64;"); }
__device__ __forceinline__ void regs_inc_216() { asm volatile("setmaxnreg.inc.sync.aligned.u32 216;"); }

// Packed f32x2 arithmetic (two lanes of a 64-bit register pair per instruction).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// D[tmem] (+)= A[tmem] * B[smem]  (A: M x K, one row per lane, 2 bf16 per column)
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

struct AttnParams {
  long long o_bs, o_hs, o_ss;
  float* lse;
  int B, H, Sq, Sk;
  float scale_log2;
  const int* kv_lo;
  const int* kv_hi;
  __nv_bfloat16* o;
  __nv_bfloat16* o_peer[DFL_MAX_PEERS];
  int o_world, seg0_len, seg0_per, seg1_per;
  float* acc_o;    // f32 [B, H, Sq, 128] running output (merge modes)
  float* acc_lse;  // f32 [B, H, Sq] running log-sum-exp
  int merge_mode;  // 0 none, 1 first partial, 2 merge, 3 merge + final bf16 store
  int kv_splits;    // > 1: CTA x = query block * kv_splits + chunk, partials to split_o / split_lse
  float* split_o;
  float* split_lse;
};

// Output row address: local, or (Ulysses) the owning rank's buffer.
__device__ __forceinline__ __nv_bfloat16* out_row(const AttnParams& p, int b, int h, int s, int* err = nullptr) {
  if (p.o_world <= 1)
    return p.o + (long long)b * p.o_bs + (long long)h * p.o_hs + (long long)s * p.o_ss;
  int owner, lrow;
  if (s < p.seg0_len) {
    owner = s / p.seg0_per;
    lrow = s - owner * p.seg0_per;
  } else {
    const int s2 = s - p.seg0_len;
    owner = s2 / p.seg1_per;
    lrow = p.seg0_per + (s2 - owner * p.seg1_per);
  }
  if (!DFL_GUARD(owner < p.o_world, err, kKidAttn, 80, s)) return nullptr;
  return p.o_peer[owner] + (long long)b * p.o_bs + (long long)h * p.o_hs + (long long)lrow * p.o_ss;
}

__device__ __forceinline__ void tma_load_4d(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Normalise and store one query row (or merge it by log-sum-exp into the running key-block
// accumulators): the tail shared by the attention kernels' softmax threads.
//   o_t: this row's O accumulator in TMEM (lane = row); have_o: the last PV has completed.
__device__ __forceinline__ void attn_epilogue(const AttnParams& p, int* err, int b, int h, int qrow, uint32_t o_t,
                                              bool ok, int n_tiles, uint64_t* o_full, volatile int* abort_flag,
                                              float m, float l, int merge_mode, float* acc_o, float* acc_lse,
                                              float* lse_out) {
  if (merge_mode != 0) {
    // Partial over one key block, merged by log-sum-exp into a running fp32
    // (acc_o, acc_lse): 1 = first partial (store), 2 = merge and store,
    // 3 = merge and write the final bf16 row (no store to the accumulator).
    const bool have = ok && n_tiles > 0 && mbar_wait(o_full, 0, err, kKidAttn, 123, abort_flag);
    if (have) tc_fence_after();
    const float lse_cur = (have && l > 0.f) ? (m + log2f(l)) * 0.69314718055994531f : -INFINITY;
    const float inv = (have && l > 0.f) ? 1.f / l : 0.f;
    const bool valid = qrow < p.Sq;
    const long long arow = ((long long)b * p.H + h) * p.Sq + qrow;
    float w_prev = 0.f, w_cur = 1.f, lse_new = lse_cur;
    if (merge_mode >= 2 && valid) {
      const float lse_prev = acc_lse[arow];
      const float mx = fmaxf(lse_prev, lse_cur);
      if (mx == -INFINITY) {
        w_prev = 0.f, w_cur = 0.f, lse_new = -INFINITY;
      } else {
        w_prev = expf(lse_prev - mx);
        w_cur = expf(lse_cur - mx);
        const float s = w_prev + w_cur;
        w_prev /= s;
        w_cur /= s;
        lse_new = mx + logf(s);
      }
    } else if (lse_cur == -INFINITY) {
      w_cur = 0.f;
    }
    __nv_bfloat16* op = (valid && merge_mode == 3) ? out_row(p, b, h, qrow, err) : nullptr;
    float* ao = valid ? acc_o + arow * kD : nullptr;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t o_raw[32];
      if (have) {
        tmem_ld_32x32b_x32(o_t + c * 32, o_raw);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) o_raw[e] = 0u;
      }
      if (!valid) continue;
      float o[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) o[e] = __uint_as_float(o_raw[e]) * inv * w_cur;
      if (merge_mode >= 2) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 a = reinterpret_cast<const float4*>(ao + c * 32)[q];
          o[4 * q] += w_prev * a.x;
          o[4 * q + 1] += w_prev * a.y;
          o[4 * q + 2] += w_prev * a.z;
          o[4 * q + 3] += w_prev * a.w;
        }
      }
      if (op != nullptr) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack_bf16x2(o[8 * q + 0], o[8 * q + 1]);
          w.y = pack_bf16x2(o[8 * q + 2], o[8 * q + 3]);
          w.z = pack_bf16x2(o[8 * q + 4], o[8 * q + 5]);
          w.w = pack_bf16x2(o[8 * q + 6], o[8 * q + 7]);
          reinterpret_cast<uint4*>(op + c * 32)[q] = w;
        }
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q)
          reinterpret_cast<float4*>(ao + c * 32)[q] = make_float4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
      }
    }
    if (valid) {
      if (merge_mode != 3) acc_lse[arow] = lse_new;
      if (lse_out) lse_out[arow] = lse_new;
    }
  } else if (ok && n_tiles > 0 && mbar_wait(o_full, 0, err, kKidAttn, 122, abort_flag)) {
    tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    __nv_bfloat16* op = qrow < p.Sq ? out_row(p, b, h, qrow, err) : nullptr;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t o_raw[32];
      tmem_ld_32x32b_x32(o_t + c * 32, o_raw);
      tmem_wait_ld();
      if (op != nullptr) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(o_raw[8 * q + 0]) * inv, __uint_as_float(o_raw[8 * q + 1]) * inv);
          w.y = pack_bf16x2(__uint_as_float(o_raw[8 * q + 2]) * inv, __uint_as_float(o_raw[8 * q + 3]) * inv);
          w.z = pack_bf16x2(__uint_as_float(o_raw[8 * q + 4]) * inv, __uint_as_float(o_raw[8 * q + 5]) * inv);
          w.w = pack_bf16x2(__uint_as_float(o_raw[8 * q + 6]) * inv, __uint_as_float(o_raw[8 * q + 7]) * inv);
          reinterpret_cast<uint4*>(op + c * 32)[q] = w;
        }
      }
    }
    if (lse_out && qrow < p.Sq)
      lse_out[((long long)b * p.H + h) * p.Sq + qrow] =
          l > 0.f ? (m + log2f(l)) * 0.69314718055994531f : -INFINITY;
  } else if (n_tiles == 0 && qrow < p.Sq) {
    __nv_bfloat16* op = out_row(p, b, h, qrow, err);
    if (op != nullptr)
      for (int d = 0; d < kD; ++d) op[d] = __float2bfloat16(0.f);
    if (lse_out) lse_out[((long long)b * p.H + h) * p.Sq + qrow] = -INFINITY;
  }
}

template <int QT>
__global__ void __launch_bounds__(AttnSmem<QT>::kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, AttnParams p, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + AttnSmem<QT>::kBar);
  uint64_t* q_full = bars;
  constexpr int R = AttnSmem<QT>::kRing;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + R;
  uint64_t* s_full = kv_empty + R;
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = p_full + 4;  // p_full[2 g + h]: keys [64 h, 64 h + 64) of P_g stored
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + AttnSmem<QT>::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int h = blockIdx.y, b = blockIdx.z;
  const int splits = p.kv_splits > 1 ? p.kv_splits : 1;
  const int chunk = blockIdx.x % splits;
  const int q0 = (blockIdx.x / splits) * (QT * kBM);
  const int lo = p.kv_lo ? max(0, p.kv_lo[b]) : 0;
  const int hi = p.kv_hi ? min(p.Sk, p.kv_hi[b]) : p.Sk;
  const int tiles_all = hi > lo ? (hi + kBN - 1) / kBN - lo / kBN : 0;
  const int per_chunk = (tiles_all + splits - 1) / splits;
  const int t_first = lo / kBN + chunk * per_chunk;
  const int n_tiles = max(0, min(per_chunk, tiles_all - chunk * per_chunk));
  // split-KV: this CTA's partial goes to its chunk's slot (the merge-mode-1 epilogue)
  const int merge_mode = splits > 1 ? 1 : p.merge_mode;
  const long long split_rows = (long long)p.B * p.H * p.Sq;
  float* const acc_o = splits > 1 ? p.split_o + (long long)chunk * split_rows * kD : p.acc_o;
  float* const acc_lse = splits > 1 ? p.split_lse + (long long)chunk * split_rows : p.acc_lse;
  float* const lse_out = splits > 1 ? nullptr : p.lse;

  if (threadIdx.x == 0) {
    for (int i = 0; i < AttnSmem<QT>::kNumBars; ++i) {
      uint64_t* bar = &bars[i];
      const bool softmax_arrivals = bar >= p_full && bar < p_full + 4;
      mbar_init(bar, softmax_arrivals ? 128 : 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_shared();
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
  }
  if (warp == AttnSmem<QT>::kMmaWarp) {
    tmem_alloc(tmem_slot, AttnSmem<QT>::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Register split for QT = 2 (launch: 384 threads x 168): the TMA / MMA warpgroup gives
  // registers back (64 each), the two softmax warpgroups take them (216 each):
  // 128 * 64 + 256 * 216 = 63488 <= 384 * 168.  Every warp of a warpgroup executes its setmaxnreg,
  // inside its role's branch so that the compiler applies the new limit to that code.
  if (warp == AttnSmem<QT>::kProducerWarp) {
    if constexpr (QT == 2) regs_dec_64();
    // ------------------------------------------------------------ producer
    if (lane == 0 && n_tiles > 0) {
      mbar_arrive_expect_tx(q_full, QT * kTileBytes);
      for (int g = 0; g < QT; ++g)
        for (int c = 0; c < 2; ++c)
          tma_load_4d(smem + AttnSmem<QT>::kQ + g * kTileBytes + c * kChunk, &tq, q_full, c * 64,
                      q0 + g * kBM, h, b);
      // load L = 2 j + which (which 0: K_j, 1: V_j) goes to slot L % R, use (L / R)
      bool issued[R];
      uint32_t par_i[R];
      for (int i = 0; i < R; ++i) issued[i] = false, par_i[i] = 0;
      bool ok = true;
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int k0 = (t_first + j) * kBN;
        for (int which = 0; which < 2; ++which) {
          const int L = 2 * j + which, slot = L % R;
          const uint32_t par = (L / R) & 1;
          if (!mbar_wait(&kv_empty[slot], par ^ 1u, err, kKidAttn, 100 + which, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + AttnSmem<QT>::kKV + slot * kTileBytes;
          const CUtensorMap* map = which == 0 ? &tk : &tv;
          mbar_arrive_expect_tx(&kv_full[slot], kTileBytes);
          for (int c = 0; c < 2; ++c) tma_load_4d(dst + c * kChunk, map, &kv_full[slot], c * 64, k0, h, b);
          issued[slot] = true;
          par_i[slot] = par;
        }
      }
      if (!ok) {  // our own bulk copies must land before the CTA exits
        mbar_wait(q_full, 0, nullptr, 0, 0, nullptr, 200000000LL);
        for (int i = 0; i < R; ++i)
          if (issued[i]) mbar_wait(&kv_full[i], par_i[i], nullptr, 0, 0, nullptr, 200000000LL);
      }
    }
  } else if (warp == AttnSmem<QT>::kMmaWarp) {
    if constexpr (QT == 2) regs_dec_64();
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_qk = make_idesc_bf16_f32(kBM, kBN, 0, 0);
      constexpr uint32_t idesc_pv = make_idesc_bf16_f32(kBM, kD, 0, 1);
      bool ok = mbar_wait(q_full, 0, err, kKidAttn, 110, abort_flag);
      // Descriptors: the high word (strides, swizzle, version) is a compile-time constant and
      // the low field is the start address in 16-byte units (every smem address here is below
      // 2^18 bytes), so a tile / k-step is a 32-bit add on the address field.
      constexpr uint64_t kHiK = make_sdesc_sw128(0, 16, 1024);      // K-major Q / K tiles
      constexpr uint64_t kHiV = make_sdesc_sw128(0, kChunk, 1024);  // MN-major V tiles
      const uint32_t q_lo = smem_u32(smem + AttnSmem<QT>::kQ) >> 4;
      const uint32_t kv_lo = smem_u32(smem + AttnSmem<QT>::kKV) >> 4;
      auto slot_lo = [&](int L) { return kv_lo + (uint32_t)(L % R) * (kTileBytes >> 4); };
      auto issue_qk = [&](int g, int jj) {
        const uint32_t qa = q_lo + (uint32_t)g * (kTileBytes >> 4), ka = slot_lo(2 * jj);
        const uint32_t d_tmem = tmem + tmem_s_col(g);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t o = (uint32_t)((((kk >> 2) * kChunk) + (kk & 3) * 32) >> 4);
          umma_f16_ss(d_tmem, kHiK | (qa + o), kHiK | (ka + o), idesc_qk, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[g]);
      };
      auto issue_pv = [&](int g, int jj) -> bool {
        const uint32_t va = slot_lo(2 * jj + 1);
        const uint32_t o_tmem = tmem + tmem_o_col<QT>(g), p_tmem = tmem + tmem_s_col(g);
        // P_g arrives in two halves: the first 64 keys' MMAs run while the softmax
        // finishes the second half
        for (int hf = 0; hf < 2; ++hf) {
          if (!mbar_wait(&p_full[2 * g + hf], jj & 1, err, kKidAttn, 130 + 2 * g + hf, abort_flag)) return false;
          tc_fence_after();
#pragma unroll
          for (int kq = 0; kq < kBN / 32; ++kq) {
            const int kk = hf * (kBN / 32) + kq;
            umma_f16_ts(o_tmem, p_tmem + kk * 8, kHiV | (va + (uint32_t)((kk * 2048) >> 4)), idesc_pv,
                        (jj > 0 || kk > 0) ? 1u : 0u);
          }
        }
        return true;
      };
      auto wait_load = [&](int L, int detail) {
        return mbar_wait(&kv_full[L % R], (L / R) & 1, err, kKidAttn, detail, abort_flag);
      };
      for (int j = 0; j < n_tiles && ok; ++j) {
        if (!wait_load(2 * j, 113)) { ok = false; break; }
        if (j > 0) {
          if (!wait_load(2 * j - 1, 114)) { ok = false; break; }
          if (!issue_pv(0, j - 1)) { ok = false; break; }
        }
        tc_fence_after();
        issue_qk(0, j);
        if (j > 0) {
          if (QT == 2 && !issue_pv(1, j - 1)) { ok = false; break; }
          umma_commit(&kv_empty[(2 * j - 1) % R]);  // V_{j-1} consumed
        }
        if (QT == 2) issue_qk(1, j);
        umma_commit(&kv_empty[(2 * j) % R]);  // K_j consumed
      }
      if (ok) {
        const int jl = n_tiles - 1;
        if (wait_load(2 * jl + 1, 115) && issue_pv(0, jl) && (QT == 1 || issue_pv(1, jl))) {
          umma_commit(&kv_empty[(2 * jl + 1) % R]);
          umma_commit(o_full);
        }
      }
    }
  } else if (warp >= AttnSmem<QT>::kProducerWarp) {
    if constexpr (QT == 2) regs_dec_64();  // the two idle warps of the last warpgroup
  } else {
    if constexpr (QT == 2) regs_inc_216();
    // ------------------------------------------------------------ softmax groups
    const int g = warp / 4;                 // Q tile of this warpgroup
    const int sub = warp & 3;               // TMEM lane quarter of this warp
    const int row = sub * 32 + lane;        // row within the Q tile == TMEM lane
    const uint32_t lane_base = (uint32_t)(sub * 32) << 16;
    const uint32_t s_t = tmem + lane_base + tmem_s_col(g);
    const uint32_t o_t = tmem + lane_base + tmem_o_col<QT>(g);
    float m = -INFINITY;  // running max (log2 domain)
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      if (!mbar_wait(&s_full[g], j & 1, err, kKidAttn, 120 + g, abort_flag)) { ok = false; break; }
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tmem_ld_32x32b_x32(s_t + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[c * 32]));
      tmem_wait_ld();
      const int k0 = (t_first + j) * kBN;
      if ((k0 < lo) || (k0 + kBN > hi)) {  // edge tile: mask keys outside [lo, hi)
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          const int key = k0 + c;
          if (key < lo || key >= hi) s[c] = -INFINITY;
        }
      }
      const float sc = p.scale_log2;
      const uint64_t sc2 = f2_pack(sc, sc);
      // P of keys [32 qtr, 32 qtr + 32) = 2^(s * scale_log2 - m_use): packed FFMA per pair, then the
      // SFU, bf16x2 into TMEM over S; row sums into rs (2 packed chains)
      auto exp_quarter = [&](int qtr, float m_use, uint64_t (&rs)[2]) {
        const uint64_t nm2 = f2_pack(-m_use, -m_use);
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const uint64_t x2 = f2_fma(f2_pack(s[qtr * 32 + 2 * c], s[qtr * 32 + 2 * c + 1]), sc2, nm2);
          float x0, x1;
          f2_unpack(x2, x0, x1);
          const float e0 = fast_exp2(x0), e1 = fast_exp2(x1);
          rs[c & 1] = f2_add(rs[c & 1], f2_pack(e0, e1));
          pk[c] = pack_bf16x2(e0, e1);
        }
        tmem_st_32x32b_x16(s_t + qtr * 16, pk);
      };
      auto signal_half = [&](int hf) {  // keys [64 hf, 64 hf + 64) of P are in TMEM
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[2 * g + hf]);
      };
      auto add_sums = [&](const uint64_t (&rs)[2]) {
        float a0, a1, b0, b1;
        f2_unpack(rs[0], a0, a1);
        f2_unpack(rs[1], b0, b1);
        l += (a0 + a1) + (b0 + b1);
      };
      // raw-score max over keys [k0, k0 + 64): 8 chains of 3-input max (short dependency depth)
      auto half_max = [&](int k0) {
        float mxa[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) mxa[t] = fmaxf(s[k0 + t], s[k0 + 8 + t]);
#pragma unroll
        for (int c = k0 + 16; c < k0 + 64; c += 16) {
#pragma unroll
          for (int t = 0; t < 8; ++t) mxa[t] = max3(mxa[t], s[c + t], s[c + 8 + t]);
        }
        return fmaxf(fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])),
                     fmaxf(fmaxf(mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7])));
      };
      // O_g *= f (TMEM round trip); O_g is stable whenever this runs (see callers)
      auto rescale_o = [&](float f) {
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          uint32_t o_raw[16];
          tmem_ld_32x32b_x16(o_t + c * 16, o_raw);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) o_raw[e] = __float_as_uint(__uint_as_float(o_raw[e]) * f);
          tmem_st_32x32b_x16(o_t + c * 16, o_raw);
        }
      };
      {
        const float mx = fmaxf(half_max(0), half_max(64));
        const float m_new = fmaxf(m, mx * sc);  // scale > 0: max commutes with it
        // the rescale decision is warp-uniform: tcgen05.ld / st are warp-collective
        const bool need = (j > 0) && __any_sync(0xffffffffu, m_new > m + 8.0f);
        const float m_old = m;
        if (j == 0 || need) m = m_new;
        const float m_use = (m == -INFINITY) ? 0.f : m;
        // O_g is stable: PV_g(j-1) completed before S_g(j) (in-order tcgen05)
        if (need) {
          const float f = (m_old == -INFINITY) ? 0.f : fast_exp2(m_old - m);
          rescale_o(f);
          l *= f;
        }
        uint64_t rs[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
        exp_quarter(0, m_use, rs);
        exp_quarter(1, m_use, rs);
        signal_half(0);
        exp_quarter(2, m_use, rs);
        exp_quarter(3, m_use, rs);
        signal_half(1);
        add_sums(rs);
      }
    }
    attn_epilogue(p, err, b, h, q0 + g * kBM + row, o_t, ok, n_tiles, o_full, abort_flag, m, l, merge_mode,
                  acc_o, acc_lse, lse_out);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == AttnSmem<QT>::kMmaWarp) tmem_dealloc(tmem, AttnSmem<QT>::kTmemCols);
}

// Split-KV combine: one warp per query row merges the kv_splits normalised partials by
// log-sum-exp and writes the bf16 row (Ulysses scatter included) and, if asked, the LSE.
__global__ void __launch_bounds__(256) attn_combine_kernel(AttnParams p) {
  const long long rows = (long long)p.B * p.H * p.Sq;
  const long long r = ((long long)blockIdx.x * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x % 32;
  if (r >= rows) return;
  const int S = p.kv_splits;
  float m = -INFINITY;
  for (int c = 0; c < S; ++c) m = fmaxf(m, p.split_lse[c * rows + r]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float wsum = 0.f;
  if (m != -INFINITY) {
    for (int c = 0; c < S; ++c) {
      const float w = expf(p.split_lse[c * rows + r] - m);
      const float4 o = reinterpret_cast<const float4*>(p.split_o + (c * rows + r) * kD)[lane];
      wsum += w;
      acc.x += w * o.x, acc.y += w * o.y, acc.z += w * o.z, acc.w += w * o.w;
    }
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  const int s = (int)(r % p.Sq), h = (int)((r / p.Sq) % p.H), b = (int)(r / ((long long)p.Sq * p.H));
  uint2 pk;
  pk.x = pack_bf16x2(acc.x * inv, acc.y * inv);
  pk.y = pack_bf16x2(acc.z * inv, acc.w * inv);
  __nv_bfloat16* op = out_row(p, b, h, s);
  if (op != nullptr) reinterpret_cast<uint2*>(op)[lane] = pk;
  if (p.lse && lane == 0) p.lse[r] = wsum > 0.f ? m + logf(wsum) : -INFINITY;
}

int make_tmap_4d(CUtensorMap* map, const void* base, long long S, int H, int B, long long ss,
                 long long hs, long long bs, int box_rows = 128) {
  dfl_host::EncodeTiledFn fn = dfl_host::get_encode_tiled();
  if (!fn) return 999;
  cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)ss * 2, (cuuint64_t)hs * 2, (cuuint64_t)bs * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return (int)fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides,
                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

template <int QT>
int launch_attn(const AttnArgs* a, const AttnParams& p, const CUtensorMap& tq, const CUtensorMap& tk,
                const CUtensorMap& tv, cudaStream_t stream) {
  static bool attr[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 15]) {
    cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         AttnSmem<QT>::kTotal);
    if (e != cudaSuccess) return (int)e;
    if (QT == 2) {  // the setmaxnreg split must fit in the registers the CTA is launched with
      cudaFuncAttributes fa;
      e = cudaFuncGetAttributes(&fa, attn_fwd_kernel<QT>);
      if (e != cudaSuccess) return (int)e;
      if (fa.numRegs * AttnSmem<QT>::kThreads < 128 * 64 + 256 * 216) return -11;
    }
    attr[dev & 15] = true;
  }
  const int splits = p.kv_splits > 1 ? p.kv_splits : 1;
  dim3 grid((a->Sq + QT * kBM - 1) / (QT * kBM) * splits, a->H, a->B);
  attn_fwd_kernel<QT><<<grid, AttnSmem<QT>::kThreads, AttnSmem<QT>::kTotal, stream>>>(tq, tk, tv, p, a->err);
  if (splits > 1) {
    const long long rows = (long long)a->B * a->H * a->Sq;
    attn_combine_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, stream>>>(p);
  }
  return (int)cudaGetLastError();
}

}  // namespace

// Key-range splits: modelled time = waves of CTAs x (one full-range CTA time / s) + the
// split overhead (partial f32 rows written and read back by the combine, CTA start-up),
// fitted on B200: 8 us + 0.4 ns per query row and split; s > 1 only with >= 4 key tiles per
// chunk and a predicted gain of 10 %.  (Measured at 4608 keys: 3 heads 68.6 -> 60.2 us with
// two chunks; 6 and 12 heads are fastest unsplit.)
extern "C" int dfl_attention_plan_splits(const AttnArgs* a) {
  if (a->merge_mode != 0 || a->dh != kD || a->Sk <= 0) return 1;
  int dev = 0;
  cudaGetDevice(&dev);
  const double sms = dfl_host::num_sms(dev);
  const double units = (double)((a->Sq + 2 * kBM - 1) / (2 * kBM)) * a->H * a->B;
  const int kv_tiles = (a->Sk + kBN - 1) / kBN;
  const double t_cta_us = 0.0172 * a->Sk;  // one 256-query CTA over every key (measured: 79 us at 4608)
  const double rows = (double)a->B * a->H * a->Sq;
  int best = 1;
  double best_t = std::ceil(units / sms) * t_cta_us;
  for (int s = 2; s <= 8; ++s) {
    if (kv_tiles / s < 4) break;
    const double t = std::ceil(units * s / sms) * t_cta_us / s + 8.0 + 4.0e-4 * rows * s;
    if (t < best_t * 0.9) best = s, best_t = t;
  }
  return best;
}

extern "C" int dfl_attention(const AttnArgs* a, cudaStream_t stream) {
  if (a->dh != kD) return -2;
  if (a->B <= 0 || a->H <= 0 || a->Sq <= 0 || a->Sk <= 0) return -3;
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  if (!al16(a->q) || !al16(a->k) || !al16(a->v) || !al16(a->o)) return -4;
  if ((a->q_ss | a->q_hs | a->q_bs | a->k_ss | a->k_hs | a->k_bs | a->v_ss | a->v_hs | a->v_bs |
       a->o_ss) % 8)
    return -5;
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_4d(&tq, a->q, a->Sq, a->H, a->B, a->q_ss, a->q_hs, a->q_bs);
  if (rc) return 1000 + rc;
  rc = make_tmap_4d(&tk, a->k, a->Sk, a->H, a->B, a->k_ss, a->k_hs, a->k_bs);
  if (rc) return 2000 + rc;
  rc = make_tmap_4d(&tv, a->v, a->Sk, a->H, a->B, a->v_ss, a->v_hs, a->v_bs);
  if (rc) return 3000 + rc;
  AttnParams p;
  p.o_bs = a->o_bs;
  p.o_hs = a->o_hs;
  p.o_ss = a->o_ss;
  p.lse = a->lse;
  p.B = a->B;
  p.H = a->H;
  p.Sq = a->Sq;
  p.Sk = a->Sk;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.kv_lo = a->kv_lo;
  p.kv_hi = a->kv_hi;
  p.o = reinterpret_cast<__nv_bfloat16*>(a->o);
  p.o_world = a->o_world;
  p.acc_o = a->acc_o;
  p.acc_lse = a->acc_lse;
  p.merge_mode = a->merge_mode;
  if (a->merge_mode != 0 && (!a->acc_o || !a->acc_lse || (reinterpret_cast<uintptr_t>(a->acc_o) & 15))) return -9;
  // seg0_per is also the row offset of a rank's seg1 rows in its own buffer, so it stays 0 for a
  // single-stream sequence (seg0_len 0); only the divisors are kept nonzero (a segment without
  // rows is never divided by)
  p.seg0_len = a->seg0_len;
  p.seg0_per = a->seg0_per;
  p.seg1_per = a->seg1_per > 0 ? a->seg1_per : 1;
  for (int r = 0; r < DFL_MAX_PEERS; ++r)
    p.o_peer[r] = reinterpret_cast<__nv_bfloat16*>(r < a->o_world ? a->o_peer[r] : nullptr);
  if (a->o_world > 1) {
    if (a->o_world > DFL_MAX_PEERS) return -6;
    if (a->seg0_len < 0 || a->seg0_per < 0 || a->seg1_per < 0) return -7;
    if (a->seg0_per * a->o_world != a->seg0_len) return -7;  // seg0_per is 0 exactly when seg0_len is
    if (a->seg1_per * a->o_world != a->Sq - a->seg0_len) return -7;
    for (int r = 0; r < a->o_world; ++r)
      if (!a->o_peer[r] || (reinterpret_cast<uintptr_t>(a->o_peer[r]) & 15)) return -8;
  }
  p.kv_splits = a->kv_splits > 1 ? a->kv_splits : 1;
  p.split_o = a->split_o;
  p.split_lse = a->split_lse;
  if (p.kv_splits > 1) {
    if (a->merge_mode != 0 || !a->split_o || !a->split_lse || (reinterpret_cast<uintptr_t>(a->split_o) & 15))
      return -10;
    return launch_attn<2>(a, p, tq, tk, tv, stream);  // 256-row query blocks, split key ranges
  }
  // Two ping-pong Q tiles per CTA unless that leaves more than half the SMs idle:
  // then one Q tile per CTA doubles the CTA count while still fitting one wave.
  int dev = 0;
  cudaGetDevice(&dev);
  const int sms = dfl_host::num_sms(dev);
  const long long ctas2 = (long long)((a->Sq + 2 * kBM - 1) / (2 * kBM)) * a->H * a->B;
  if (ctas2 * 2 <= sms) return launch_attn<1>(a, p, tq, tk, tv, stream);
  return launch_attn<2>(a, p, tq, tk, tv, stream);
}
