// Implicit-GEMM convolution on tcgen05 (sm_100a): 2-D and 3-D, stride 1, kernel
// 1 or 3 per axis, channels-last bf16 (N, T, H, W, C), fp32 accumulation in TMEM.
//
//   out[n, t, h, w, co] = bias[co] (+ resid) + sum_{tap, ci} in[n, t+dt-pt, h+dh-ph, w+dw-pw, ci]
//                                                         * wgt[co, tap, ci]
//
// GEMM view: M = output positions, tiled as 128 consecutive w of one (n, t, h) row;
// N = C_out; K = taps x C_in.  For every K step the TMA warp loads the shifted input
// window of one tap (a 5-D tiled load at coordinates offset by the tap; windows that
// fall outside the volume -- the zero padding, including the causal front padding in
// time -- are filled with zeros by the TMA unit) and the matching weight tile; the
// MMA warp accumulates 128 x BN x BK per step; four epilogue warps add the bias and
// the residual and store bf16 rows.  Channel steps of 64 use 128-byte swizzled tiles,
// of 32 (96 / 192-channel VAEs) 64-byte swizzled tiles.
//
// Reference parity: the causal Conv3d / Conv2d stacks of the VAE decoders
// (difflet/models/wan/vae/modeling_vae.py:92-134, difflet/models/flux/vae/
// modeling_vae.py:39-141, difflet/models/hunyuan_video/vae/modeling_vae.py:85-489),
// which the reference runs through cuDNN.
#include "common.cuh"
#include "gemm_epilogue.cuh"
#include "kernels.h"

namespace {
using namespace dfl;

constexpr int BM = 128;
constexpr int kThreads = 192;

DFL_DEVICE void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2, int c3,
                            int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// K-major smem descriptor: 128-byte (BK 64) or 64-byte (BK 32) swizzle, 8-row groups.
template <int BK>
DFL_DEVICE uint64_t make_sdesc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((16u >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(((BK * 2 * 8) >> 4) & 0x3FFFu) << 32;  // 8 rows of BK bf16
  d |= 1ull << 46;
  d |= (BK == 64 ? 2ull : 4ull) << 61;  // SWIZZLE_128B : SWIZZLE_64B
  return d;
}

struct ConvGeom {
  int N, T, H, W, Ci, Co;  // output extents
  int Ti, Hi, Wi;          // input frames / rows / columns
  int kt, kh, kw, pt, ph, pw;
  int wtiles;   // ceil(W / 128)
  int csteps;   // Ci / BK
};

template <int BN, int BK, int STAGES>
struct ConvSmem {
  static constexpr int kA = BM * BK * 2;
  static constexpr int kB = BN * BK * 2;
  static constexpr int kStage = kA + kB;
  static constexpr int kBar = STAGES * kStage;
  static constexpr int kTotal = kBar + (2 * STAGES + 4) * 8 + 16 + 1024;
};

template <int BN, int BK, int STAGES, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    conv_tcgen05_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                        ConvGeom g, EpiParams ep, int* err) {
  using S = ConvSmem<BN, BK, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S::kBar);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int num_m = g.N * g.T * g.H * g.wtiles;
  const int num_n = g.Co / BN;
  const int num_tiles = num_m * num_n;
  const int taps = g.kt * g.kh * g.kw;
  const int num_k = taps * g.csteps;
  const long long M_total = (long long)g.N * g.T * g.H * g.W;
  // accumulator buffers 64-column aligned (96 -> 128, 192 -> 256); allocation a power of two
  constexpr uint32_t kAcc = (BN + 63) / 64 * 64;
  constexpr uint32_t kTmemCols = 2 * kAcc <= 128 ? 128 : 2 * kAcc <= 256 ? 256 : 512;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_shared();
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool issued[STAGES];
      uint32_t issued_parity[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = false, issued_parity[s] = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        const int wt = mb % g.wtiles;
        int rest = mb / g.wtiles;
        const int h = rest % g.H;
        rest /= g.H;
        const int tt = rest % g.T;
        const int n = rest / g.T;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, err, kKidGemm, 210 + stage, abort_flag)) {
            ok = false;
            break;
          }
          const int tap = kb / g.csteps, cs = kb % g.csteps;
          const int dw = tap % g.kw, dh = (tap / g.kw) % g.kh, dt = tap / (g.kw * g.kh);
          uint8_t* sa = smem + stage * S::kStage;
          mbar_arrive_expect_tx(&full_bar[stage], S::kStage);
          // shifted input window (out-of-volume parts are zero-filled by TMA)
          tma_load_5d(sa, &tmap_x, &full_bar[stage], cs * BK, wt * BM + dw - g.pw, h + dh - g.ph, tt + dt - g.pt, n);
          tma_load_2d(sa + S::kA, &tmap_w, &full_bar[stage], kb * BK, nb * BN);
          issued[stage] = true;
          issued_parity[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        for (int s = 0; s < STAGES; ++s)
          if (issued[s]) mbar_wait(&full_bar[s], issued_parity[s], nullptr, 0, 0, nullptr, 200000000LL);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16_f32(BM, BN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, err, kKidGemm, 220 + acc, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kAcc;
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, err, kKidGemm, 230 + stage, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * S::kStage);
          const uint32_t b_addr = a_addr + S::kA;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16_ss(d_tmem, make_sdesc<BK>(a_addr + k * 32), make_sdesc<BK>(b_addr + k * 32), idesc,
                        (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    const int sub = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      if (!mbar_wait(&tfull_bar[acc], acc_phase, err, kKidGemm, 240 + acc, abort_flag)) break;
      tc_fence_after();
      const int wt = mb % g.wtiles;
      const long long row_base = (long long)(mb / g.wtiles) * g.W;  // ((n*T + t)*H + h) * W
      const int w = wt * BM + sub * 32 + lane;
      const long long row = w < g.W ? row_base + w : M_total;  // masked rows are skipped
      const uint32_t tbase = tmem_base + ((uint32_t)(sub * 32) << 16) + acc * kAcc;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tbase + c * 32, r);
        tmem_wait_ld();
        epilogue_chunk<EPI, false>(r, (int)row, nb * BN + c * 32, (int)M_total, g.Co, ep);
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

int make_tmap_x(CUtensorMap* map, const void* base, const ConvGeom& g, int BK) {
  auto fn = dfl_host::get_encode_tiled();
  if (!fn) return 999;
  cuuint64_t dims[5] = {(cuuint64_t)g.Ci, (cuuint64_t)g.Wi, (cuuint64_t)g.Hi, (cuuint64_t)g.Ti, (cuuint64_t)g.N};
  cuuint64_t strides[4] = {(cuuint64_t)g.Ci * 2, (cuuint64_t)g.Wi * g.Ci * 2, (cuuint64_t)g.Hi * g.Wi * g.Ci * 2,
                           (cuuint64_t)g.Ti * g.Hi * g.Wi * g.Ci * 2};
  cuuint32_t box[5] = {(cuuint32_t)BK, (cuuint32_t)BM, 1, 1, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return (int)fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(base), dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, BK == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

int make_tmap_w(CUtensorMap* map, const void* base, long long K, int Co, int BK, int BN) {
  auto fn = dfl_host::get_encode_tiled();
  if (!fn) return 999;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)Co};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)BN};
  cuuint32_t estr[2] = {1, 1};
  return (int)fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, BK == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

template <int BN, int BK>
constexpr int conv_stages() {
  // as many stages as ~200 KB of shared memory holds, capped at 12 (small tiles need depth)
  return (200 * 1024) / ((BM + BN) * BK * 2) > 12 ? 12 : (200 * 1024) / ((BM + BN) * BK * 2);
}

template <int BN, int BK, int EPI>
int launch_conv(const CUtensorMap& tx, const CUtensorMap& tw, const ConvGeom& g, const EpiParams& ep, int* err,
                cudaStream_t stream, int dev) {
  constexpr int STAGES = conv_stages<BN, BK>();
  using S = ConvSmem<BN, BK, STAGES>;
  auto kern = conv_tcgen05_kernel<BN, BK, STAGES, EPI>;
  static bool attr[16] = {false};
  if (!attr[dev & 15]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
    if (e != cudaSuccess) return (int)e;
    attr[dev & 15] = true;
  }
  const long long tiles = (long long)g.N * g.T * g.H * g.wtiles * (g.Co / BN);
  const int sms = dfl_host::num_sms(dev);
  kern<<<(int)(tiles < sms ? tiles : sms), kThreads, S::kTotal, stream>>>(tx, tw, g, ep, err);
  return (int)cudaGetLastError();
}

template <int BK, int EPI>
int dispatch_bn(int BN, const CUtensorMap& tx, const CUtensorMap& tw, const ConvGeom& g, const EpiParams& ep, int* err,
                cudaStream_t s, int dev) {
  switch (BN) {
    case 256: return launch_conv<256, BK, EPI>(tx, tw, g, ep, err, s, dev);
    case 192: return launch_conv<192, BK, EPI>(tx, tw, g, ep, err, s, dev);
    case 128: return launch_conv<128, BK, EPI>(tx, tw, g, ep, err, s, dev);
    case 96: return launch_conv<96, BK, EPI>(tx, tw, g, ep, err, s, dev);
    case 64: return launch_conv<64, BK, EPI>(tx, tw, g, ep, err, s, dev);
    default: return launch_conv<32, BK, EPI>(tx, tw, g, ep, err, s, dev);
  }
}

}  // namespace

extern "C" int dfl_conv3d(const ConvArgs* a, cudaStream_t stream) {
  ConvGeom g{};
  g.N = a->N, g.Ti = a->T, g.Hi = a->H, g.Wi = a->W, g.Ci = a->Ci, g.Co = a->Co;
  g.kt = a->kt, g.kh = a->kh, g.kw = a->kw;
  g.pt = a->valid_t ? 0 : (a->causal ? a->kt - 1 : a->kt / 2);
  g.ph = a->valid_h ? 0 : a->kh / 2;
  g.pw = a->valid_w ? 0 : a->kw / 2;
  g.T = a->valid_t ? g.Ti - a->kt + 1 : g.Ti;
  g.H = a->valid_h ? g.Hi - a->kh + 1 : g.Hi;
  g.W = a->valid_w ? g.Wi - a->kw + 1 : g.Wi;
  if (g.N <= 0 || g.T <= 0 || g.H <= 0 || g.W <= 0) return -2;
  for (int k : {g.kt, g.kh, g.kw})
    if (k != 1 && k != 3) return -3;
  const int BK = g.Ci % 64 == 0 ? 64 : (g.Ci % 32 == 0 ? 32 : 0);
  if (!BK) return -4;
  // widest N tile that divides Co (one tile for the narrow VAE layers)
  int BN = 0;
  for (int c : {256, 192, 128, 96, 64, 32})
    if (g.Co % c == 0) {
      BN = c;
      break;
    }
  if (!BN) return -5;
  if ((reinterpret_cast<uintptr_t>(a->x) | reinterpret_cast<uintptr_t>(a->w) | reinterpret_cast<uintptr_t>(a->y)) & 15)
    return -6;
  if (a->resid && (reinterpret_cast<uintptr_t>(a->resid) & 15)) return -6;
  g.wtiles = (g.W + BM - 1) / BM;
  g.csteps = g.Ci / BK;
  int dev = 0;
  cudaGetDevice(&dev);
  CUtensorMap tx, tw;
  int rc = make_tmap_x(&tx, a->x, g, BK);
  if (rc) return 1000 + rc;
  rc = make_tmap_w(&tw, a->w, (long long)g.kt * g.kh * g.kw * g.Ci, g.Co, BK, BN);
  if (rc) return 2000 + rc;
  EpiParams ep{};
  ep.D = a->y;
  ep.ldd = g.Co;
  ep.bias = reinterpret_cast<const __nv_bfloat16*>(a->bias);
  ep.alpha = 1.f;
  ep.act_lo = 0;
  ep.act_hi = g.Co;
  const long long M = (long long)g.N * g.T * g.H * g.W;
  if (M >= (1LL << 31)) return -7;
  ep.rows_per_batch = (int)M;
  if (a->resid) {  // out = resid + 1 * conv: the gated-residual epilogue with a unit gate
    ep.gate = a->ones;
    ep.gate_bstride = 0;
    ep.resid = reinterpret_cast<const __nv_bfloat16*>(a->resid);
    ep.ldr = g.Co;
    if (!a->ones) return -8;
    return BK == 64 ? dispatch_bn<64, kEpiGateResid>(BN, tx, tw, g, ep, a->err, stream, dev)
                    : dispatch_bn<32, kEpiGateResid>(BN, tx, tw, g, ep, a->err, stream, dev);
  }
  if (a->silu)
    return BK == 64 ? dispatch_bn<64, kEpiSilu>(BN, tx, tw, g, ep, a->err, stream, dev)
                    : dispatch_bn<32, kEpiSilu>(BN, tx, tw, g, ep, a->err, stream, dev);
  return BK == 64 ? dispatch_bn<64, kEpiNone>(BN, tx, tw, g, ep, a->err, stream, dev)
                  : dispatch_bn<32, kEpiNone>(BN, tx, tw, g, ep, a->err, stream, dev);
}
