// MXFP8 for sm_100a: the OCP-MX quantizer and a block-scaled tcgen05 GEMM.
//
// Format (OCP Microscaling Formats v1.0): FP8 E4M3 elements, one E8M0 scale per
// 32 consecutive K values; scale exponent = floor(log2(amax)) - 8 (E4M3's largest
// binade), elements = x * 2^-e converted with saturation.
//
// Scale layout ("blocked", what the tensor cores read through TMEM): for a
// [R, K] operand, one 512-byte atom per (128 rows, 128 K values), atoms ordered
// K-fastest; inside an atom byte (r%32)*16 + ((r%128)/32)*4 + (k/32)%4.  One
// atom is exactly the scales of one 128-row x 128-K smem stage, so the
// producer moves it with one bulk copy and the MMA warp moves it into TMEM with
// one tcgen05.cp (32 lanes x 128 bits, replicated to the 4 lane quarters).
//
// GEMM: persistent, warp-specialised like the bf16 GEMM (TMA warp, MMA warp, 4
// epilogue warps), 128 x 256 tiles, K step 128 (one 128-byte swizzle row of
// FP8), 4 stages.  Per stage the MMA warp issues 3 tcgen05.cp (A scales, 2 x B
// scales) and 4 tcgen05.mma kind::mxf8f6f4.block_scale (K = 32 each; the scale
// byte of each K block is selected by the instruction descriptor's scale-factor
// ids).  TMEM: accumulator 256 columns, A scales 4, B scales 8 (512 allocated);
// the accumulator is single-buffered (the scales take the second buffer's room).
//
// Reference parity: the MX surface difflet/ops/mx.py:10-87 and its scale law
// (difflet/backends/cpu/ops_impl/mx.py:15-88); the reference's block-scaled
// kernels are Trainium NKI (difflet/backends/trainium/nki_kernels/mx.py:226-1179).
#include <cuda_fp8.h>

#include "common.cuh"
#include "gemm_epilogue.cuh"
#include "kernels.h"

namespace {
using namespace dfl;

// ---------------------------------------------------------------------------- quantizer
__global__ void __launch_bounds__(256) mx_quant_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                       int R, int K, uint8_t* __restrict__ q, long long ldq,
                                                       uint8_t* __restrict__ sf, int blocked) {
  const int kb_per_row = K / 32;
  const long long n = (long long)R * kb_per_row;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / kb_per_row);
    const int kb = (int)(i - (long long)r * kb_per_row);
    const uint4* src = reinterpret_cast<const uint4*>(x + (long long)r * ldx + kb * 32);
    float v[32];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 w = src[c];
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = unpack_bf16x2(ws[h]);
        v[c * 8 + 2 * h] = f.x;
        v[c * 8 + 2 * h + 1] = f.y;
      }
    }
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
    // floor(log2(amax)) from the exponent field; 0 / denormals clamp to the smallest scale
    int e = (int)((__float_as_uint(amax) >> 23) & 0xFF) - 127 - 8;
    e = amax > 0.f ? e : -127;
    e = max(-127, min(127, e));
    const float inv = __uint_as_float((uint32_t)(127 - e) << 23);  // 2^-e, e in [-127, 119]
    uint32_t packed[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(v[4 * j] * inv, v[4 * j + 1] * inv),
                                                                __NV_SATFINITE, __NV_E4M3);
      const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(
          make_float2(v[4 * j + 2] * inv, v[4 * j + 3] * inv), __NV_SATFINITE, __NV_E4M3);
      packed[j] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    uint4* dst = reinterpret_cast<uint4*>(q + (long long)r * ldq + kb * 32);
    dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    const uint8_t s = (uint8_t)(e + 127);
    if (blocked) {
      const long long atom = (long long)(r / 128) * (K / 128) + kb / 4;
      sf[atom * 512 + (r % 32) * 16 + ((r % 128) / 32) * 4 + (kb % 4)] = s;
    } else {
      sf[(long long)r * kb_per_row + kb] = s;
    }
  }
}

// ---------------------------------------------------------------------------- GEMM
constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4;
constexpr int kThreads = 192;
constexpr int kABytes = BM * BK;        // 16 KB
constexpr int kBBytes = BN * BK;        // 32 KB
constexpr int kSfaBytes = 512;
constexpr int kSfbBytes = 2 * 512;
constexpr int kAOff = 0;
constexpr int kBOff = kAOff + STAGES * kABytes;
constexpr int kSfaOff = kBOff + STAGES * kBBytes;
constexpr int kSfbOff = kSfaOff + STAGES * kSfaBytes;
constexpr int kBarOff = kSfbOff + STAGES * kSfbBytes;
constexpr int kSmemTotal = kBarOff + (2 * STAGES + 2) * 8 + 16 + 1024;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSfaCol = 256, kSfbCol = 264;

DFL_DEVICE void bulk_load(uint8_t* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// smem -> TMEM: 32 rows x 128 bits, written to all four 32-lane quarters
DFL_DEVICE void tmem_cp_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Descriptor of a non-swizzled K-major smem matrix of 16-byte rows (8-row core
// matrices 128 bytes apart).
DFL_DEVICE uint64_t make_sdesc_plain(uint32_t smem_addr, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  return d;          // layout type 0: no swizzle
}

DFL_DEVICE void umma_mxf8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t sfa,
                             uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

// Instruction descriptor, kind::mxf8f6f4 with block scaling: E4M3 x E4M3, E8M0
// scales, both operands K-major; scale-factor ids select the byte (K block) of
// each 32-bit scale word.
__host__ __device__ constexpr uint32_t make_idesc_mxf8(int M, int N, uint32_t sf_id) {
  return (sf_id << 4)                      // B scale-factor id
         | (0u << 7) | (0u << 10)          // A / B format: E4M3
         | ((uint32_t)(N >> 3) << 17)      // N / 8
         | (1u << 23)                      // scale format: E8M0
         | ((uint32_t)(M >> 4) << 24)      // M / 16
         | (sf_id << 29);                  // A scale-factor id
}

template <int EPI, bool OUT_F32>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_mx_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const uint8_t* __restrict__ sfa, const uint8_t* __restrict__ sfb, int M, int N, int K,
                   EpiParams ep, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int num_m = (M + BM - 1) / BM, num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_k = K / BK;
  const int k_atoms = K / 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(tempty_bar, 128);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_shared();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
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
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, err, kKidGemm, 110 + stage, abort_flag)) {
            ok = false;
            break;
          }
          uint64_t* bar = &full_bar[stage];
          mbar_arrive_expect_tx(bar, kABytes + kBBytes + kSfaBytes + kSfbBytes);
          tma_load_2d(smem + kAOff + stage * kABytes, &tmap_a, bar, kb * BK, mb * BM);
          tma_load_2d(smem + kBOff + stage * kBBytes, &tmap_b, bar, kb * BK, nb * BN);
          bulk_load(smem + kSfaOff + stage * kSfaBytes, sfa + ((long long)mb * k_atoms + kb) * 512, 512, bar);
          uint8_t* sb = smem + kSfbOff + stage * kSfbBytes;
          bulk_load(sb, sfb + ((long long)(2 * nb) * k_atoms + kb) * 512, 512, bar);
          bulk_load(sb + 512, sfb + ((long long)(2 * nb + 1) * k_atoms + kb) * 512, 512, bar);
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
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      const uint32_t t_sfa = tmem_base + kSfaCol, t_sfb = tmem_base + kSfbCol;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(tempty_bar, acc_phase ^ 1u, err, kKidGemm, 120, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, err, kKidGemm, 130 + stage, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + kAOff + stage * kABytes);
          const uint32_t b_addr = smem_u32(smem + kBOff + stage * kBBytes);
          const uint32_t sa_addr = smem_u32(smem + kSfaOff + stage * kSfaBytes);
          const uint32_t sb_addr = smem_u32(smem + kSfbOff + stage * kSfbBytes);
          tmem_cp_32x128b_warpx4(t_sfa, make_sdesc_plain(sa_addr, 128));
          tmem_cp_32x128b_warpx4(t_sfb, make_sdesc_plain(sb_addr, 128));
          tmem_cp_32x128b_warpx4(t_sfb + 4, make_sdesc_plain(sb_addr + 512, 128));
#pragma unroll
          for (uint32_t j = 0; j < 4; ++j) {
            const uint64_t ad = make_sdesc_sw128(a_addr + j * 32, 16, 1024);
            const uint64_t bd = make_sdesc_sw128(b_addr + j * 32, 16, 1024);
            umma_mxf8_ss(tmem_base, ad, bd, make_idesc_mxf8(BM, BN, j), t_sfa | (j << 30), t_sfb | (j << 30),
                         (kb > 0 || j > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(tfull_bar);
        acc_phase ^= 1u;
      }
    }
  } else {
    const int sub = warp & 3;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      if (!mbar_wait(tfull_bar, acc_phase, err, kKidGemm, 140, abort_flag)) break;
      tc_fence_after();
      const int row = mb * BM + sub * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(sub * 32) << 16);
      // TMEM is released once the tile's last chunk is in registers.
      epilogue_tile<EPI, OUT_F32, BN>(tbase, row, nb * BN, M, N, ep, [&]() {
        tc_fence_before();
        mbar_arrive(tempty_bar);
      });
      acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

int make_tmap_2d_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride,
                    uint32_t box_inner, uint32_t box_outer) {
  auto fn = dfl_host::get_encode_tiled();
  if (!fn) return 999;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return (int)fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

template <int EPI, bool OUT_F32>
int launch_mx(const CUtensorMap& ta, const CUtensorMap& tb, const MxGemmArgs* a, const EpiParams& ep,
              cudaStream_t stream, int dev) {
  auto kern = gemm_mx_kernel<EPI, OUT_F32>;
  static bool attr[16] = {false};
  if (!attr[dev & 15]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTotal);
    if (e != cudaSuccess) return (int)e;
    attr[dev & 15] = true;
  }
  const int tiles = ((a->g.M + BM - 1) / BM) * ((a->g.N + BN - 1) / BN);
  const int sms = dfl_host::num_sms(dev);
  kern<<<tiles < sms ? tiles : sms, kThreads, kSmemTotal, stream>>>(
      ta, tb, reinterpret_cast<const uint8_t*>(a->sfa), reinterpret_cast<const uint8_t*>(a->sfb), a->g.M, a->g.N,
      a->g.K, ep, a->g.err);
  return (int)cudaGetLastError();
}

}  // namespace

extern "C" int dfl_mx_quantize(const void* x, long long ldx, int R, int K, void* q, long long ldq, void* scales,
                               int blocked, cudaStream_t stream) {
  if (R <= 0 || K <= 0) return 0;
  if (K % 32 || (blocked && K % 128)) return -2;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(q)) & 15) return -3;
  if (ldx % 8 || ldq % 16) return -4;
  const long long n = (long long)R * (K / 32);
  long long blocks = (n + 255) / 256;
  if (blocks > 8192) blocks = 8192;
  mx_quant_kernel<<<(int)blocks, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx, R, K,
                                                    reinterpret_cast<uint8_t*>(q), ldq,
                                                    reinterpret_cast<uint8_t*>(scales), blocked);
  return (int)cudaGetLastError();
}

extern "C" int dfl_gemm_mx(const MxGemmArgs* a, cudaStream_t stream) {
  const GemmArgs& g = a->g;
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return -2;
  if (g.K % BK) return -5;
  if ((reinterpret_cast<uintptr_t>(g.A) | reinterpret_cast<uintptr_t>(g.B)) & 15) return -3;
  if (g.lda % 16 || g.ldb % 16) return -4;
  if ((reinterpret_cast<uintptr_t>(a->sfa) | reinterpret_cast<uintptr_t>(a->sfb)) & 15) return -10;
  const void* dchk = g.out_world > 0 ? g.out_peer[0] : g.D;
  if (g.epi == kEpiQkv && g.D == nullptr) dchk = nullptr;  // every column goes to the head scatter
  if (!g.out_f32 && ((g.ldd % 8) || (reinterpret_cast<uintptr_t>(dchk) & 15))) return -6;
  if (g.out_f32 && ((g.ldd % 4) || (reinterpret_cast<uintptr_t>(dchk) & 15))) return -6;
  if (g.bias && (reinterpret_cast<uintptr_t>(g.bias) & 15)) return -7;
  if (g.epi == kEpiGateResid && (!g.gate || !g.resid || g.rows_per_batch <= 0)) return -8;
  if (g.out_world < 0 || g.out_world > DFL_MAX_PEERS) return -9;
  int dev = 0;
  cudaGetDevice(&dev);
  CUtensorMap ta, tb;
  int rc = make_tmap_2d_u8(&ta, g.A, g.K, g.M, g.lda, BK, BM);
  if (rc) return 1000 + rc;
  rc = make_tmap_2d_u8(&tb, g.B, g.K, g.N, g.ldb, BK, BN);
  if (rc) return 2000 + rc;
  EpiParams ep;
  rc = dfl_host::fill_epi_params(g, ep);
  if (rc) return rc;
  switch (g.epi) {
    case kEpiNone:
      return g.out_f32 ? launch_mx<kEpiNone, true>(ta, tb, a, ep, stream, dev)
                       : launch_mx<kEpiNone, false>(ta, tb, a, ep, stream, dev);
    case kEpiGelu:
      return launch_mx<kEpiGelu, false>(ta, tb, a, ep, stream, dev);
    case kEpiSilu:
      return launch_mx<kEpiSilu, false>(ta, tb, a, ep, stream, dev);
    case kEpiGateResid:
      return launch_mx<kEpiGateResid, false>(ta, tb, a, ep, stream, dev);
    case kEpiQkv:
      return launch_mx<kEpiQkv, false>(ta, tb, a, ep, stream, dev);
    default:
      return -1;
  }
}
