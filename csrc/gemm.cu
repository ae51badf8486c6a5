// Persistent tcgen05 GEMM for sm_100a:  D[M,N] = epi(A[M,K] . B[N,K]^T + bias)
//
// A is the activation (row-major, K contiguous), B is an nn.Linear weight
// ([out, in], K contiguous): both operands are K-major, bf16, fp32 accumulate
// in tensor memory.  One CTA per SM, warp-specialised:
//   warp 0      TMA producer (one lane): A/B tiles -> smem ring (128B swizzle)
//   warp 1      MMA issuer (one lane) + TMEM owner; tcgen05.mma 128xBNx16
//   warps 2..5  epilogue: tcgen05.ld the accumulator, fuse bias, GELU-tanh /
//               SiLU on a column window, or residual + gate * y, store bf16/f32
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue
// of tile i overlaps the main loop of tile i+1.
//
// Reference parity: every projection that the reference runs through
// F.linear (difflet/backends/_torch_megatron/linear.py:123,193), the fused
// GELU of NeuronGELU (difflet/layers/activations.py:62-65) and the gated
// residual of the FLUX blocks (difflet/models/flux/modeling_flux.py:712,
// 721-729, 844-867).
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "gemm_epilogue.cuh"
#include "kernels.h"

namespace {

using namespace dfl;

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int kThreads = 192;

template <int BN, int STAGES>
struct Smem {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBBytes = BN * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  // full[S], empty[S], tmem_full[2], tmem_empty[2], then tmem addr + abort flag
  // q/k/v head-scatter staging (kEpiQkv) after the barriers, then the 1024-byte align slack
  static constexpr int kStageOff = (kBarOffset + (2 * STAGES + 4) * 8 + 16 + 15) / 16 * 16;
  static constexpr int kTotal = kStageOff + kHeadStageBytes + 1024;
  static_assert(kTotal <= 232448, "shared memory budget");
};

template <int BN, int STAGES, int EPI, bool OUT_F32>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ GemmGroup grp, int* err) {
  using S = Smem<BN, STAGES>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128B-swizzle atoms
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* split_ok = reinterpret_cast<volatile int*>(tmem_slot + 2);  // split-K wait outcome

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int num_tiles = grp.total_tiles;
  constexpr uint32_t kTmemCols = 2 * BN;

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
    for (int i = 0; i < grp.count; ++i) {
      prefetch_tmap(&grp.p[i].ta);
      prefetch_tmap(&grp.p[i].tb);
    }
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
      uint32_t issued_parity[STAGES];
      bool issued[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = false, issued_parity[s] = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int lt, mb, nb, kb0, kb1;
        const GemmProblem& P = group_tile(grp, t, lt);
        tile_coords(lt / P.splits, P.num_m, P.num_n, mb, nb);
        split_k_range(P, lt % P.splits, BK, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, err, kKidGemm, 10 + stage, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_arrive_expect_tx(&full_bar[stage], S::kStageBytes);
          tma_load_2d(sa, &P.ta, &full_bar[stage], kb * BK, mb * BM);
          tma_load_2d(sb, &P.tb, &full_bar[stage], kb * BK, nb * BN);
          issued[stage] = true;
          issued_parity[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Drain: our own bulk copies must land before the CTA exits.
        for (int s = 0; s < STAGES; ++s)
          if (issued[s]) mbar_wait(&full_bar[s], issued_parity[s], nullptr, 0, 0, nullptr, 200000000LL);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, err, kKidGemm, 20 + acc, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        int lt, kb0, kb1;
        const GemmProblem& P = group_tile(grp, t, lt);
        split_k_range(P, lt % P.splits, BK, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, err, kKidGemm, 30 + stage, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * S::kStageBytes);
          const uint32_t b_addr = a_addr + S::kABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            uint64_t ad = make_sdesc_sw128(a_addr + k * 32, 16, 1024);
            uint64_t bd = make_sdesc_sw128(b_addr + k * 32, 16, 1024);
            umma_f16_ss(d_tmem, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
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
    // Epilogue warps 2..5 -> TMEM lane quarter (warp % 4)
    const int sub = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int lt, mb, nb;
      const GemmProblem& P = group_tile(grp, t, lt);
      const int tile = lt / P.splits;
      tile_coords(tile, P.num_m, P.num_n, mb, nb);
      if (!mbar_wait(&tfull_bar[acc], acc_phase, err, kKidGemm, 40 + acc, abort_flag)) break;
      tc_fence_after();
      const int row = mb * BM + sub * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(sub * 32) << 16) + acc * BN;
      auto release = [&]() {
        tc_fence_before();
        mbar_arrive(&tempty_bar[acc]);
      };
      if constexpr (EPI != kEpiSwiGLU && EPI != kEpiQkv) {
        if (P.splits > 1) {
          epilogue_tile_split<EPI, OUT_F32, BN>(tbase, sub * 32 + lane, row, nb * BN, P, tile, lt % P.splits,
                                                release, err, abort_flag, split_ok);
          acc ^= 1;
          if (acc == 0) acc_phase ^= 1u;
          continue;
        }
      }
      epilogue_tile<EPI, OUT_F32, BN>(tbase, row, nb * BN, P.M, P.N, P.ep, release,
                                      EPI == kEpiQkv ? smem + S::kStageOff + sub * kHeadStageWarp : nullptr);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

template <int BN, int STAGES, int EPI, bool OUT_F32>
int launch_variant(const GemmGroup& g, int* err, cudaStream_t stream, int device) {
  using S = Smem<BN, STAGES>;
  auto kern = gemm_tcgen05_kernel<BN, STAGES, EPI, OUT_F32>;
  static bool attr_set[16] = {false};
  if (!attr_set[device & 15]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kTotal);
    if (e != cudaSuccess) return (int)e;
    attr_set[device & 15] = true;
  }
  const int sms = dfl_host::num_sms(device);
  const int grid = g.total_tiles < sms ? g.total_tiles : sms;
  kern<<<grid, kThreads, S::kTotal, stream>>>(g, err);
  return (int)cudaGetLastError();
}

template <int BN, int STAGES>
int dispatch_epi(int epi, bool out_f32, const GemmGroup& g, int* err, cudaStream_t s, int dev) {
  switch (epi) {
    case kEpiNone:
      return out_f32 ? launch_variant<BN, STAGES, kEpiNone, true>(g, err, s, dev)
                     : launch_variant<BN, STAGES, kEpiNone, false>(g, err, s, dev);
    case kEpiGelu:
      return launch_variant<BN, STAGES, kEpiGelu, false>(g, err, s, dev);
    case kEpiSilu:
      return launch_variant<BN, STAGES, kEpiSilu, false>(g, err, s, dev);
    case kEpiGateResid:
      return launch_variant<BN, STAGES, kEpiGateResid, false>(g, err, s, dev);
    case kEpiSwiGLU:
      return launch_variant<BN, STAGES, kEpiSwiGLU, false>(g, err, s, dev);
    case kEpiQkv:
      return launch_variant<BN, STAGES, kEpiQkv, false>(g, err, s, dev);
    default:
      return -1;
  }
}

// Host-side argument checks (TMA: 16-byte aligned bases and row strides).
int check_args(const GemmArgs* a) {
  if (a->M <= 0 || a->N <= 0 || a->K <= 0) return -2;
  if ((reinterpret_cast<uintptr_t>(a->A) & 15) || (reinterpret_cast<uintptr_t>(a->B) & 15)) return -3;
  if ((a->lda * 2) % 16 || (a->ldb * 2) % 16) return -4;
  if (a->K % 8) return -5;
  const void* dchk = a->out_world > 0 ? a->out_peer[0] : a->D;
  if (!a->out_f32 && ((a->ldd % 8) || (reinterpret_cast<uintptr_t>(dchk) & 15))) return -6;
  if (a->out_f32 && ((a->ldd % 4) || (reinterpret_cast<uintptr_t>(dchk) & 15))) return -6;
  if (a->bias && (reinterpret_cast<uintptr_t>(a->bias) & 15)) return -7;
  if (a->epi == kEpiGateResid) {
    if (!a->gate || !a->resid || a->rows_per_batch <= 0) return -8;
    if ((reinterpret_cast<uintptr_t>(a->gate) & 15) || (reinterpret_cast<uintptr_t>(a->resid) & 15) ||
        (a->ldr % 8) || (a->gate_bstride % 4))
      return -8;
  }
  return 0;
}

}  // namespace

extern "C" int dfl_gemm_pair_launch(const void* group, int epi, int out_f32, int* err, cudaStream_t stream, int dev);

// Automatic choice of the CTA-pair kernel for wide GEMMs with M >= 1024 (on by default;
// dfl_gemm_set_pair_auto(0) restores the one-CTA kernel everywhere).
static int g_pair_auto = 1;
extern "C" void dfl_gemm_set_pair_auto(int on) { g_pair_auto = on; }

// Split-K workspace of each device (set by the host runtime; none = no split-K).
static float* g_split_ws[16];
static long long g_split_ws_floats[16];
static int* g_split_sem[16];
static int g_split_sem_count[16];
extern "C" void dfl_gemm_set_split_workspace(int device, void* ws, long long ws_bytes, void* sem, int sem_count) {
  const int d = device & 15;
  g_split_ws[d] = reinterpret_cast<float*>(ws);
  g_split_ws_floats[d] = ws_bytes / 4;
  g_split_sem[d] = reinterpret_cast<int*>(sem);
  g_split_sem_count[d] = sem_count;
}

// Small-M launches whose CTAs fill under 60 % of the SMs split K into s = 2..4 ranges (problems
// with at least 4 K blocks per range).  s minimises a time model in units of one K block of one
// CTA's 128 x 256 tile: waves(CTAs * s) * ceil(k_blocks / s) * kb_cost + (s - 1) * fixup.  The
// fixup (one f32 partial tile written to and read back from L2 per extra range, ranges finished
// in order) is priced at 12 K blocks (6 for 128 x 128 tiles): fitted on B200 to the measured
// small-M shapes (576 x 3072 x 15360 fastest at 2 ranges, 512 x 3072 x 12288 at 3), where the
// whole launch is bound by streaming the weights rather than by each SM's tensor rate.
// kb_cost: 1 for one CTA per tile, 0.92 for a CTA pair (each SM streams half of B: 32 instead
// of 48 KB per K block; measured 3-8 % faster per K block at these shapes).
constexpr double kPairKbCost = 0.92;
constexpr double kFixup256 = 12.0, kFixup128 = 6.0;

static double split_model(long long tiles, int ctas, int kb_max, int sms, double kb_cost, double fixup, int* best_s) {
  const int slots = ctas == 2 ? (sms / 2) : sms;  // pairs occupy two SMs
  int best = 1;
  double best_t = (double)((tiles + slots - 1) / slots) * kb_max * kb_cost;
  if (tiles * ctas * 10 <= (long long)sms * 6) {
    for (int sp = 2; sp <= 4; ++sp) {
      const int per = (kb_max + sp - 1) / sp;
      if (per < 4 || (sp - 1) * per >= kb_max) break;
      const long long items = tiles * sp;
      const double t = (double)((items + slots - 1) / slots) * per * kb_cost + (sp - 1) * fixup;
      if (t < best_t) best = sp, best_t = t;
    }
  }
  if (best_s) *best_s = best;
  return best_t;
}

// Measurement switch: 0 = the model decides, 1..4 = that many K ranges wherever splitting is allowed.
static int g_split_force = 0;
extern "C" void dfl_gemm_set_split_force(int s) { g_split_force = (s >= 0 && s <= 4) ? s : 0; }

static void plan_split_k(GemmGroup& g, int epi, int bn, int sms, int dev, int ctas) {
  const int d = dev & 15;
  if (!g_split_ws[d] || epi == kEpiSwiGLU || epi == kEpiQkv) return;
  int kb_max = 0;
  for (int i = 0; i < g.count; ++i) kb_max = std::max(kb_max, (g.p[i].K + BK - 1) / BK);
  int best = 1;
  split_model(g.total_tiles, ctas, kb_max, sms, ctas == 2 ? kPairKbCost : 1.0, bn >= 256 ? kFixup256 : kFixup128,
              &best);
  if (g_split_force) best = g_split_force;
  if (best == 1) return;
  long long ws_off = 0;
  int sem_off = 0;
  for (int i = 0; i < g.count; ++i) {
    GemmProblem& P = g.p[i];
    const int base_tiles = P.num_m * P.num_n;
    const int kb = (P.K + BK - 1) / BK;
    const int per = (kb + best - 1) / best;
    if (per < 4 || (best - 1) * per >= kb) continue;  // every range must hold K blocks
    const long long need = (long long)base_tiles * ctas * BM * bn;  // one partial per CTA tile
    if (ws_off + need > g_split_ws_floats[d] || sem_off + base_tiles * ctas > g_split_sem_count[d]) continue;
    P.splits = best;
    P.ws = g_split_ws[d] + ws_off;
    P.sem = g_split_sem[d] + sem_off;
    ws_off += need;
    sem_off += base_tiles * ctas;
    g.total_tiles += base_tiles * (best - 1);  // one more item per tile and extra range
    P.tiles = base_tiles * best;
  }
}

extern "C" int dfl_gemm_pair_can_split(int epi);

// One launch for `count` GEMMs that share the epilogue kind and output type.  The tile
// shape (CTA pairs with 256 x 256 tiles, or one CTA with 128 x 256 / 128 x 128 tiles)
// follows the first problem; the others are tiled the same way.
extern "C" int dfl_gemm_bf16_group(const GemmArgs* const* args, int count, cudaStream_t stream) {
  if (count < 1 || count > kMaxGroup) return -12;
  const GemmArgs* a0 = args[0];
  for (int i = 0; i < count; ++i) {
    const int rc = check_args(args[i]);
    if (rc) return rc;
    if (args[i]->epi != a0->epi || args[i]->out_f32 != a0->out_f32 || args[i]->err != a0->err) return -12;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  bool wide = a0->cta_mode != 3;  // cta_mode 3: one CTA per tile, 128-column tiles (6 stages)
  for (int i = 0; i < count; ++i) wide = wide && args[i]->N >= 1024;
  bool pair = a0->cta_mode == 2 || (a0->cta_mode == 0 && g_pair_auto && wide && a0->M >= 1024);
  const int sms = dfl_host::num_sms(dev);
  if (!pair && a0->cta_mode == 0 && g_pair_auto && wide && g_split_ws[dev & 15] && dfl_gemm_pair_can_split(a0->epi)) {
    // small M: CTA pairs (with split-K) against single CTAs (with split-K), by the model above
    long long t1 = 0, t2 = 0;
    int kb_max = 0;
    for (int i = 0; i < count; ++i) {
      const long long nn = (args[i]->N + 255) / 256;
      t1 += (args[i]->M + BM - 1) / BM * nn;
      t2 += (args[i]->M + 2 * BM - 1) / (2 * BM) * nn;
      kb_max = std::max(kb_max, (args[i]->K + BK - 1) / BK);
    }
    pair = split_model(t2, 2, kb_max, sms, kPairKbCost, kFixup256, nullptr) <
           split_model(t1, 1, kb_max, sms, 1.0, kFixup256, nullptr);
  }
  const int bm = pair ? 2 * BM : BM;
  const int bn = (pair || wide) ? 256 : 128;
  GemmGroup g;
  std::memset(&g, 0, sizeof(g));
  g.count = count;
  for (int i = 0; i < count; ++i) {
    const GemmArgs* a = args[i];
    GemmProblem& P = g.p[i];
    int rc = dfl_host::make_tmap_2d_bf16(&P.ta, a->A, a->K, a->M, a->lda, BK, BM, true);
    if (rc) return 1000 + rc;
    rc = dfl_host::make_tmap_2d_bf16(&P.tb, a->B, a->K, a->N, a->ldb, BK, pair ? 128 : bn, true);
    if (rc) return 2000 + rc;
    rc = dfl_host::fill_epi_params(*a, P.ep);
    if (rc) return rc;
    P.M = a->M;
    P.N = a->N;
    P.K = a->K;
    P.num_m = (a->M + bm - 1) / bm;
    P.num_n = (a->N + bn - 1) / bn;
    P.tiles = P.num_m * P.num_n;
    P.splits = 1;
    g.total_tiles += P.tiles;
  }
  if (pair) {
    if (dfl_gemm_pair_can_split(a0->epi)) plan_split_k(g, a0->epi, 256, sms, dev, 2);
    return dfl_gemm_pair_launch(&g, a0->epi, a0->out_f32, a0->err, stream, dev);
  }
  plan_split_k(g, a0->epi, bn, sms, dev, 1);
  if (wide) return dispatch_epi<256, 4>(a0->epi, a0->out_f32, g, a0->err, stream, dev);
  return dispatch_epi<128, 6>(a0->epi, a0->out_f32, g, a0->err, stream, dev);
}

extern "C" int dfl_gemm_bf16(const GemmArgs* a, cudaStream_t stream) { return dfl_gemm_bf16_group(&a, 1, stream); }

// ---------------------------------------------------------------------------
// Host helpers shared by every TMA user in this library.
// ---------------------------------------------------------------------------
namespace dfl_host {

EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                      uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                      bool swizzle128) {
  EncodeTiledFn fn = get_encode_tiled();
  if (!fn) return 999;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return (int)r;
}

int make_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                      uint64_t stride1_elems, uint64_t stride2_elems, uint32_t b0, uint32_t b1,
                      uint32_t b2, bool swizzle128) {
  EncodeTiledFn fn = get_encode_tiled();
  if (!fn) return 999;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_elems * 2, stride2_elems * 2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return (int)r;
}

int num_sms(int device) {
  static int cache[16] = {0};
  int d = device & 15;
  if (cache[d] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    cache[d] = n > 0 ? n : 148;
  }
  return cache[d];
}

}  // namespace dfl_host
