// Persistent 2-CTA tcgen05 GEMM (sm_100a): D[M,N] = epi(A[M,K] . B[N,K]^T + bias).
//
// A cluster of two CTAs on neighbouring SMs computes one 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256): CTA r loads its own 128 rows of A and its own
// 128 rows of B (one half of the tile's N) into its own shared memory; the MMA
// issued by CTA 0 reads both CTAs' tiles, so each SM streams half the B operand a
// 1-CTA 128 x 256 tile needs.  Each CTA's tensor memory holds its 128 rows x 256
// columns of the accumulator (double-buffered) and its four epilogue warps store
// them.  Loads are plain TMA tile loads (no cross-CTA broadcast); the two CTAs'
// loads complete on CTA 0's stage barrier, CTA 0's MMA completion is signalled to
// both CTAs' barriers (tcgen05.commit multicast), and CTA 1's epilogue reports
// "accumulator drained" to CTA 0 by a remote mbarrier arrive.  Every wait is
// bounded (error word + abort flag), as in the 1-CTA kernel.
#include "common.cuh"
#include "gemm_epilogue.cuh"
#include "kernels.h"

namespace {
using namespace dfl;

constexpr int BM = 128;      // rows per CTA (256 per pair)
constexpr int BN = 256;      // columns per pair tile; each CTA loads BN / 2 rows of B
constexpr int BK = 64;
constexpr int kABytes = BM * BK * 2;        // 16 KB
constexpr int kBBytes = (BN / 2) * BK * 2;  // 16 KB
constexpr int kStageBytes = kABytes + kBBytes;

// Launch shape for EW epilogue warps (4: one per TMEM lane quarter, each owning all BN columns
// of its 32 rows; 8: two per lane quarter, each owning BN / 2 columns, so two epilogue warps
// share every SM sub-partition and hide each other's TMEM / L2 latency).  The q/k/v head
// scatter stages 8 KB per epilogue warp, which with 8 warps costs one operand stage.
template <int EPI, int EW>
struct PairCfg {
  // EW == 8: warpgroup 0 = TMA warp, MMA warp and two idle warps, warpgroups 1-2 = epilogue,
  // with a register split (128 x 64 + 256 x 216 = 63488 <= 384 x 168 at launch).
  static constexpr int kThreads = EW == 8 ? 384 : 192;
  static constexpr int kFirstEpiWarp = EW == 8 ? 4 : 2;
  static constexpr int kCols = BN * 4 / EW;  // accumulator columns per epilogue warp
  static constexpr int STAGES = (EPI == kEpiQkv && EW == 8) ? 5 : 6;
  static constexpr int kBarOff = STAGES * kStageBytes;
  static constexpr int kStageOff = (kBarOff + (2 * STAGES + 4) * 8 + 16 + 15) / 16 * 16;  // head-scatter staging
  static constexpr int kSmemTotal = kStageOff + (EPI == kEpiQkv ? EW * kHeadStageWarp : 0) + 1024;
  static_assert(kSmemTotal <= 232448, "shared memory budget");
  static_assert(EW == 4 || EW == 8, "epilogue warps");
};
constexpr uint32_t kTmemCols = 2 * BN;
constexpr int kRegsLow = 64, kRegsHigh = 216;  // EW == 8 register split

DFL_DEVICE void regs_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 64;"); }
DFL_DEVICE void regs_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 216;"); }
constexpr uint32_t kPeerMask = 0xFEFFFFFFu;  // shared::cluster address of CTA 0's copy

DFL_DEVICE uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

DFL_DEVICE void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

DFL_DEVICE void fence_mbar_init_cluster() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// TMA tile load into this CTA's smem whose completion is counted on CTA 0's barrier.
DFL_DEVICE void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar) & kPeerMask), "r"(c0), "r"(c1)
      : "memory");
}

DFL_DEVICE void umma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}

// Arrive (one count) on the same barrier in both CTAs once this thread's MMAs complete.
DFL_DEVICE void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)0x3)
      : "memory");
}

DFL_DEVICE void mbar_arrive_cta0(uint64_t* bar) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(remote) : "r"(smem_u32(bar)));
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}

template <int EPI, bool OUT_F32, int EW>
__global__ void __launch_bounds__(PairCfg<EPI, EW>::kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ GemmGroup grp, int* err) {
  using C = PairCfg<EPI, EW>;
  constexpr int STAGES = C::STAGES;
  constexpr int kBarOff = C::kBarOff;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* split_ok = reinterpret_cast<volatile int*>(tmem_slot + 2);  // split-K wait outcome

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x / 2, num_pairs = gridDim.x / 2;
  const int num_tiles = grp.total_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);   // CTA 0's producer posts the pair's bytes
      mbar_init(&empty_bar[s], 1);  // CTA 0's MMA commit, multicast to both CTAs
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 2 * 32 * EW);  // both CTAs' epilogue threads (CTA 0's copy is the one used)
    }
    *abort_flag = 0;
    fence_mbar_init_cluster();
    fence_proxy_async_shared();
    for (int i = 0; i < grp.count; ++i) {
      prefetch_tmap(&grp.p[i].ta);
      prefetch_tmap(&grp.p[i].tb);
    }
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote traffic
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if constexpr (EW == 8) regs_dec();
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool issued[STAGES];
      uint32_t issued_parity[STAGES];
      for (int s = 0; s < STAGES; ++s) issued[s] = false, issued_parity[s] = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += num_pairs) {
        int lt, mb, nb, kb0, kb1;
        const GemmProblem& P = group_tile(grp, t, lt);
        tile_coords(lt / P.splits, P.num_m, P.num_n, mb, nb);
        split_k_range(P, lt % P.splits, BK, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, err, kKidGemm, 310 + stage, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * kStageBytes;
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * kStageBytes);
          tma_load_2d_pair(sa, &P.ta, &full_bar[stage], kb * BK, mb * 2 * BM + (int)rank * BM);
          tma_load_2d_pair(sa + kABytes, &P.tb, &full_bar[stage], kb * BK, nb * BN + (int)rank * (BN / 2));
          issued[stage] = true;
          issued_parity[stage] = phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && rank == 0) {
        for (int s = 0; s < STAGES; ++s)
          if (issued[s]) mbar_wait(&full_bar[s], issued_parity[s], nullptr, 0, 0, nullptr, 200000000LL);
      }
    }
  } else if (warp == 1) {
    if constexpr (EW == 8) regs_dec();
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = make_idesc_bf16_f32(2 * BM, BN);
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += num_pairs) {
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1u, err, kKidGemm, 320 + acc, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        int lt, kb0, kb1;
        const GemmProblem& P = group_tile(grp, t, lt);
        split_k_range(P, lt % P.splits, BK, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, err, kKidGemm, 330 + stage, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * kStageBytes);
          const uint32_t b_addr = a_addr + kABytes;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16_pair(d_tmem, make_sdesc_sw128(a_addr + k * 32, 16, 1024),
                          make_sdesc_sw128(b_addr + k * 32, 16, 1024), idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          umma_commit_pair(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull_bar[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else if (warp < C::kFirstEpiWarp) {
    if constexpr (EW == 8) regs_dec();  // the idle warps of warpgroup 0
  } else {
    if constexpr (EW == 8) regs_inc();
    const int ew = warp - C::kFirstEpiWarp;  // epilogue warp 0 .. EW-1
    const int sub = warp & 3;  // the TMEM lane quarter this warp may access
    const int slice = ew >> 2;  // which kCols columns of the tile (EW == 8: two slices)
    uint8_t* stage = EPI == kEpiQkv ? smem + C::kStageOff + ew * kHeadStageWarp : nullptr;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = pair; t < num_tiles; t += num_pairs) {
      int lt, mb, nb;
      const GemmProblem& P = group_tile(grp, t, lt);
      const int tile = lt / P.splits;
      tile_coords(tile, P.num_m, P.num_n, mb, nb);
      if (!mbar_wait(&tfull_bar[acc], acc_phase, err, kKidGemm, 340 + acc, abort_flag)) break;
      tc_fence_after();
      const int row = mb * 2 * BM + (int)rank * BM + sub * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(sub * 32) << 16) + acc * BN + slice * C::kCols;
      auto release = [&]() {
        tc_fence_before();
        if (rank == 0)
          mbar_arrive(&tempty_bar[acc]);
        else
          mbar_arrive_cta0(&tempty_bar[acc]);
      };
      if constexpr (EW == 4 && EPI != kEpiSwiGLU && EPI != kEpiQkv) {
        if (P.splits > 1) {  // each CTA owns its 128 rows: partial tile / counter 2 * tile + rank
          epilogue_tile_split<EPI, OUT_F32, BN>(tbase, sub * 32 + lane, row, nb * BN, P, 2 * tile + (int)rank,
                                                lt % P.splits, release, err, abort_flag, split_ok);
          acc ^= 1;
          if (acc == 0) acc_phase ^= 1u;
          continue;
        }
      }
      epilogue_tile<EPI, OUT_F32, C::kCols>(tbase, row, nb * BN + slice * C::kCols, P.M, P.N, P.ep, release, stage);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no remote arrive or load is in flight towards a CTA that leaves
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols));
}

// Epilogue warps per pair CTA: 0 = 8 for the q/k/v head scatter (the heaviest epilogue), 4 for
// the rest; 4 or 8 = that count for every epilogue.
int g_epi_warps = 0;

template <int EPI, bool OUT_F32, int EW>
int launch_pair_ew(const GemmGroup& g, int* err, cudaStream_t stream, int dev) {
  using C = PairCfg<EPI, EW>;
  auto kern = gemm_pair_kernel<EPI, OUT_F32, EW>;
  static bool attr[16] = {false};
  if (!attr[dev & 15]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemTotal);
    if (e != cudaSuccess) return (int)e;
    if (EW == 8) {  // the setmaxnreg split must fit in the registers the CTA is launched with
      cudaFuncAttributes fa;
      e = cudaFuncGetAttributes(&fa, kern);
      if (e != cudaSuccess) return (int)e;
      if (fa.numRegs * C::kThreads < 128 * kRegsLow + 256 * kRegsHigh) return -11;
    }
    attr[dev & 15] = true;
  }
  const int pairs_max = dfl_host::num_sms(dev) / 2;
  const int pairs = g.total_tiles < pairs_max ? g.total_tiles : pairs_max;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(C::kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::kSmemTotal;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, g, err);
  return (int)e;
}

template <int EPI, bool OUT_F32>
int launch_pair(const GemmGroup& g, int* err, cudaStream_t stream, int dev) {
  const int ew = g_epi_warps ? g_epi_warps : (EPI == kEpiQkv ? 8 : 4);
  return ew == 8 ? launch_pair_ew<EPI, OUT_F32, 8>(g, err, stream, dev)
                 : launch_pair_ew<EPI, OUT_F32, 4>(g, err, stream, dev);
}

}  // namespace

extern "C" void dfl_gemm_set_epi_warps(int n) { g_epi_warps = (n == 4 || n == 8) ? n : 0; }

// Split-K runs in the pair kernel only with four epilogue warps (the fixup's 128-thread barrier).
extern "C" int dfl_gemm_pair_can_split(int epi) {
  const int ew = g_epi_warps ? g_epi_warps : (epi == kEpiQkv ? 8 : 4);
  return ew == 4 && epi != kEpiQkv && epi != kEpiSwiGLU;
}

// Grouped launch prepared by dfl_gemm_bf16_group (tiles of 256 rows, B boxes of 128 rows).
extern "C" int dfl_gemm_pair_launch(const void* group, int epi, int out_f32, int* err, cudaStream_t stream, int dev) {
  const GemmGroup& g = *reinterpret_cast<const GemmGroup*>(group);
  switch (epi) {
    case kEpiNone:
      return out_f32 ? launch_pair<kEpiNone, true>(g, err, stream, dev)
                     : launch_pair<kEpiNone, false>(g, err, stream, dev);
    case kEpiGelu:
      return launch_pair<kEpiGelu, false>(g, err, stream, dev);
    case kEpiSilu:
      return launch_pair<kEpiSilu, false>(g, err, stream, dev);
    case kEpiGateResid:
      return launch_pair<kEpiGateResid, false>(g, err, stream, dev);
    case kEpiSwiGLU:
      return launch_pair<kEpiSwiGLU, false>(g, err, stream, dev);
    case kEpiQkv:
      return launch_pair<kEpiQkv, false>(g, err, stream, dev);
    default:
      return -1;
  }
}
