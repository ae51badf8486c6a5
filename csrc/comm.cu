// Communication runtime for NVLink / NVSwitch peer memory (sm_100a).
//
//   * symmetric buffers: every rank cudaMalloc's the same sizes and exports a
//     CUDA IPC handle; peers open it, giving each kernel a table of peer
//     pointers (plain P2P loads / stores over NVLink, no NVLS objects)
//   * peer barrier: one tiny kernel; each rank release-stores an epoch into
//     every peer's flag slot and acquire-polls its own slots.  The epoch is a
//     device-side counter, so the barrier stays correct across CUDA-graph
//     replays.  Every wait is bounded: on timeout the kernel records
//     kErrPeerTimeout in the error word and returns (no trap, no hang)
//   * peer all-gather of a small f32 vector (sharded GEMV results)
//
// Reference parity: the NCCL bootstrap / groups of
// difflet/backends/cuda/ops_impl/parallel_mesh.py:80-118 and the collectives
// of difflet/backends/neuron/ops_impl/collectives.py:115-368, whose data
// movement the fused kernels (attention epilogue, q/k/v scatter) now perform.
#include "common.cuh"
#include "kernels.h"

namespace {
using namespace dfl;

DFL_DEVICE void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
DFL_DEVICE int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void peer_barrier_kernel(BarrierArgs a) {
  __shared__ int epoch;
  // A peer already timed out on this device: fail fast instead of waiting again.
  if (a.err != nullptr && *(volatile int*)a.err == kErrPeerTimeout) return;
  if (threadIdx.x == 0) epoch = *a.counter + 1;
  __syncthreads();
  const int e = epoch;
  const int t = threadIdx.x;
  if (t < a.world) {
    __threadfence_system();
    st_release_sys(a.flags[t] + a.rank, e);
  }
  if (t < a.world) {
    const int* mine = a.flags[a.rank] + t;
    long long t0 = clock64();
    unsigned it = 0;
    while ((int)(ld_acquire_sys(mine) - e) < 0) {
      if ((++it & 63u) == 0 && clock64() - t0 > a.timeout_cycles) {
        record_error(a.err, kErrPeerTimeout, kKidComm, t, e);
        break;
      }
    }
    __threadfence_system();
  }
  __syncthreads();
  if (threadIdx.x == 0) *a.counter = e;
}

// dst[r] + offset <- src (this rank's slice) for every peer r, f32 vectors.
__global__ void peer_put_f32_kernel(PeerPutArgs a) {
  const long long n = a.n;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float v = a.src[i];
    for (int r = 0; r < a.world; ++r) a.dst[r][a.dst_offset + i] = v;
  }
}

// CFG-parallel exchange fused with the guidance combine: this rank holds one
// branch's prediction, the partner's is read straight from its memory over
// NVLink; out (f32) = u + s (c - u).
__global__ void cfg_combine_kernel(const __nv_bfloat16* __restrict__ mine, const __nv_bfloat16* peer,
                                   float* __restrict__ out, long long n, float s, int mine_is_cond) {
  const long long n8 = n / 8;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
    const uint4 a = reinterpret_cast<const uint4*>(mine)[i];
    const uint4 b = reinterpret_cast<const uint4*>(peer)[i];
    const uint32_t av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
    float r[8];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float2 fa = unpack_bf16x2(av[h]), fb = unpack_bf16x2(bv[h]);
      const float2 u = mine_is_cond ? fb : fa, c = mine_is_cond ? fa : fb;
      r[2 * h] = u.x + s * (c.x - u.x);
      r[2 * h + 1] = u.y + s * (c.y - u.y);
    }
    reinterpret_cast<float4*>(out)[2 * i] = make_float4(r[0], r[1], r[2], r[3]);
    reinterpret_cast<float4*>(out)[2 * i + 1] = make_float4(r[4], r[5], r[6], r[7]);
  }
  for (long long i = n8 * 8 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float fa = __bfloat162float(mine[i]), fb = __bfloat162float(peer[i]);
    const float u = mine_is_cond ? fb : fa, c = mine_is_cond ? fa : fb;
    out[i] = u + s * (c - u);
  }
}

// Sum of the world partials of this rank's rows (fp32, fixed source order:
// deterministic), bias, gated residual, bf16 stores to every destination rank.
__global__ void __launch_bounds__(256) tp_reduce_kernel(TpReduceArgs a) {
  const int n8 = a.N / 8;
  const long long total = (long long)a.rows * n8;
  const __nv_bfloat16* slots = reinterpret_cast<const __nv_bfloat16*>(a.slots);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(i / n8);
    const int c = (int)(i - (long long)r * n8) * 8;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int src = 0; src < a.world; ++src) {
      const uint4 w = *reinterpret_cast<const uint4*>(slots + ((long long)src * a.slot_rows + r) * a.N + c);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = unpack_bf16x2(ws[h]);
        v[2 * h] += f.x;
        v[2 * h + 1] += f.y;
      }
    }
    if (a.bias) {
      const uint4 w = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.bias) + c);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = unpack_bf16x2(ws[h]);
        v[2 * h] += f.x;
        v[2 * h + 1] += f.y;
      }
    }
    const long long grow = a.row0 + r;
    if (a.gate) {
      const float* g = a.gate + (grow / a.rows_per_batch) * a.gate_bstride + c;
      const uint4 w = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.resid) +
                                                      (grow - a.resid_row0) * a.ldr + c);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 f = unpack_bf16x2(ws[h]);
        v[2 * h] = f.x + g[2 * h] * v[2 * h];
        v[2 * h + 1] = f.y + g[2 * h + 1] * v[2 * h + 1];
      }
    }
    uint4 o;
    o.x = pack_bf16x2(v[0], v[1]);
    o.y = pack_bf16x2(v[2], v[3]);
    o.z = pack_bf16x2(v[4], v[5]);
    o.w = pack_bf16x2(v[6], v[7]);
    const long long orow = a.out_row0 + r;
    for (int d = 0; d < a.out_world; ++d)
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.out[d]) + orow * a.ldo + c) = o;
  }
}

}  // namespace

extern "C" int dfl_tp_reduce(const TpReduceArgs* a, cudaStream_t stream) {
  if (a->rows <= 0) return 0;
  if (a->N % 8 || a->ldo % 8 || (a->gate && (a->ldr % 8 || a->gate_bstride % 4 || a->rows_per_batch <= 0)))
    return -2;
  if (a->out_world < 1 || a->out_world > DFL_MAX_PEERS || a->world < 1) return -3;
  uintptr_t al = reinterpret_cast<uintptr_t>(a->slots) | reinterpret_cast<uintptr_t>(a->bias) |
                 reinterpret_cast<uintptr_t>(a->resid) | reinterpret_cast<uintptr_t>(a->gate);
  for (int d = 0; d < a->out_world; ++d) al |= reinterpret_cast<uintptr_t>(a->out[d]);
  if (al & 15) return -4;
  long long blocks = ((long long)a->rows * (a->N / 8) + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  tp_reduce_kernel<<<(int)blocks, 256, 0, stream>>>(*a);
  return (int)cudaGetLastError();
}

extern "C" int dfl_cfg_combine(const void* mine, const void* peer, float* out, long long n, float scale,
                               int mine_is_cond, cudaStream_t stream) {
  if (n == 0) return 0;
  if ((reinterpret_cast<uintptr_t>(mine) | reinterpret_cast<uintptr_t>(peer) | reinterpret_cast<uintptr_t>(out)) & 15)
    return -2;
  long long blocks = (n / 8 + 255) / 256;
  if (blocks > 2048) blocks = 2048;
  if (blocks < 1) blocks = 1;
  cfg_combine_kernel<<<(int)blocks, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(mine),
                                                      reinterpret_cast<const __nv_bfloat16*>(peer), out, n, scale,
                                                      mine_is_cond);
  return (int)cudaGetLastError();
}

extern "C" int dfl_ipc_handle(const void* ptr, void* out64) {
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return (int)e;
  memcpy(out64, &h, sizeof(h));
  return 0;
}

extern "C" int dfl_ipc_open(const void* handle64, void** out) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(out, h, cudaIpcMemLazyEnablePeerAccess);
  return (int)e;
}

extern "C" int dfl_ipc_close(void* ptr) { return (int)cudaIpcCloseMemHandle(ptr); }

extern "C" int dfl_memcpy_async(void* dst, const void* src, long long nbytes, cudaStream_t stream) {
  return (int)cudaMemcpyAsync(dst, src, (size_t)nbytes, cudaMemcpyDeviceToDevice, stream);
}

extern "C" int dfl_peer_barrier(const BarrierArgs* a, cudaStream_t stream) {
  if (a->world < 1 || a->world > DFL_MAX_PEERS || a->rank < 0 || a->rank >= a->world) return -2;
  peer_barrier_kernel<<<1, 32, 0, stream>>>(*a);
  return (int)cudaGetLastError();
}

extern "C" int dfl_peer_put_f32(const PeerPutArgs* a, cudaStream_t stream) {
  if (a->world < 1 || a->world > DFL_MAX_PEERS) return -2;
  if (a->n == 0) return 0;
  long long blocks = (a->n + 255) / 256;
  if (blocks > 1024) blocks = 1024;
  peer_put_f32_kernel<<<(int)blocks, 256, 0, stream>>>(*a);
  return (int)cudaGetLastError();
}
