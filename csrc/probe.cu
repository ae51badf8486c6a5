// TeaCache probe for sm_100a: relative L1 distance between two bf16 tensors,
// reduced on the device to one f32 scalar:  out = sum|a - b| / sum|b|.
//
// Two passes in one launch: every block writes its partial sums to a scratch
// buffer, the last block to finish (an atomic ticket in the same scratch)
// reduces the partials in a fixed order (deterministic) and resets the ticket.
// Reference parity: the block-0 modulated-input probe of TeaCache
// (difflet/models/wan/modeling_wan.py:1069-1115, difflet/pipeline/teacache.py:180-280),
// which the reference evaluates with host-side torch ops.
#include "common.cuh"
#include "kernels.h"

namespace {
using namespace dfl;

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) rel_l1_kernel(const __nv_bfloat16* __restrict__ a,
                                                          const __nv_bfloat16* __restrict__ b, long long n,
                                                          float* scratch, float* out) {
  // scratch layout: [0] uint32 ticket (fixed slot, whatever the grid), then 2 partials per block
  float num = 0.f, den = 0.f;
  const long long n8 = n / 8;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const uint4 va = reinterpret_cast<const uint4*>(a)[i];
    const uint4 vb = reinterpret_cast<const uint4*>(b)[i];
    const uint32_t xa[4] = {va.x, va.y, va.z, va.w}, xb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float2 fa = unpack_bf16x2(xa[h]), fb = unpack_bf16x2(xb[h]);
      num += fabsf(fa.x - fb.x) + fabsf(fa.y - fb.y);
      den += fabsf(fb.x) + fabsf(fb.y);
    }
  }
  for (long long i = n8 * 8 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float fa = __bfloat162float(a[i]), fb = __bfloat162float(b[i]);
    num += fabsf(fa - fb);
    den += fabsf(fb);
  }
  __shared__ float s_num[kThreads / 32], s_den[kThreads / 32];
  __shared__ bool s_last;
  num = warp_sum(num);
  den = warp_sum(den);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (lane == 0) s_num[warp] = num, s_den[warp] = den;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tn = 0.f, td = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) tn += s_num[w], td += s_den[w];
    scratch[1 + 2 * blockIdx.x] = tn;
    scratch[2 + 2 * blockIdx.x] = td;
    __threadfence();
    unsigned int* ticket = reinterpret_cast<unsigned int*>(scratch);
    s_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    __threadfence();
    float tn = 0.f, td = 0.f;
    const volatile float* vs = scratch;
    for (unsigned int blk = 0; blk < gridDim.x; ++blk) {
      tn += vs[1 + 2 * blk];
      td += vs[2 + 2 * blk];
    }
    *out = td > 0.f ? tn / td : 0.f;
    *reinterpret_cast<unsigned int*>(scratch) = 0u;  // ready for the next call
  }
}

}  // namespace

// Scratch floats needed for `blocks` blocks (partials + ticket).
extern "C" long long dfl_rel_l1_scratch_floats(int blocks) { return 2LL * blocks + 1; }

extern "C" int dfl_rel_l1_blocks(long long n, int num_sms) {
  long long b = (n / 8 + kThreads - 1) / kThreads;
  long long cap = (long long)num_sms * 4;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (int)b;
}

extern "C" int dfl_rel_l1(const void* a, const void* b, long long n, float* scratch, int blocks, float* out,
                          cudaStream_t stream) {
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) return -2;
  if (blocks < 1 || !scratch || !out) return -3;
  rel_l1_kernel<<<blocks, kThreads, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(a),
                                                 reinterpret_cast<const __nv_bfloat16*>(b), n, scratch, out);
  return (int)cudaGetLastError();
}
