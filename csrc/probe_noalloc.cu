// Allocation-free relative-L1 reduction (see probe_noalloc.h for the contract:
// who needs it, the scratch size, the first-call set-up and the race rule).
// No counterpart in the reference.
#include <mutex>

#include "common.cuh"
#include "probe_noalloc.h"

namespace {
using namespace dfl;

constexpr int kThreads = 256;
constexpr int kScratchFloats = 1 + 2 * DFL_NOALLOC_MAX_BLOCKS;

// The reduction's scratch: [0] completion ticket, then two partial sums per
// block.  One copy per device, alive until the process exits.
static __device__ __align__(256) float g_noalloc_scratch[kScratchFloats];

__global__ void __launch_bounds__(kThreads) rel_l1_noalloc_kernel(const __nv_bfloat16* __restrict__ a,
                                                                  const __nv_bfloat16* __restrict__ b,
                                                                  long long n, float* scratch, float* out) {
  float num = 0.f, den = 0.f;
  const long long n8 = n / 8;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8;
       i += (long long)gridDim.x * blockDim.x) {
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
  if (lane == 0) {
    s_num[warp] = num;
    s_den[warp] = den;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float tn = 0.f, td = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) {
      tn += s_num[w];
      td += s_den[w];
    }
    scratch[1 + 2 * blockIdx.x] = tn;
    scratch[2 + 2 * blockIdx.x] = td;
    __threadfence();
    s_last = atomicAdd(reinterpret_cast<unsigned int*>(scratch), 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    __threadfence();
    const volatile float* vs = scratch;
    float tn = 0.f, td = 0.f;
    for (unsigned int blk = 0; blk < gridDim.x; ++blk) {
      tn += vs[1 + 2 * blk];
      td += vs[2 + 2 * blk];
    }
    *out = td > 0.f ? tn / td : 0.f;
  }
}

// Device address of the static scratch, resolved once per device.
constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_ptr[kMaxDevices] = {nullptr};
int g_sms[kMaxDevices] = {0};

int setup_device(int dev, float** ptr, int* sms) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // this device is current
    if (e != cudaSuccess || p == nullptr) return DFL_NOALLOC_ERR_SYMBOL;
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return (int)e;
    g_sms[dev] = n;
    g_ptr[dev] = static_cast<float*>(p);
  }
  *ptr = g_ptr[dev];
  *sms = g_sms[dev];
  return 0;
}

}  // namespace

extern "C" int dfl_rel_l1_noalloc(const void* a, const void* b, long long n, float* out, cudaStream_t stream) {
  if (a == nullptr || b == nullptr || out == nullptr || n < 0) return DFL_NOALLOC_ERR_ARGS;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) return DFL_NOALLOC_ERR_ALIGN;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return DFL_NOALLOC_ERR_ARGS;
  float* scratch = nullptr;
  int sms = 0;
  int rc = setup_device(dev, &scratch, &sms);
  if (rc) return rc;
  long long blocks = (n / 8 + kThreads - 1) / kThreads;
  const long long cap = 4LL * sms;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  if (blocks > DFL_NOALLOC_MAX_BLOCKS) return DFL_NOALLOC_ERR_TOO_LARGE;
  // the completion ticket must start at zero: clear it on the caller's stream
  e = cudaMemsetAsync(scratch, 0, sizeof(float), stream);
  if (e != cudaSuccess) return (int)e;
  rel_l1_noalloc_kernel<<<(int)blocks, kThreads, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(a),
                                                              reinterpret_cast<const __nv_bfloat16*>(b), n,
                                                              scratch, out);
  return (int)cudaGetLastError();
}

extern "C" const char* dfl_rel_l1_noalloc_error_string(int code) {
  switch (code) {
    case 0:
      return "success";
    case DFL_NOALLOC_ERR_ALIGN:
      return "input pointers must be 16-byte aligned";
    case DFL_NOALLOC_ERR_ARGS:
      return "null pointer, negative length or device index out of range";
    case DFL_NOALLOC_ERR_TOO_LARGE:
      return "the reduction would need more blocks than the static scratch holds (DFL_NOALLOC_MAX_BLOCKS)";
    case DFL_NOALLOC_ERR_SYMBOL:
      return "cudaGetSymbolAddress failed for the static scratch array";
    default:
      return code > 0 ? cudaGetErrorString(static_cast<cudaError_t>(code)) : "unknown error";
  }
}
