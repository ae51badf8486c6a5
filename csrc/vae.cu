// Channels-last helpers of the causal video VAE decoders (sm_100a), with the spatial-slab
// halo exchange of the multi-GPU decode fused into their stores.
//
//   chan_norm:  y = x / max(||x||_C, 1e-12) * sqrt(C) * gamma  (RMS over the channels of a
//               pixel, diffusers' ``F.normalize(x, dim=1) * C^0.5 * gamma``), optional SiLU
//   upsample2x: nearest 2x along H and W
//
// Geometry: x is [F, Hl, W, C] (F = batch x frames, Hl = this rank's rows of the frame, C
// channels, contiguous); y is [F, Hl' + 2 halo, W', C] with this rank's rows at row offset
// `halo`.  With halo = 1 the first output row is also stored into the slab above (rank - 1:
// its bottom halo row) and the last output row into the slab below (rank + 1: its top halo
// row), straight into those ranks' buffers over NVLink -- the halo exchange a 3x3 convolution
// of the slab needs is the producer's store pattern, so the convolution then reads its slab
// with one row of context on each side (valid padding along H).  Rows outside the picture
// (top of rank 0, bottom of the last rank) are never written and stay zero.
//
// Reference parity: the RMS norms and nearest upsamplers of the Wan VAE decoder
// (difflet/models/wan/vae/modeling_vae.py:92-551); the reference decodes each frame whole on
// one device (difflet/models/wan/vae/regions.py:64-340), the slab split is this engine's.
#include "common.cuh"
#include "kernels.h"

namespace {
using namespace dfl;

// Store one 16-byte chunk of output row `row` (local row index, halo offset applied by the
// caller) and, for boundary rows, into the neighbours' halo rows.
__device__ __forceinline__ void store_chunk(const VaeRowArgs& a, long long f, int row, int w, int chunk, uint4 v) {
  const long long Wo = a.Wo;
  const long long C = a.C;
  const long long rows_loc = (long long)a.Ho + 2 * a.halo;
  auto* y = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.y) +
                                     ((f * rows_loc + row + a.halo) * Wo + w) * C) + chunk;
  *y = v;
  if (!a.halo) return;
  if (row == 0 && a.up != nullptr) {  // our first row = the bottom halo row of the slab above
    auto* p = reinterpret_cast<__nv_bfloat16*>(a.up) + ((f * (a.up_rows + 2) + a.up_rows + 1) * Wo + w) * C;
    reinterpret_cast<uint4*>(p)[chunk] = v;
  }
  if (row == a.Ho - 1 && a.down != nullptr) {  // our last row = the top halo row of the slab below
    auto* p = reinterpret_cast<__nv_bfloat16*>(a.down) + ((f * (a.down_rows + 2)) * Wo + w) * C;
    reinterpret_cast<uint4*>(p)[chunk] = v;
  }
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.f + __expf(-v)); }

// One warp per pixel; lane l handles 8-channel chunks l, l + 32, ...
__global__ void __launch_bounds__(256) chan_norm_kernel(VaeRowArgs a) {
  const long long pixels = (long long)a.F * a.Ho * a.Wo;
  const int lane = threadIdx.x & 31;
  const int chunks = a.C / 8;
  const float scale = sqrtf((float)a.C);
  const auto* gamma = reinterpret_cast<const __nv_bfloat16*>(a.gamma);
  for (long long p = ((long long)blockIdx.x * blockDim.x + threadIdx.x) / 32; p < pixels;
       p += (long long)gridDim.x * blockDim.x / 32) {
    const auto* xp = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(a.x) + p * a.C);
    uint4 raw[2];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int c = lane + 32 * k;
      if (c < chunks) {
        raw[k] = xp[c];
        const uint32_t wv[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float2 f = unpack_bf16x2(wv[h]);
          ss += f.x * f.x + f.y * f.y;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = scale / fmaxf(sqrtf(ss), 1e-12f);
    const long long f = p / ((long long)a.Ho * a.Wo);
    const int row = (int)((p / a.Wo) % a.Ho), w = (int)(p % a.Wo);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int c = lane + 32 * k;
      if (c >= chunks) continue;
      const uint4 g = reinterpret_cast<const uint4*>(gamma)[c];
      const uint32_t wv[4] = {raw[k].x, raw[k].y, raw[k].z, raw[k].w};
      const uint32_t gv[4] = {g.x, g.y, g.z, g.w};
      uint32_t out[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 xf = unpack_bf16x2(wv[h]), gf = unpack_bf16x2(gv[h]);
        float v0 = xf.x * inv * gf.x, v1 = xf.y * inv * gf.y;
        if (a.silu) v0 = silu_f(v0), v1 = silu_f(v1);
        out[h] = pack_bf16x2(v0, v1);
      }
      store_chunk(a, f, row, w, c, make_uint4(out[0], out[1], out[2], out[3]));
    }
  }
}

// One thread per 16-byte chunk of an input pixel, written to its 2 x 2 output pixels.
__global__ void __launch_bounds__(256) upsample2x_kernel(VaeRowArgs a) {
  const int chunks = a.C / 8;
  const int Hi = a.Ho / 2, Wi = a.Wo / 2;
  const long long total = (long long)a.F * Hi * Wi * chunks;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(i % chunks);
    const long long p = i / chunks;
    const int w = (int)(p % Wi), h = (int)((p / Wi) % Hi);
    const long long f = p / ((long long)Wi * Hi);
    const uint4 v = reinterpret_cast<const uint4*>(a.x)[i];
#pragma unroll
    for (int dy = 0; dy < 2; ++dy)
#pragma unroll
      for (int dx = 0; dx < 2; ++dx) store_chunk(a, f, 2 * h + dy, 2 * w + dx, c, v);
  }
}

int launch_grid(long long work, int per_block) {
  int dev = 0;
  cudaGetDevice(&dev);
  const long long want = (work + per_block - 1) / per_block;
  const long long cap = 16LL * dfl_host::num_sms(dev);
  return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

int check(const VaeRowArgs* a) {
  if (!a->x || !a->y || a->F <= 0 || a->Ho <= 0 || a->Wo <= 0) return -2;
  if (a->C % 8 || a->C > 512) return -3;  // 16-byte chunks, at most two per lane
  auto al = [](const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al(a->x) || !al(a->y) || !al(a->up) || !al(a->down) || !al(a->gamma)) return -4;
  if (!a->halo && (a->up || a->down)) return -5;
  return 0;
}

}  // namespace

extern "C" int dfl_vae_chan_norm(const VaeRowArgs* a, cudaStream_t stream) {
  int rc = check(a);
  if (rc) return rc;
  if (!a->gamma) return -6;
  chan_norm_kernel<<<launch_grid((long long)a->F * a->Ho * a->Wo, 8), 256, 0, stream>>>(*a);
  return (int)cudaGetLastError();
}

extern "C" int dfl_vae_upsample2x(const VaeRowArgs* a, cudaStream_t stream) {
  int rc = check(a);
  if (rc) return rc;
  if (a->Ho % 2 || a->Wo % 2) return -7;
  upsample2x_kernel<<<launch_grid((long long)a->F * (a->Ho / 2) * (a->Wo / 2) * (a->C / 8), 256), 256, 0, stream>>>(*a);
  return (int)cudaGetLastError();
}
