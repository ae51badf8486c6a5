// Channels-last GroupNorm, replicate padding and causal 2x upsampling for the HunyuanVideo-style
// causal 3-D VAE decoder (sm_100a).
//
//   GroupNorm over a whole clip: the statistics of group g of sample n run over every frame,
//   row, column and the group's C / G channels (diffusers' GroupNorm on [N, C, T, H, W]).  Two
//   passes, both deterministic: block partial sums of x, then of (x - mean)^2 (a centred second
//   pass instead of E[x^2] - E[x]^2, which cancels badly over ~10^7 values), each reduced over the
//   blocks in a fixed order; then y = (x - mean) * rstd * gamma + beta (+ SiLU), stored into the
//   interior of the next convolution's input buffer.
//   Replicate padding: the buffer's border frames / rows / columns copy the nearest interior
//   element, per dimension (the corners take the corner values), as a 'replicate' pad does; the
//   convolution then runs with valid_t / valid_h / valid_w.
//   Causal upsampling: nearest 2x along H and W; along T (when asked) the first frame stays one
//   frame and every later frame is repeated twice.
//
// Reference parity: the HunyuanVideo VAE decoder (difflet/models/hunyuan_video/vae/
// modeling_vae.py:85-489: GroupNorm(32) resnets, causal replicate-padded Conv3d, the first-frame
// rule of the upsamplers).
#include "common.cuh"
#include "kernels.h"

namespace {
using namespace dfl;

constexpr int kThreads = 256;

__device__ __forceinline__ float silu_g(float v) { return v / (1.f + __expf(-v)); }

// Block partial of one sample's pixel range: per-channel sums in registers (8 channels per thread),
// then per channel over the threads of the block, then per group -- all in a fixed order.
__global__ void __launch_bounds__(kThreads) gn_partial_kernel(const __nv_bfloat16* x, long long P, int C, int G,
                                                              const float* stats, float* partial) {
  __shared__ float red[kThreads][8];
  __shared__ float csum[1024];
  const int n = blockIdx.y, N = gridDim.y, nblk = gridDim.x, blk = blockIdx.x;
  const int chunks = C / 8, cpg = C / G, rows_per_iter = kThreads / chunks;
  const int t = threadIdx.x, ch = t % chunks, pr = t / chunks;
  const long long begin = P * blk / nblk, end = P * (blk + 1) / nblk;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  float mu[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) mu[j] = stats ? stats[((long long)n * G + (ch * 8 + j) / cpg) * 2] : 0.f;
  const uint4* xp = reinterpret_cast<const uint4*>(x) + (long long)n * P * chunks;
  for (long long p = begin + pr; p < end; p += rows_per_iter) {
    const uint4 v = xp[p * chunks + ch];
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float2 f = unpack_bf16x2(wv[h]);
      if (stats) {
        const float d0 = f.x - mu[2 * h], d1 = f.y - mu[2 * h + 1];
        acc[2 * h] += d0 * d0;
        acc[2 * h + 1] += d1 * d1;
      } else {
        acc[2 * h] += f.x;
        acc[2 * h + 1] += f.y;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[t][j] = acc[j];
  __syncthreads();
  for (int c = t; c < C; c += kThreads) {
    const int c8 = c / 8, j = c % 8;
    float s = 0.f;
    for (int r = 0; r < rows_per_iter; ++r) s += red[r * chunks + c8][j];
    csum[c] = s;
  }
  __syncthreads();
  if (t < G) {
    float s = 0.f;
    for (int k = 0; k < cpg; ++k) s += csum[t * cpg + k];
    partial[((long long)blk * N + n) * G + t] = s;
  }
}

// stats[n][g] = {mean, rstd}: mode 0 writes the mean, mode 1 the reciprocal deviation.
__global__ void gn_finalize_kernel(const float* partial, int nblk, int NG, double count, int mode, float eps,
                                   float* stats) {
  for (int i = threadIdx.x; i < NG; i += blockDim.x) {
    float s = 0.f;
    for (int b = 0; b < nblk; ++b) s += partial[(long long)b * NG + i];
    const float v = (float)(s / count);
    if (mode == 0)
      stats[2 * i] = v;
    else
      stats[2 * i + 1] = rsqrtf(v + eps);
  }
}

__global__ void __launch_bounds__(kThreads) gn_apply_kernel(GnApplyArgs a) {
  const int chunks = a.C / 8, cpg = a.C / a.G;
  const long long total = (long long)a.N * a.T * a.H * a.W * chunks;
  const uint4* xp = reinterpret_cast<const uint4*>(a.x);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int ch = (int)(i % chunks);
    long long p = i / chunks;
    const int w = (int)(p % a.W);
    p /= a.W;
    const int h = (int)(p % a.H);
    p /= a.H;
    const int t = (int)(p % a.T);
    const int n = (int)(p / a.T);
    const uint4 v = xp[i];
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
    uint32_t out[4];
#pragma unroll
    for (int h2 = 0; h2 < 4; ++h2) {
      const float2 f = unpack_bf16x2(wv[h2]);
      float r[2] = {f.x, f.y};
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = ch * 8 + 2 * h2 + e;
        const float* st = a.stats + ((long long)n * a.G + c / cpg) * 2;
        float y = (r[e] - st[0]) * st[1] * a.gamma[c] + a.beta[c];
        r[e] = a.silu ? silu_g(y) : y;
      }
      out[h2] = pack_bf16x2(r[0], r[1]);
    }
    const long long o = ((((long long)n * a.Ty + t + a.ot) * a.Hy + h + a.oh) * a.Wy + w + a.ow) * chunks + ch;
    reinterpret_cast<uint4*>(a.y)[o] = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

// Border elements of y [N, Ty, Hy, Wy, C] around the interior box at (pt, ph, pw) of size
// (T, H, W): each copies the nearest interior element (clamped per dimension).
__global__ void __launch_bounds__(kThreads) pad_replicate_kernel(PadArgs a) {
  const int chunks = a.C / 8;
  const long long total = (long long)a.N * a.Ty * a.Hy * a.Wy * chunks;
  uint4* yp = reinterpret_cast<uint4*>(a.y);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int ch = (int)(i % chunks);
    long long p = i / chunks;
    const int w = (int)(p % a.Wy);
    p /= a.Wy;
    const int h = (int)(p % a.Hy);
    p /= a.Hy;
    const int t = (int)(p % a.Ty);
    const int n = (int)(p / a.Ty);
    const int ts = min(max(t, a.pt), a.pt + a.T - 1);
    const int hs = min(max(h, a.ph), a.ph + a.H - 1);
    const int ws = min(max(w, a.pw), a.pw + a.W - 1);
    if (ts == t && hs == h && ws == w) continue;  // interior
    yp[i] = yp[((((long long)n * a.Ty + ts) * a.Hy + hs) * a.Wy + ws) * chunks + ch];
  }
}

// Nearest 2x along H, W; along T (up_t) frame 0 stays one frame, frame f >= 1 becomes 2f - 1, 2f.
__global__ void __launch_bounds__(kThreads) upsample_causal_kernel(UpsampleArgs a) {
  const int chunks = a.C / 8;
  const int To = a.up_t ? 2 * a.T - 1 : a.T, Ho = 2 * a.H, Wo = 2 * a.W;
  const long long total = (long long)a.N * To * Ho * Wo * chunks;
  const uint4* xp = reinterpret_cast<const uint4*>(a.x);
  uint4* yp = reinterpret_cast<uint4*>(a.y);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int ch = (int)(i % chunks);
    long long p = i / chunks;
    const int w = (int)(p % Wo);
    p /= Wo;
    const int h = (int)(p % Ho);
    p /= Ho;
    const int t = (int)(p % To);
    const int n = (int)(p / To);
    const int ti = (a.up_t && t > 0) ? 1 + (t - 1) / 2 : t;
    const uint4 v = xp[((((long long)n * a.T + ti) * a.H + h / 2) * a.W + w / 2) * chunks + ch];
    yp[((((long long)n * a.Ty + t + a.ot) * a.Hy + h + a.oh) * a.Wy + w + a.ow) * chunks + ch] = v;
  }
}

int grid_for(long long work) {
  int dev = 0;
  cudaGetDevice(&dev);
  const long long want = (work + kThreads - 1) / kThreads;
  const long long cap = 16LL * dfl_host::num_sms(dev);
  return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" int dfl_gn_stats(const void* x, int N, long long P, int C, int G, float eps, float* partial, int nblk,
                            float* stats, cudaStream_t stream) {
  if (!x || !partial || !stats || N <= 0 || P <= 0 || G <= 0 || nblk <= 0) return -2;
  if (C % 8 || C > 1024 || C % G || kThreads % (C / 8) || G > kThreads) return -3;
  if (!al16(x)) return -4;
  const double count = (double)P * (C / G);
  const dim3 grid(nblk, N);
  gn_partial_kernel<<<grid, kThreads, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x), P, C, G, nullptr,
                                                   partial);
  gn_finalize_kernel<<<1, kThreads, 0, stream>>>(partial, nblk, N * G, count, 0, eps, stats);
  gn_partial_kernel<<<grid, kThreads, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x), P, C, G, stats,
                                                   partial);
  gn_finalize_kernel<<<1, kThreads, 0, stream>>>(partial, nblk, N * G, count, 1, eps, stats);
  return (int)cudaGetLastError();
}

extern "C" int dfl_gn_apply(const GnApplyArgs* a, cudaStream_t stream) {
  if (!a->x || !a->y || !a->stats || !a->gamma || !a->beta) return -2;
  if (a->C % 8 || a->C % a->G) return -3;
  if (!al16(a->x) || !al16(a->y)) return -4;
  if (a->ot < 0 || a->oh < 0 || a->ow < 0 || a->ot + a->T > a->Ty || a->oh + a->H > a->Hy || a->ow + a->W > a->Wy)
    return -5;
  gn_apply_kernel<<<grid_for((long long)a->N * a->T * a->H * a->W * (a->C / 8)), kThreads, 0, stream>>>(*a);
  return (int)cudaGetLastError();
}

extern "C" int dfl_pad_replicate(const PadArgs* a, cudaStream_t stream) {
  if (!a->y || a->C % 8 || !al16(a->y)) return -2;
  if (a->T <= 0 || a->H <= 0 || a->W <= 0 || a->pt < 0 || a->ph < 0 || a->pw < 0 || a->pt + a->T > a->Ty ||
      a->ph + a->H > a->Hy || a->pw + a->W > a->Wy)
    return -3;
  pad_replicate_kernel<<<grid_for((long long)a->N * a->Ty * a->Hy * a->Wy * (a->C / 8)), kThreads, 0, stream>>>(*a);
  return (int)cudaGetLastError();
}

extern "C" int dfl_upsample_causal(const UpsampleArgs* a, cudaStream_t stream) {
  if (!a->x || !a->y || a->C % 8 || !al16(a->x) || !al16(a->y)) return -2;
  const int To = a->up_t ? 2 * a->T - 1 : a->T;
  if (a->ot < 0 || a->oh < 0 || a->ow < 0 || a->ot + To > a->Ty || a->oh + 2 * a->H > a->Hy ||
      a->ow + 2 * a->W > a->Wy)
    return -3;
  upsample_causal_kernel<<<grid_for((long long)a->N * To * 4 * a->H * a->W * (a->C / 8)), kThreads, 0, stream>>>(*a);
  return (int)cudaGetLastError();
}
