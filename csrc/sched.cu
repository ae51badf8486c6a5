// Guidance combine fused with the sampler update (one pass over the latents).
//
// Per element, with every coefficient a host-computed scalar of this step and
// u = (x, last, m1, m2, m) the element's sampler state:
//   v   = a + s (b - a)                       guidance combine (b == NULL: v = a)
//   m   = x + k_v v                           data prediction (flow matching: k_v = -sigma)
//   xc  = e . u                               corrected sample (UniC; e = (1,0,0,0,0) without)
//   xn  = g . u + g_v v                       next sample (UniP through xc, or Euler: g_x = 1, g_v = dt)
//   x <- xn, x16 <- bf16(xn), last <- xc (store_last), m_out <- m (m_out != NULL)
// a / b are the bf16 uncond / cond predictions (swap_ab: b is uncond); under CFG parallelism
// a is this rank's branch and b the partner rank's buffer, read over NVLink by this kernel (the cond/uncond exchange is its
// load pattern), and both ranks compute the identical update.  The multistep history
// (m1 = previous data prediction, m2 = the one before, last = previous corrected sample)
// stays in f32 on the device; the host rotates the buffers, so nothing is copied.
//
// UniPC (bh2, order <= 2) is linear in u, so its corrector and predictor reduce to the e / g
// weights of the step, which the host derives from the scheduler's own update rule.
//
// Reference parity: CFG combine difflet/models/wan/pipeline.py:403-405, UniPC steps
// :525-582, FLUX / Qwen Euler difflet/models/flux/pipeline.py:414-420.
#include "common.cuh"
#include "kernels.h"

namespace {
using namespace dfl;

__device__ __forceinline__ void load8_bf16(const __nv_bfloat16* p, long long i, float (&r)[8]) {
  const uint4 q = reinterpret_cast<const uint4*>(p)[i];
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    const float2 f = unpack_bf16x2(w[h]);
    r[2 * h] = f.x;
    r[2 * h + 1] = f.y;
  }
}

__device__ __forceinline__ void load8_f32(const float* p, long long i, float (&r)[8]) {
  const float4 lo = reinterpret_cast<const float4*>(p)[2 * i];
  const float4 hi = reinterpret_cast<const float4*>(p)[2 * i + 1];
  r[0] = lo.x, r[1] = lo.y, r[2] = lo.z, r[3] = lo.w, r[4] = hi.x, r[5] = hi.y, r[6] = hi.z, r[7] = hi.w;
}

__device__ __forceinline__ void store8_f32(float* p, long long i, const float (&r)[8]) {
  reinterpret_cast<float4*>(p)[2 * i] = make_float4(r[0], r[1], r[2], r[3]);
  reinterpret_cast<float4*>(p)[2 * i + 1] = make_float4(r[4], r[5], r[6], r[7]);
}

struct Elem {
  float v, m, xc, xn;
};

__device__ __forceinline__ Elem update(const GuidedStepArgs& a, float va, float vb, float x, float last, float m1,
                                       float m2) {
  Elem e;
  if (a.b) {
    const float u = a.swap_ab ? vb : va, c = a.swap_ab ? va : vb;  // the same formula on every rank
    e.v = u + a.scale * (c - u);
  } else {
    e.v = va;
  }
  e.m = x + a.k_v * e.v;
  e.xc = a.e[0] * x + a.e[1] * last + a.e[2] * m1 + a.e[3] * m2 + a.e[4] * e.m;
  e.xn = a.g[0] * x + a.g[1] * last + a.g[2] * m1 + a.g[3] * m2 + a.g[4] * e.m + a.g[5] * e.v;
  return e;
}

__global__ void __launch_bounds__(256) guided_step_kernel(GuidedStepArgs a) {
  const auto* A = reinterpret_cast<const __nv_bfloat16*>(a.a);
  const auto* Bp = reinterpret_cast<const __nv_bfloat16*>(a.b);
  auto* x16 = reinterpret_cast<__nv_bfloat16*>(a.x16);
  const long long n8 = a.n / 8;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += stride) {
    float va[8], vb[8], x[8], last[8], m1[8], m2[8];
    load8_bf16(A, i, va);
    if (Bp) load8_bf16(Bp, i, vb);
    load8_f32(a.x, i, x);
#pragma unroll
    for (int t = 0; t < 8; ++t) last[t] = m1[t] = m2[t] = 0.f;
    if (a.last) load8_f32(a.last, i, last);
    if (a.m1) load8_f32(a.m1, i, m1);
    if (a.m2) load8_f32(a.m2, i, m2);
    float xc[8], xn[8], m[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const Elem e = update(a, va[t], Bp ? vb[t] : 0.f, x[t], last[t], m1[t], m2[t]);
      xc[t] = e.xc, xn[t] = e.xn, m[t] = e.m;
    }
    store8_f32(a.x, i, xn);
    if (a.store_last) store8_f32(a.last, i, xc);
    if (a.m_out) store8_f32(a.m_out, i, m);
    if (x16) {
      uint4 q;
      q.x = pack_bf16x2(xn[0], xn[1]);
      q.y = pack_bf16x2(xn[2], xn[3]);
      q.z = pack_bf16x2(xn[4], xn[5]);
      q.w = pack_bf16x2(xn[6], xn[7]);
      reinterpret_cast<uint4*>(x16)[i] = q;
    }
  }
  // ragged tail (n not a multiple of 8)
  for (long long i = n8 * 8 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += stride) {
    const float va = __bfloat162float(A[i]), vb = Bp ? __bfloat162float(Bp[i]) : 0.f;
    const float last = a.last ? a.last[i] : 0.f;
    const float m1 = a.m1 ? a.m1[i] : 0.f, m2 = a.m2 ? a.m2[i] : 0.f;
    const Elem e = update(a, va, vb, a.x[i], last, m1, m2);
    a.x[i] = e.xn;
    if (a.store_last) a.last[i] = e.xc;
    if (a.m_out) a.m_out[i] = e.m;
    if (x16) x16[i] = __float2bfloat16(e.xn);
  }
}

}  // namespace

extern "C" int dfl_guided_step(const GuidedStepArgs* a, cudaStream_t stream) {
  if (!a->a || !a->x || a->n < 0) return -2;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al(a->a) || !al(a->x) || (a->b && !al(a->b)) || (a->last && !al(a->last)) || (a->m1 && !al(a->m1)) ||
      (a->m2 && !al(a->m2)) || (a->m_out && !al(a->m_out)) || (a->x16 && !al(a->x16)))
    return -3;
  if (a->store_last && !a->last) return -4;
  if (a->n == 0) return 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const long long want = (a->n / 8 + 255) / 256 + 1;
  const long long cap = 8LL * dfl_host::num_sms(dev);
  guided_step_kernel<<<(int)(want < cap ? want : cap), 256, 0, stream>>>(*a);
  return (int)cudaGetLastError();
}
