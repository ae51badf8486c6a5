// C interface between the sm_100a kernels (plain CUDA translation units, no
// torch headers) and the torch bindings.  Every launcher returns 0 on success
// and a non-zero code otherwise; device-side failures land in `err` (see
// common.cuh for the error-word protocol).
#pragma once
#include <cuda_runtime_api.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { kEpiNone = 0, kEpiGelu = 1, kEpiGateResid = 2, kEpiSilu = 3, kEpiSwiGLU = 4, kEpiQkv = 5 };
// kEpiSwiGLU: the weight rows are interleaved in 32-row groups [h_32 | g_32] and the
// GEMM writes N/2 columns  out = (h + b_h) * silu(g + b_g).
// kEpiQkv: the q / k / v column blocks named by GemmArgs.qkv are normalised, rotated and
// scattered by head exactly as dfl_qkv_scatter would do on the stored rows (no round trip
// through D); every other column takes the GELU window epilogue into D.

struct QkvScatterArgs;

#define DFL_MAX_PEERS 8

typedef struct GemmArgs {
  const void* A;   // bf16 [M, K], row stride lda (elements)
  const void* B;   // bf16 [N, K], row stride ldb
  void* D;         // bf16 or f32 [M, N], row stride ldd
  long long lda, ldb, ldd;
  int M, N, K;
  int out_f32;
  const void* bias;  // bf16 [N] or NULL
  int epi;           // kEpi*
  int act_lo, act_hi;  // activation column window for GELU / SiLU
  const float* gate;   // f32 [batch, gate_bstride] for kEpiGateResid
  long long gate_bstride;
  int rows_per_batch;
  const int* gate_row_map;  // optional: gate row of every output row (packed sequences)
  const void* resid;   // bf16 [M, ldr] (may alias D)
  long long ldr;
  float alpha;         // scales the accumulator before bias
  int* err;
  // Row scatter (out_world > 0): row r is stored to out_peer[r / rows_per_rank]
  // at row peer_row_off + r % rows_per_rank with stride ldd (tensor-parallel
  // partial sums sent to the rank that reduces them); D is unused then.
  void* out_peer[DFL_MAX_PEERS];
  int out_world;
  int rows_per_rank;
  long long peer_row_off;
  // 0: automatic choice, 1: one CTA per 128 x BN tile, 2: CTA pairs (cta_group::2, 256 x 256 tiles),
  // 3: one CTA per 128 x 128 tile (six operand stages)
  int cta_mode;
  // kEpiQkv: the head scatter applied in the epilogue (its qkv / ld / rows fields are unused;
  // the source rows are the GEMM rows).  Per-head RMS (norm_mode 0 / 1), full-width RoPE,
  // dh 64 or 128, column offsets multiples of dh.
  const struct QkvScatterArgs* qkv;
} GemmArgs;

int dfl_gemm_bf16(const GemmArgs* a, cudaStream_t stream);
// Split-K workspace of `device` (f32 partial tiles + int counters that must start at 0 and
// are left at 0 by every launch); GEMMs that use it must not run concurrently on the device.
void dfl_gemm_set_split_workspace(int device, void* ws, long long ws_bytes, void* sem, int sem_count);
void dfl_gemm_set_epi_warps(int n);  // pair-kernel epilogue warps: 0 auto (8 for the q/k/v scatter), 4 or 8
// Up to 2 GEMMs with the same epilogue kind and output type in one persistent launch
// (their tiles share the grid; the tile shape follows args[0]).
int dfl_gemm_bf16_group(const GemmArgs* const* args, int count, cudaStream_t stream);
void dfl_gemm_set_pair_auto(int on);
void dfl_gemm_set_split_force(int s);  // measurement: 0 = modelled split-K choice, 1..4 = forced K ranges

// MXFP8 GEMM on the block-scaled tensor cores (tcgen05 kind::mxf8f6f4):
//   D = epi(A . B^T), A [M, K] / B [N, K] FP8 E4M3 (K-major, row strides in
//   bytes g.lda / g.ldb), one E8M0 scale per 32 K values in the blocked layout
//   written by dfl_mx_quantize (128-row x 128-K atoms of 512 bytes).  The
//   epilogue fields of g are those of dfl_gemm_bf16; g.A / g.B are the FP8 data.
typedef struct MxGemmArgs {
  GemmArgs g;
  const void* sfa;   // uint8 blocked scales of A (rows padded to 128)
  const void* sfb;   // uint8 blocked scales of B
} MxGemmArgs;
int dfl_gemm_mx(const MxGemmArgs* a, cudaStream_t stream);

// bf16 [R, K] -> FP8 E4M3 [R, K] (row stride ldq bytes) + E8M0 scales, one per
// 32 K values (OCP MX: exponent = floor(log2(amax)) - 8, saturating convert).
// blocked = 1: the tensor-core layout (atom (r/128, k/128) at byte
// ((r/128) * (K/128) + k/128) * 512, inside it (r%32)*16 + ((r%128)/32)*4 +
// (k/32)%4; rows padded to 128), blocked = 0: plain [R, K/32].
int dfl_mx_quantize(const void* x, long long ldx, int R, int K, void* q, long long ldq, void* scales,
                    int blocked, cudaStream_t stream);

// y = (LN(x) [* w + b]) [* (1 + scale[b]) + shift[b]]      (fp32 statistics)
typedef struct LnModArgs {
  const void* x; long long ldx;      // bf16 [M, D]
  void* y; long long ldy;            // bf16 [M, D]
  const void* w; const void* b;      // bf16 [D] affine or NULL
  const float* shift; const float* scale;  // f32 [batch, mod_bstride] or NULL
  long long mod_bstride;
  int rows_per_batch;
  int M, D;
  float eps;
  int rms;                           // 1: RMSNorm (no mean subtraction, no bias)
  const int* row_map;                // optional: modulation row of every row (packed sequences)
  // Sequence-parallel all-gather fused into the norm: process rows [row0, row0 + M) only
  // and store each output row into y_peer[0..y_world) (every rank's full buffer) instead of y.
  long long row0;
  void* y_peer[DFL_MAX_PEERS];
  int y_world;
} LnModArgs;
int dfl_ln_modulate(const LnModArgs* a, cudaStream_t stream);

// q/k RMSNorm + RoPE + scatter to head-major [B, H_local, S_dst, dh] buffers.
// Source rows are tokens; destination tables hold one pointer per rank so the
// same pass performs the Ulysses sequence->head all-to-all over NVLink stores.
typedef struct QkvScatterArgs {
  const void* qkv; long long ld;     // bf16 [rows, ld]
  int q_off, k_off, v_off;           // column offsets of the q / k / v blocks
  int rows, S_src;                   // rows = B * S_src
  int H, dh;                         // heads in the source row, head dim
  int norm_mode;                     // 0 none, 1 per-head RMS, 2 across-heads RMS
  const void* wq; const void* wk;    // bf16 [dh] (mode 1) or [H*dh] (mode 2), may be NULL
  float eps;
  const float* cos_t; const float* sin_t;  // f32 [pos, dh/2] or NULL (no RoPE)
  int rope_pos_off;                  // table row = rope_pos_off + s
  int rope_half;                     // 0 interleaved pairs, 1 half-split
  int world, heads_per_rank;
  void* q_dst[DFL_MAX_PEERS]; void* k_dst[DFL_MAX_PEERS]; void* v_dst[DFL_MAX_PEERS];
  int S_dst, seq_off;                // destination seq length / offset of row 0
  int out_token_major;               // 1: dst is [B, S_dst, H_local*dh] instead
  // Gather-KV context parallelism: k / v of every head go to all `world`
  // destinations (heads_per_rank == H), q only to q_dst[0] with its own
  // sequence length / offset (the local query rows).
  int kv_replicate;
  int q_S_dst, q_seq_off;
  // 0: one RoPE table row [dh/2] per position shared by all heads; n > 0: each
  // row holds n heads' tables ([n * dh/2], head h uses slice h) -- rotary
  // frequencies spread over the whole inner dimension.
  int rope_heads;
  // Rotary applied to the first rope_dims channels of each head (half-split pairs
  // (i, i + rope_dims/2)), the rest passed through; 0 = all dh channels.
  int rope_dims;
  // Two-segment rows (a rank's [text ; image] slice of a joint sequence): source rows
  // s >= seg_rows of each batch land at seg1_seq_off + (s - seg_rows) and use RoPE
  // table row seg1_rope_off + (s - seg_rows).  0 = one segment.
  int seg_rows, seg1_seq_off, seg1_rope_off;
  // norm_mode 3 (across-heads RMS under tensor parallelism): the row's sum of squares
  // over ALL heads, already reduced across ranks: row_sumsq[2 r] (q), [2 r + 1] (k);
  // rstd = rsqrt(sum / norm_total + eps), the weights wq / wk hold this rank's heads.
  const float* row_sumsq;
  int norm_total;
} QkvScatterArgs;
int dfl_qkv_scatter(const QkvScatterArgs* a, cudaStream_t stream);

// Per-row partial sums of squares of two column blocks (q and k of a tensor-parallel
// shard): out[2 r + i] = sum_c x[r, off_i + c]^2 over c < width (0 when off_i < 0).
int dfl_row_sumsq(const void* x, long long ld, int rows, int off0, int off1, int width, float* out,
                  cudaStream_t stream);

// y[b, n] = act_in(x[b, :]) . W[n, :] + bias[n]   (bf16 W, f32 x / y; batch <= 8)
typedef struct GemvArgs {
  const void* W; long long ldw;      // bf16 [N, K]
  const float* x; int batch;         // f32 [batch, K]
  const void* bias;                  // bf16 [N] or NULL
  float* y; long long ldy;           // f32 [batch, ldy]
  int N, K;
  int silu_in;                       // apply SiLU to x first
  int silu_out;                      // apply SiLU to y
} GemvArgs;
int dfl_gemv(const GemvArgs* a, cudaStream_t stream);

// Flow-matching Euler with optional CFG combine:
//   v = u + s (c - u)  (when cond != NULL), x32 += dt * v, x16 = bf16(x32)
typedef struct SchedArgs {
  float* x32; void* x16;             // f32 master latents, optional bf16 mirror
  const void* v;                     // bf16 prediction (uncond when cond != NULL)
  const void* cond;                  // bf16 cond prediction or NULL
  long long n;
  float dt, guidance;
} SchedArgs;
int dfl_euler_step(const SchedArgs* a, cudaStream_t stream);

// Guidance combine fused with a sampler update (sched.cu), u = (x, last, m1, m2, m):
//   v = a + scale (b - a) (b NULL: v = a; swap_ab: v = b + scale (a - b)); m = x + k_v v;
//   xc = e . u; xn = g[0..4] . u + g[5] v;
//   x <- xn, x16 <- bf16(xn) (x16 != NULL), last <- xc (store_last), m_out <- m (m_out != NULL).
// a / b bf16 (either may be a peer rank's buffer), x / last / m1 / m2 / m_out f32, all n elements,
// 16-byte aligned; NULL last / m1 / m2 read as zero.  m_out may alias m2 (each element is read
// before it is written).
typedef struct GuidedStepArgs {
  const void* a;
  const void* b;
  float scale;
  float* x;
  void* x16;
  float* last;
  const float* m1;
  const float* m2;
  float* m_out;
  long long n;
  float k_v;
  float e[5];
  float g[6];
  int store_last;
  int swap_ab;
} GuidedStepArgs;
int dfl_guided_step(const GuidedStepArgs* a, cudaStream_t stream);

// Sinusoidal timestep features: out[b, :] = [cos(t f) | sin(t f)] (flip) or [sin | cos].
int dfl_timestep_embed(const float* t, int batch, int dim, float max_period, int flip_sin_to_cos,
                       float downscale_freq_shift, float scale, float* out, cudaStream_t stream);

// Flash attention forward, bf16 in / bf16 out, fp32 softmax.
typedef struct AttnArgs {
  const void* q; const void* k; const void* v;  // [B, H, S, dh] (strides below)
  void* o;                                      // output
  long long q_bs, q_hs, q_ss;                   // element strides (batch, head, seq)
  long long k_bs, k_hs, k_ss;
  long long v_bs, v_hs, v_ss;
  long long o_bs, o_hs, o_ss;
  float* lse;                                   // f32 [B, H, Sq] natural-log LSE or NULL
  int B, H, Sq, Sk, dh;
  float scale;
  const int* kv_lo; const int* kv_hi;           // per-batch key window [lo, hi) or NULL
  int* err;
  // Output scatter (Ulysses head->sequence all-to-all in the epilogue): when
  // o_world > 1, query row s is stored at o_peer[owner(s)] + b*o_bs + h*o_hs +
  // local_row(s)*o_ss.  Rows form two segments: the first seg0_len rows are
  // split seg0_per per rank and land first in each owner's local layout; the
  // remaining rows are split seg1_per per rank and land after them.
  void* o_peer[DFL_MAX_PEERS];
  int o_world;
  int seg0_len, seg0_per, seg1_per;
  // Log-sum-exp merge of key-block partials (ring / gather context parallelism):
  // merge_mode 1 writes this partial to acc_o / acc_lse, 2 merges into them,
  // 3 merges and writes the final bf16 output.  acc_o f32 [B, H, Sq, 128].
  float* acc_o;
  float* acc_lse;
  int merge_mode;
  // Split-KV (launches whose query blocks leave SMs idle): kv_splits CTAs share a query
  // block, each over a contiguous key range, writing its normalised partial and LSE to
  // split_o f32 [kv_splits][B*H*Sq][128] / split_lse [kv_splits][B*H*Sq]; a combine pass
  // merges them by log-sum-exp into the output.  Ask dfl_attention_plan_splits first.
  int kv_splits;
  float* split_o;
  float* split_lse;
} AttnArgs;
int dfl_attention(const AttnArgs* a, cudaStream_t stream);
// Key-range split count that minimises the modelled time of this launch (1 = none).
int dfl_attention_plan_splits(const AttnArgs* a);

// ---------------------------------------------------------------------------
// Peer-memory communication runtime (comm.cu)
// ---------------------------------------------------------------------------
int dfl_ipc_handle(const void* ptr, void* out64);
int dfl_ipc_open(const void* handle64, void** out);
int dfl_ipc_close(void* ptr);

typedef struct BarrierArgs {
  int* flags[DFL_MAX_PEERS];  // flags[r] = rank r's flag array (world ints), peer-mapped
  int* counter;               // this rank's device epoch counter
  int rank, world;
  long long timeout_cycles;
  int* err;
} BarrierArgs;
int dfl_peer_barrier(const BarrierArgs* a, cudaStream_t stream);

typedef struct PeerPutArgs {
  const float* src; long long n;
  float* dst[DFL_MAX_PEERS];  // every rank's destination buffer
  long long dst_offset;       // element offset of this rank's slice
  int world;
} PeerPutArgs;
int dfl_peer_put_f32(const PeerPutArgs* a, cudaStream_t stream);

// Tensor-parallel reduction of row-parallel partials (the second half of the
// fused GEMM -> reduce-scatter / all-reduce): this rank owns `rows` rows starting
// at global row row0; slots holds every source rank's bf16 partial of them
// ([world][slot_rows][N], written by the GEMM epilogue's row scatter).  y = sum +
// bias, optionally resid + gate[b] * y, stored to out[0..out_world) at row row0 + r
// (out_world = tp: all-reduce; 1: reduce-scatter for sequence parallelism).
typedef struct TpReduceArgs {
  const void* slots;
  long long slot_rows;
  int world, rows, N;
  long long row0;
  const void* bias;                     // bf16 [N] or NULL
  const float* gate; long long gate_bstride; int rows_per_batch;  // gated residual or NULL
  const void* resid; long long ldr;     // bf16, indexed by global row
  void* out[DFL_MAX_PEERS]; long long ldo; int out_world;
  long long out_row0;                   // row of out that receives global row row0
  long long resid_row0;                 // global row held by resid's row 0
} TpReduceArgs;
int dfl_tp_reduce(const TpReduceArgs* a, cudaStream_t stream);

// Implicit-GEMM convolution, stride 1, kernel 1 or 3 per axis, channels-last bf16:
// x [N, T, H, W, Ci], w [Co, kt*kh*kw, Ci] (tap-major: t, h, w), y [N, T, H, W, Co].
// Spatial zero padding k/2; temporal causal (kt - 1 frames in front) or symmetric.
// Ci a multiple of 32, Co a multiple of 32.  Optional bias, residual (y = resid + conv,
// `ones` = f32 [Co] of ones), SiLU.
typedef struct ConvArgs {
  const void* x; const void* w; void* y;
  const void* bias; const void* resid; const float* ones;
  int N, T, H, W, Ci, Co;  // input extents (x is [N, T, H, W, Ci])
  int kt, kh, kw, causal, silu;
  // valid_t: no temporal padding (the input already starts with the causal context, e.g. a
  // streaming cache), T_out = T - kt + 1; valid_h: no padding along H (the input carries halo
  // rows from the neighbouring spatial slabs), H_out = H - kh + 1; valid_w: no padding along W
  // (the input carries its own border columns, e.g. replicate padding), W_out = W - kw + 1.
  // Otherwise T / H / W are kept.
  int valid_t, valid_h, valid_w;
  int* err;
} ConvArgs;
int dfl_conv3d(const ConvArgs* a, cudaStream_t stream);

// Channels-last VAE helpers (vae.cu) on spatial slabs.  x [F, Hl, W, C]; y [F, Ho + 2 halo, Wo, C]
// (this rank's Ho rows after `halo` rows of context); with halo the first / last output rows are
// also stored into the slab above (`up`: a peer's y with up_rows own rows) / below (`down`).
typedef struct VaeRowArgs {
  const void* x; void* y;
  const void* gamma;          // chan_norm: [C] bf16
  int F, Ho, Wo, C;           // frames, output rows / width of this rank's slab, channels (% 8)
  int halo;
  void* up; int up_rows;
  void* down; int down_rows;
  int silu;
} VaeRowArgs;
// y = silu?(x / max(||x||_C, 1e-12) * sqrt(C) * gamma), Ho = Hl, Wo = W
int dfl_vae_chan_norm(const VaeRowArgs* a, cudaStream_t stream);
// nearest 2x upsample: Ho = 2 Hl, Wo = 2 W
int dfl_vae_upsample2x(const VaeRowArgs* a, cudaStream_t stream);

// Channels-last GroupNorm / replicate padding / causal upsampling of the HunyuanVideo-style VAE
// (vae_gn.cu).  Volumes are bf16 [N, T, H, W, C] contiguous, C a multiple of 8; destinations are
// larger buffers [N, Ty, Hy, Wy, C] written at the offset (ot, oh, ow).
// Clip statistics of GroupNorm(G): stats f32 [N][G][2] = {mean, 1 / sqrt(var + eps)} over the
// P = T * H * W pixels and C / G channels of each group; partial: f32 scratch [nblk][N][G].
int dfl_gn_stats(const void* x, int N, long long P, int C, int G, float eps, float* partial, int nblk,
                 float* stats, cudaStream_t stream);
typedef struct GnApplyArgs {
  const void* x; void* y; const float* stats; const float* gamma; const float* beta;  // gamma / beta f32 [C]
  int N, T, H, W, C, G;
  int Ty, Hy, Wy, ot, oh, ow;
  int silu;
} GnApplyArgs;
int dfl_gn_apply(const GnApplyArgs* a, cudaStream_t stream);
typedef struct PadArgs {  // fill the border of y around its interior box (pt, ph, pw) + (T, H, W)
  void* y;
  int N, Ty, Hy, Wy, C;
  int pt, ph, pw, T, H, W;
} PadArgs;
int dfl_pad_replicate(const PadArgs* a, cudaStream_t stream);
typedef struct UpsampleArgs {  // nearest 2x in H, W; up_t: frame 0 once, later frames twice
  const void* x; void* y;
  int N, T, H, W, C, up_t;
  int Ty, Hy, Wy, ot, oh, ow;
} UpsampleArgs;
int dfl_upsample_causal(const UpsampleArgs* a, cudaStream_t stream);

// Copy-engine copy (peer -> local over NVLink; no SM work, no kernel).
int dfl_memcpy_async(void* dst, const void* src, long long nbytes, cudaStream_t stream);

// CFG-parallel: out (f32) = u + s (c - u), partner branch read over NVLink.
int dfl_cfg_combine(const void* mine, const void* peer, float* out, long long n, float scale,
                    int mine_is_cond, cudaStream_t stream);

// TeaCache probe: out = sum|a - b| / sum|b| (bf16 inputs, f32 scalar out).  `scratch`
// holds dfl_rel_l1_scratch_floats(blocks) floats, zero on first use (the kernel
// leaves its ticket at zero again for the next call).
long long dfl_rel_l1_scratch_floats(int blocks);
int dfl_rel_l1_blocks(long long n, int num_sms);
int dfl_rel_l1(const void* a, const void* b, long long n, float* scratch, int blocks, float* out,
               cudaStream_t stream);

#ifdef __cplusplus
}
#endif
