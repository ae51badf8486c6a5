// torch bindings for the difflet_b200 sm_100a kernels.
//
// The kernels live in torch-free .cu translation units behind the C interface
// in kernels.h; this file only validates tensors, picks strides and streams,
// and forwards.  Every entry point raises on a non-zero launcher status.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <algorithm>
#include <string>
#include <vector>

#include "kernels.h"

namespace {

#define DFL_CHECK_RC(rc, what) TORCH_CHECK((rc) == 0, what, " launch failed with status ", (rc))

void check_bf16_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
}

void check_rowmajor(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.dim() == 2, name, " must be 2-D");
  TORCH_CHECK(t.stride(1) == 1, name, " must have a unit inner stride");
}

// Per-device 4-int error word (see common.cuh).
at::Tensor& error_buffer(int device) {
  static at::Tensor bufs[16];
  TORCH_CHECK(device >= 0 && device < 16, "device index out of range");
  if (!bufs[device].defined()) {
    bufs[device] = at::zeros({4}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, device));
  }
  return bufs[device];
}

int* err_ptr() {
  int dev = c10::cuda::current_device();
  return error_buffer(dev).data_ptr<int>();
}

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

const void* opt_ptr(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? t->data_ptr() : nullptr;
}

// ---------------------------------------------------------------------------
// Output + epilogue fields shared by the bf16 and MXFP8 GEMMs.  With out_peer
// (tensor-parallel row scatter) rows go to peer buffers and no local D exists.
static at::Tensor gemm_epilogue_args(GemmArgs& a, const at::Tensor& A, int64_t M, int64_t N,
                                     const c10::optional<at::Tensor>& bias, c10::optional<at::Tensor> out,
                                     int64_t epi, int64_t act_lo, int64_t act_hi,
                                     const c10::optional<at::Tensor>& gate, int64_t rows_per_batch,
                                     const c10::optional<at::Tensor>& resid, double alpha, bool out_f32,
                                     const std::vector<int64_t>& out_peer, int64_t rows_per_rank,
                                     int64_t peer_row_off, int64_t ldd_peer,
                                     const c10::optional<at::Tensor>& gate_row_map, const std::string& qkv_plan) {
  at::Tensor D;
  const int64_t N_out = epi == kEpiSwiGLU ? N / 2 : N;
  if (epi == kEpiQkv) {
    TORCH_CHECK(qkv_plan.size() == sizeof(QkvScatterArgs), "epi=qkv needs a qkv_plan (from qkv_plan())");
    a.qkv = reinterpret_cast<const QkvScatterArgs*>(qkv_plan.data());
    TORCH_CHECK(!out_f32 && out_peer.empty(), "the qkv epilogue stores bf16 locally");
  }
  if (epi == kEpiQkv && !(out.has_value() && out->defined())) {
    D = at::empty({0}, A.options());  // every column goes to the head scatter (checked natively)
    a.D = nullptr;
    a.ldd = 0;
  } else if (!out_peer.empty()) {
    TORCH_CHECK(out_peer.size() <= DFL_MAX_PEERS, "at most 8 output peers");
    TORCH_CHECK(rows_per_rank > 0 && ldd_peer > 0, "out_peer needs rows_per_rank and ldd");
    a.out_world = (int)out_peer.size();
    for (size_t r = 0; r < out_peer.size(); ++r) a.out_peer[r] = reinterpret_cast<void*>(out_peer[r]);
    a.rows_per_rank = (int)rows_per_rank;
    a.peer_row_off = peer_row_off;
    a.ldd = ldd_peer;
    D = at::empty({0}, A.options());
  } else {
    if (out.has_value() && out->defined()) {
      D = *out;
      check_rowmajor(D, "out");
      TORCH_CHECK(D.size(0) == M && D.size(1) == N_out, "out shape mismatch");
      TORCH_CHECK(D.scalar_type() == (out_f32 ? at::kFloat : at::kBFloat16), "out dtype mismatch");
    } else {
      D = at::empty({M, N_out}, A.options().dtype(out_f32 ? at::kFloat : at::kBFloat16));
    }
    a.D = D.data_ptr();
    a.ldd = D.stride(0);
  }
  a.M = (int)M;
  a.N = (int)N;
  a.out_f32 = out_f32 ? 1 : 0;
  if (bias.has_value() && bias->defined()) {
    check_bf16_cuda(*bias, "bias");
    TORCH_CHECK(bias->numel() == N && bias->is_contiguous(), "bias must be contiguous [N]");
    a.bias = bias->data_ptr();
  }
  a.epi = (int)epi;
  a.act_lo = (int)act_lo;
  a.act_hi = act_hi < 0 ? (int)N : (int)act_hi;
  if (epi == kEpiGateResid) {
    TORCH_CHECK(gate.has_value() && resid.has_value(), "gate/resid required");
    TORCH_CHECK(gate->scalar_type() == at::kFloat, "gate must be float32");
    TORCH_CHECK(gate->dim() == 2 && gate->stride(1) == 1 && gate->size(1) >= N, "gate must be [B, >=N]");
    check_bf16_cuda(*resid, "resid");
    check_rowmajor(*resid, "resid");
    a.gate = gate->data_ptr<float>();
    a.gate_bstride = gate->stride(0);
    a.resid = resid->data_ptr();
    a.ldr = resid->stride(0);
    a.rows_per_batch = (int)(rows_per_batch > 0 ? rows_per_batch : M);
    if (gate_row_map.has_value() && gate_row_map->defined()) {
      TORCH_CHECK(gate_row_map->scalar_type() == at::kInt && gate_row_map->is_contiguous() &&
                      gate_row_map->numel() == M, "gate_row_map must be int32 [M]");
      a.gate_row_map = gate_row_map->data_ptr<int>();
    }
  }
  a.alpha = (float)alpha;
  a.err = err_ptr();
  return D;
}

at::Tensor gemm(const at::Tensor& A, const at::Tensor& B, const c10::optional<at::Tensor>& bias,
                c10::optional<at::Tensor> out, int64_t epi, int64_t act_lo, int64_t act_hi,
                const c10::optional<at::Tensor>& gate, int64_t rows_per_batch,
                const c10::optional<at::Tensor>& resid, double alpha, bool out_f32,
                std::vector<int64_t> out_peer, int64_t rows_per_rank, int64_t peer_row_off, int64_t ldd_peer,
                const c10::optional<at::Tensor>& gate_row_map, int64_t cta_mode, const std::string& qkv_plan) {
  check_bf16_cuda(A, "A");
  check_bf16_cuda(B, "B");
  check_rowmajor(A, "A");
  check_rowmajor(B, "B");
  TORCH_CHECK(A.size(1) == B.size(1), "K mismatch: A ", A.sizes(), " B ", B.sizes());
  const c10::cuda::CUDAGuard guard(A.device());
  GemmArgs a{};
  at::Tensor D = gemm_epilogue_args(a, A, A.size(0), B.size(0), bias, out, epi, act_lo, act_hi, gate,
                                    rows_per_batch, resid, alpha, out_f32, out_peer, rows_per_rank, peer_row_off,
                                    ldd_peer, gate_row_map, qkv_plan);
  a.A = A.data_ptr();
  a.B = B.data_ptr();
  a.lda = A.stride(0);
  a.ldb = B.stride(0);
  a.K = (int)A.size(1);
  a.cta_mode = (int)cta_mode;
  DFL_CHECK_RC(dfl_gemm_bf16(&a, cur_stream()), "gemm");
  return D;
}

// ---------------------------------------------------------------- MXFP8
std::vector<at::Tensor> mx_quantize(const at::Tensor& x, bool blocked) {
  check_bf16_cuda(x, "x");
  check_rowmajor(x, "x");
  TORCH_CHECK(x.dim() == 2, "x must be [R, K]");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t R = x.size(0), K = x.size(1);
  TORCH_CHECK(K % (blocked ? 128 : 32) == 0, "K must be a multiple of ", blocked ? 128 : 32);
  at::Tensor q = at::empty({R, K}, x.options().dtype(at::kFloat8_e4m3fn));
  // blocked scales: rows padded to 256 (the MXFP8 GEMM reads two 128-row atoms per 256-column B tile)
  at::Tensor sf = blocked ? at::zeros({(R + 255) / 256 * 256 * (K / 32)}, x.options().dtype(at::kByte))
                          : at::empty({R, K / 32}, x.options().dtype(at::kByte));
  DFL_CHECK_RC(dfl_mx_quantize(x.data_ptr(), x.stride(0), (int)R, (int)K, q.data_ptr(), q.stride(0),
                               sf.data_ptr(), blocked ? 1 : 0, cur_stream()),
               "mx_quantize");
  return {q, sf};
}

// Grouped GEMM: problem i is gemm(A[i], B[i], bias[i], out[i], epi, ...); one launch.
std::vector<at::Tensor> gemm_group(std::vector<at::Tensor> A, std::vector<at::Tensor> B,
                                   std::vector<c10::optional<at::Tensor>> bias,
                                   std::vector<c10::optional<at::Tensor>> out, int64_t epi, std::vector<int64_t> act_lo,
                                   std::vector<int64_t> act_hi, std::vector<c10::optional<at::Tensor>> gate,
                                   std::vector<int64_t> rows_per_batch, std::vector<c10::optional<at::Tensor>> resid,
                                   std::vector<std::string> qkv_plan, int64_t cta_mode) {
  const size_t n = A.size();
  TORCH_CHECK(n >= 1 && n <= 2 && B.size() == n && bias.size() == n && out.size() == n && act_lo.size() == n &&
                  act_hi.size() == n && gate.size() == n && rows_per_batch.size() == n && resid.size() == n &&
                  qkv_plan.size() == n,
              "gemm_group: 1 or 2 problems, one entry per problem in every list");
  const c10::cuda::CUDAGuard guard(A[0].device());
  std::vector<GemmArgs> args(n);
  std::vector<at::Tensor> outs;
  for (size_t i = 0; i < n; ++i) {
    check_bf16_cuda(A[i], "A");
    check_bf16_cuda(B[i], "B");
    check_rowmajor(A[i], "A");
    check_rowmajor(B[i], "B");
    TORCH_CHECK(A[i].size(1) == B[i].size(1), "K mismatch in problem ", i);
    TORCH_CHECK(A[i].device() == A[0].device(), "all problems on one device");
    GemmArgs& a = args[i];
    a = GemmArgs{};
    outs.push_back(gemm_epilogue_args(a, A[i], A[i].size(0), B[i].size(0), bias[i], out[i], epi, act_lo[i],
                                      act_hi[i], gate[i], rows_per_batch[i], resid[i], 1.0, false, {}, 0, 0, 0,
                                      c10::nullopt, qkv_plan[i]));
    a.A = A[i].data_ptr();
    a.B = B[i].data_ptr();
    a.lda = A[i].stride(0);
    a.ldb = B[i].stride(0);
    a.K = (int)A[i].size(1);
    a.cta_mode = (int)cta_mode;
  }
  std::vector<const GemmArgs*> ptrs;
  for (auto& a : args) ptrs.push_back(&a);
  DFL_CHECK_RC(dfl_gemm_bf16_group(ptrs.data(), (int)n, cur_stream()), "gemm_group");
  return outs;
}

at::Tensor gemm_mx(const at::Tensor& A, const at::Tensor& sfa, const at::Tensor& B, const at::Tensor& sfb,
                   const c10::optional<at::Tensor>& bias, c10::optional<at::Tensor> out, int64_t epi,
                   int64_t act_lo, int64_t act_hi, const c10::optional<at::Tensor>& gate, int64_t rows_per_batch,
                   const c10::optional<at::Tensor>& resid, double alpha, bool out_f32, std::vector<int64_t> out_peer,
                   int64_t rows_per_rank, int64_t peer_row_off, int64_t ldd_peer,
                   const c10::optional<at::Tensor>& gate_row_map, const std::string& qkv_plan) {
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && A.scalar_type() == at::kFloat8_e4m3fn &&
                  B.scalar_type() == at::kFloat8_e4m3fn, "A and B must be CUDA float8_e4m3fn");
  check_rowmajor(A, "A");
  check_rowmajor(B, "B");
  TORCH_CHECK(A.size(1) == B.size(1), "K mismatch");
  const int64_t M = A.size(0), N = B.size(0), K = A.size(1);
  TORCH_CHECK(sfa.scalar_type() == at::kByte && sfa.is_contiguous() && sfa.numel() >= (M + 127) / 128 * 128 * (K / 32),
              "sfa must be the blocked uint8 scales of A");
  TORCH_CHECK(sfb.scalar_type() == at::kByte && sfb.is_contiguous() &&
                  sfb.numel() >= (N + 255) / 256 * 256 * (K / 32),
              "sfb must be the blocked uint8 scales of B (rows padded to 256)");
  const c10::cuda::CUDAGuard guard(A.device());
  MxGemmArgs m{};
  TORCH_CHECK(epi != kEpiSwiGLU, "the MXFP8 GEMM has no SwiGLU epilogue");
  at::Tensor D = gemm_epilogue_args(m.g, A, M, N, bias, out, epi, act_lo, act_hi, gate, rows_per_batch, resid,
                                    alpha, out_f32, out_peer, rows_per_rank, peer_row_off, ldd_peer, gate_row_map,
                                    qkv_plan);
  m.g.A = A.data_ptr();
  m.g.B = B.data_ptr();
  m.g.lda = A.stride(0);
  m.g.ldb = B.stride(0);
  m.g.K = (int)K;
  m.sfa = sfa.data_ptr();
  m.sfb = sfb.data_ptr();
  DFL_CHECK_RC(dfl_gemm_mx(&m, cur_stream()), "gemm_mx");
  return D;
}

at::Tensor ln_modulate(const at::Tensor& x, c10::optional<at::Tensor> out,
                       const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& b,
                       const c10::optional<at::Tensor>& shift, const c10::optional<at::Tensor>& scale,
                       int64_t rows_per_batch, double eps, bool rms, const c10::optional<at::Tensor>& row_map,
                       std::vector<int64_t> y_peer, int64_t row0, int64_t rows) {
  check_bf16_cuda(x, "x");
  check_rowmajor(x, "x");
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor y = (out.has_value() && out->defined()) ? *out : at::empty_like(x);
  check_rowmajor(y, "out");
  LnModArgs a{};
  TORCH_CHECK(y_peer.size() <= DFL_MAX_PEERS, "at most 8 output peers");
  a.y_world = (int)y_peer.size();
  for (size_t d = 0; d < y_peer.size(); ++d) a.y_peer[d] = reinterpret_cast<void*>(y_peer[d]);
  a.row0 = row0;
  a.x = x.data_ptr();
  a.ldx = x.stride(0);
  a.y = y.data_ptr();
  a.ldy = y.stride(0);
  a.w = opt_ptr(w);
  a.b = opt_ptr(b);
  long long bstride = 0;
  if (shift.has_value() && shift->defined()) {
    TORCH_CHECK(shift->scalar_type() == at::kFloat && shift->dim() == 2 && shift->stride(1) == 1, "shift must be f32 [B, D]");
    a.shift = shift->data_ptr<float>();
    bstride = shift->stride(0);
  }
  if (scale.has_value() && scale->defined()) {
    TORCH_CHECK(scale->scalar_type() == at::kFloat && scale->dim() == 2 && scale->stride(1) == 1, "scale must be f32 [B, D]");
    a.scale = scale->data_ptr<float>();
    TORCH_CHECK(bstride == 0 || bstride == scale->stride(0), "shift/scale batch strides differ");
    bstride = scale->stride(0);
  }
  a.mod_bstride = bstride;
  a.rows_per_batch = (int)(rows_per_batch > 0 ? rows_per_batch : x.size(0));
  a.M = (int)(rows >= 0 ? rows : x.size(0));
  TORCH_CHECK(row0 >= 0 && row0 + a.M <= x.size(0), "row range out of bounds");
  a.D = (int)x.size(1);
  a.eps = (float)eps;
  a.rms = rms ? 1 : 0;
  if (row_map.has_value() && row_map->defined()) {
    TORCH_CHECK(row_map->scalar_type() == at::kInt && row_map->is_contiguous() && row_map->numel() == x.size(0),
                "row_map must be int32 [M]");
    a.row_map = row_map->data_ptr<int>();
  }
  DFL_CHECK_RC(dfl_ln_modulate(&a, cur_stream()), "ln_modulate");
  return y;
}

// Head-scatter description shared by the standalone qkv_scatter kernel and the GEMM
// qkv epilogue (source fields qkv / ld / rows are filled by the caller).
QkvScatterArgs make_qkv_args(int64_t q_off, int64_t k_off, int64_t v_off, int64_t S_src, int64_t H, int64_t dh,
                             int64_t norm_mode, const c10::optional<at::Tensor>& wq,
                             const c10::optional<at::Tensor>& wk, double eps, const c10::optional<at::Tensor>& cos_t,
                             const c10::optional<at::Tensor>& sin_t, int64_t rope_pos_off, bool rope_half,
                             int64_t heads_per_rank, const std::vector<int64_t>& q_dst,
                             const std::vector<int64_t>& k_dst, const std::vector<int64_t>& v_dst, int64_t S_dst,
                             int64_t seq_off, bool out_token_major, bool kv_replicate, int64_t q_S_dst,
                             int64_t q_seq_off, int64_t seg_rows, int64_t seg1_seq_off, int64_t seg1_rope_off, const c10::optional<at::Tensor>& row_sumsq, int64_t norm_total) {
  const int world = (int)q_dst.size();
  TORCH_CHECK(world >= 1 && world <= DFL_MAX_PEERS, "1..8 destinations");
  TORCH_CHECK(k_dst.size() == q_dst.size() && v_dst.size() == q_dst.size(), "dst tables differ");
  QkvScatterArgs a{};
  a.q_off = (int)q_off;
  a.k_off = (int)k_off;
  a.v_off = (int)v_off;
  a.S_src = (int)S_src;
  a.H = (int)H;
  a.dh = (int)dh;
  a.norm_mode = (int)norm_mode;
  a.wq = opt_ptr(wq);
  a.wk = opt_ptr(wk);
  a.eps = (float)eps;
  if (cos_t.has_value() && cos_t->defined()) {
    TORCH_CHECK(cos_t->scalar_type() == at::kFloat && cos_t->is_contiguous(), "cos must be f32 contiguous");
    TORCH_CHECK(sin_t.has_value() && sin_t->scalar_type() == at::kFloat && sin_t->is_contiguous(), "sin must be f32 contiguous");
    const int64_t half = dh / 2, width = cos_t->size(-1);
    TORCH_CHECK(width == H * half || (width <= half && width > 0),
                "RoPE table rows must hold dh/2 (shared), H*dh/2 (per head) or fewer (partial rotary) values");
    a.rope_heads = (width == H * half && H > 1) ? (int)H : 0;
    a.rope_dims = (a.rope_heads == 0 && width < half) ? (int)(2 * width) : 0;
    a.cos_t = cos_t->data_ptr<float>();
    a.sin_t = sin_t->data_ptr<float>();
  }
  a.rope_pos_off = (int)rope_pos_off;
  a.rope_half = rope_half ? 1 : 0;
  a.world = world;
  a.heads_per_rank = (int)heads_per_rank;
  for (int r = 0; r < world; ++r) {
    a.q_dst[r] = reinterpret_cast<void*>(q_dst[r]);
    a.k_dst[r] = reinterpret_cast<void*>(k_dst[r]);
    a.v_dst[r] = reinterpret_cast<void*>(v_dst[r]);
  }
  a.S_dst = (int)S_dst;
  a.seq_off = (int)seq_off;
  a.out_token_major = out_token_major ? 1 : 0;
  a.kv_replicate = kv_replicate ? 1 : 0;
  a.q_S_dst = (int)q_S_dst;
  a.q_seq_off = (int)q_seq_off;
  a.seg_rows = (int)seg_rows;
  a.seg1_seq_off = (int)seg1_seq_off;
  a.seg1_rope_off = (int)seg1_rope_off;
  if (norm_mode == 3) {
    TORCH_CHECK(row_sumsq.has_value() && row_sumsq->defined() && row_sumsq->scalar_type() == at::kFloat &&
                    row_sumsq->is_contiguous(), "norm_mode 3 needs row_sumsq (f32 [rows, 2], contiguous)");
    a.row_sumsq = row_sumsq->data_ptr<float>();
    a.norm_total = (int)norm_total;
  }
  return a;
}

void qkv_scatter(const at::Tensor& qkv, int64_t q_off, int64_t k_off, int64_t v_off, int64_t S_src,
                 int64_t H, int64_t dh, int64_t norm_mode, const c10::optional<at::Tensor>& wq,
                 const c10::optional<at::Tensor>& wk, double eps,
                 const c10::optional<at::Tensor>& cos_t, const c10::optional<at::Tensor>& sin_t,
                 int64_t rope_pos_off, bool rope_half, int64_t heads_per_rank,
                 std::vector<int64_t> q_dst, std::vector<int64_t> k_dst, std::vector<int64_t> v_dst,
                 int64_t S_dst, int64_t seq_off, bool out_token_major, bool kv_replicate, int64_t q_S_dst,
                 int64_t q_seq_off, int64_t seg_rows, int64_t seg1_seq_off, int64_t seg1_rope_off, const c10::optional<at::Tensor>& row_sumsq, int64_t norm_total) {
  check_bf16_cuda(qkv, "qkv");
  check_rowmajor(qkv, "qkv");
  const c10::cuda::CUDAGuard guard(qkv.device());
  QkvScatterArgs a = make_qkv_args(q_off, k_off, v_off, S_src, H, dh, norm_mode, wq, wk, eps, cos_t, sin_t,
                                   rope_pos_off, rope_half, heads_per_rank, q_dst, k_dst, v_dst, S_dst, seq_off,
                                   out_token_major, kv_replicate, q_S_dst, q_seq_off, seg_rows, seg1_seq_off,
                                   seg1_rope_off, row_sumsq, norm_total);
  a.qkv = qkv.data_ptr();
  a.ld = qkv.stride(0);
  a.rows = (int)qkv.size(0);
  DFL_CHECK_RC(dfl_qkv_scatter(&a, cur_stream()), "qkv_scatter");
}

at::Tensor row_sumsq(const at::Tensor& x, int64_t off0, int64_t off1, int64_t width) {
  check_bf16_cuda(x, "x");
  check_rowmajor(x, "x");
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor out = at::empty({x.size(0), 2}, x.options().dtype(at::kFloat));
  DFL_CHECK_RC(dfl_row_sumsq(x.data_ptr(), x.stride(0), (int)x.size(0), (int)off0, (int)off1, (int)width,
                             out.data_ptr<float>(), cur_stream()),
               "row_sumsq");
  return out;
}

// The same description packed for the GEMM's qkv epilogue (epi = 5, argument qkv_plan).
py::bytes qkv_plan(int64_t q_off, int64_t k_off, int64_t v_off, int64_t S_src, int64_t H, int64_t dh,
                   int64_t norm_mode, const c10::optional<at::Tensor>& wq, const c10::optional<at::Tensor>& wk,
                   double eps, const c10::optional<at::Tensor>& cos_t, const c10::optional<at::Tensor>& sin_t,
                   int64_t rope_pos_off, bool rope_half, int64_t heads_per_rank, std::vector<int64_t> q_dst,
                   std::vector<int64_t> k_dst, std::vector<int64_t> v_dst, int64_t S_dst, int64_t seq_off,
                   bool out_token_major, bool kv_replicate, int64_t q_S_dst, int64_t q_seq_off, int64_t seg_rows, int64_t seg1_seq_off, int64_t seg1_rope_off, const c10::optional<at::Tensor>& row_sumsq, int64_t norm_total) {
  QkvScatterArgs a = make_qkv_args(q_off, k_off, v_off, S_src, H, dh, norm_mode, wq, wk, eps, cos_t, sin_t,
                                   rope_pos_off, rope_half, heads_per_rank, q_dst, k_dst, v_dst, S_dst, seq_off,
                                   out_token_major, kv_replicate, q_S_dst, q_seq_off, seg_rows, seg1_seq_off,
                                   seg1_rope_off, row_sumsq, norm_total);
  return py::bytes(reinterpret_cast<const char*>(&a), sizeof(a));
}

at::Tensor gemv(const at::Tensor& W, const at::Tensor& x, const c10::optional<at::Tensor>& bias,
                c10::optional<at::Tensor> out, bool silu_in, bool silu_out) {
  check_bf16_cuda(W, "W");
  check_rowmajor(W, "W");
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.dim() == 2 && x.is_contiguous(), "x must be f32 [B, K]");
  TORCH_CHECK(x.size(1) == W.size(1), "K mismatch");
  const c10::cuda::CUDAGuard guard(W.device());
  at::Tensor y = (out.has_value() && out->defined()) ? *out
                                                     : at::empty({x.size(0), W.size(0)}, x.options());
  TORCH_CHECK(y.scalar_type() == at::kFloat && y.dim() == 2 && y.stride(1) == 1, "out must be f32 [B, N]");
  GemvArgs a{};
  a.W = W.data_ptr();
  a.ldw = W.stride(0);
  a.x = x.data_ptr<float>();
  a.batch = (int)x.size(0);
  a.bias = opt_ptr(bias);
  a.y = y.data_ptr<float>();
  a.ldy = y.stride(0);
  a.N = (int)W.size(0);
  a.K = (int)W.size(1);
  a.silu_in = silu_in ? 1 : 0;
  a.silu_out = silu_out ? 1 : 0;
  DFL_CHECK_RC(dfl_gemv(&a, cur_stream()), "gemv");
  return y;
}

void euler_step(at::Tensor x32, const c10::optional<at::Tensor>& x16, const at::Tensor& v,
                const c10::optional<at::Tensor>& cond, double dt, double guidance) {
  TORCH_CHECK(x32.scalar_type() == at::kFloat && x32.is_contiguous(), "x32 must be f32 contiguous");
  check_bf16_cuda(v, "v");
  TORCH_CHECK(v.is_contiguous() && v.numel() == x32.numel(), "v must match x32");
  const c10::cuda::CUDAGuard guard(x32.device());
  SchedArgs a{};
  a.x32 = x32.data_ptr<float>();
  a.x16 = nullptr;
  if (x16.has_value() && x16->defined()) {
    check_bf16_cuda(*x16, "x16");
    TORCH_CHECK(x16->is_contiguous() && x16->numel() == x32.numel(), "x16 must match x32");
    a.x16 = x16->data_ptr();
  }
  a.v = v.data_ptr();
  a.cond = nullptr;
  if (cond.has_value() && cond->defined()) {
    check_bf16_cuda(*cond, "cond");
    TORCH_CHECK(cond->is_contiguous() && cond->numel() == x32.numel(), "cond must match x32");
    a.cond = cond->data_ptr();
  }
  a.n = x32.numel();
  a.dt = (float)dt;
  a.guidance = (float)guidance;
  DFL_CHECK_RC(dfl_euler_step(&a, cur_stream()), "euler_step");
}

// Guidance + sampler update (see kernels.h GuidedStepArgs).  b_ptr: the other branch's prediction
// (0 = none) as a raw device pointer, so it may be a peer rank's buffer; coeffs = (k_v, e[5], g[6]).
void guided_step(const at::Tensor& a, int64_t b_ptr, double scale, at::Tensor x, const c10::optional<at::Tensor>& x16,
                 const c10::optional<at::Tensor>& last, const c10::optional<at::Tensor>& m1,
                 const c10::optional<at::Tensor>& m2, const c10::optional<at::Tensor>& m_out,
                 std::vector<double> coeffs, bool store_last, bool swap_ab) {
  check_bf16_cuda(a, "a");
  TORCH_CHECK(a.is_contiguous(), "a must be contiguous");
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous() && x.numel() == a.numel(), "x must be f32 like a");
  TORCH_CHECK(coeffs.size() == 12, "coeffs: k_v, e[5] (x, last, m1, m2, m), g[6] (x, last, m1, m2, m, v)");
  auto f32 = [&](const c10::optional<at::Tensor>& t, const char* name) -> float* {
    if (!(t.has_value() && t->defined())) return nullptr;
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == x.numel(), name,
                " must be f32 contiguous like x");
    return t->data_ptr<float>();
  };
  const c10::cuda::CUDAGuard guard(x.device());
  GuidedStepArgs g{};
  g.a = a.data_ptr();
  g.b = reinterpret_cast<const void*>(b_ptr);
  g.scale = (float)scale;
  g.x = x.data_ptr<float>();
  if (x16.has_value() && x16->defined()) {
    check_bf16_cuda(*x16, "x16");
    TORCH_CHECK(x16->is_contiguous() && x16->numel() == x.numel(), "x16 must match x");
    g.x16 = x16->data_ptr();
  }
  g.last = f32(last, "last");
  g.m1 = f32(m1, "m1");
  g.m2 = f32(m2, "m2");
  g.m_out = f32(m_out, "m_out");
  g.n = x.numel();
  g.k_v = (float)coeffs[0];
  for (int t = 0; t < 5; ++t) g.e[t] = (float)coeffs[1 + t];
  for (int t = 0; t < 6; ++t) g.g[t] = (float)coeffs[6 + t];
  g.store_last = store_last ? 1 : 0;
  g.swap_ab = swap_ab ? 1 : 0;
  DFL_CHECK_RC(dfl_guided_step(&g, cur_stream()), "guided_step");
}

at::Tensor timestep_embed(const at::Tensor& t, int64_t dim, double max_period, bool flip_sin_to_cos,
                          double downscale_freq_shift, double scale) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.dim() == 1 && t.is_contiguous(), "t must be f32 [B]");
  const c10::cuda::CUDAGuard guard(t.device());
  at::Tensor out = at::empty({t.size(0), dim}, t.options());
  int rc = dfl_timestep_embed(t.data_ptr<float>(), (int)t.size(0), (int)dim, (float)max_period,
                              flip_sin_to_cos ? 1 : 0, (float)downscale_freq_shift, (float)scale,
                              out.data_ptr<float>(), cur_stream());
  DFL_CHECK_RC(rc, "timestep_embed");
  return out;
}

// q, k, v: [B, H, S, dh] views (any strides with unit inner stride).
at::Tensor attention(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double scale,
                     c10::optional<at::Tensor> out, const c10::optional<at::Tensor>& lse,
                     const c10::optional<at::Tensor>& kv_lo, const c10::optional<at::Tensor>& kv_hi,
                     std::vector<int64_t> o_peer, int64_t seg0_len, int64_t seg0_per, int64_t seg1_per, std::vector<int64_t> o_strides,
                     const c10::optional<at::Tensor>& acc_o, const c10::optional<at::Tensor>& acc_lse, int64_t merge_mode,
                     int64_t kv_split) {
  check_bf16_cuda(q, "q");
  check_bf16_cuda(k, "k");
  check_bf16_cuda(v, "v");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "q/k/v must be [B, H, S, dh]");
  TORCH_CHECK(q.stride(3) == 1 && k.stride(3) == 1 && v.stride(3) == 1, "unit inner stride required");
  const c10::cuda::CUDAGuard guard(q.device());
  const bool scatter = !o_peer.empty();
  const bool no_out = scatter || merge_mode == 1 || merge_mode == 2;  // partials write only acc_o / acc_lse
  at::Tensor o = (out.has_value() && out->defined()) ? *out : (no_out ? at::empty({0}, q.options()) : at::empty_like(q));
  TORCH_CHECK(no_out || (o.dim() == 4 && o.stride(3) == 1), "out must be [B, H, S, dh] with unit inner stride");
  TORCH_CHECK(!scatter || o_strides.size() == 3, "o_strides (batch, head, seq) required with o_peer");
  AttnArgs a{};
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.o = o.data_ptr();
  a.q_bs = q.stride(0); a.q_hs = q.stride(1); a.q_ss = q.stride(2);
  a.k_bs = k.stride(0); a.k_hs = k.stride(1); a.k_ss = k.stride(2);
  a.v_bs = v.stride(0); a.v_hs = v.stride(1); a.v_ss = v.stride(2);
  if (scatter) {
    a.o_bs = o_strides[0]; a.o_hs = o_strides[1]; a.o_ss = o_strides[2];
    a.o = reinterpret_cast<void*>(o_peer[0]);
  } else if (o.dim() != 4) {
    a.o_bs = a.o_hs = a.o_ss = 0;
  } else {
    a.o_bs = o.stride(0); a.o_hs = o.stride(1); a.o_ss = o.stride(2);
  }
  a.B = (int)q.size(0);
  a.H = (int)q.size(1);
  a.Sq = (int)q.size(2);
  a.Sk = (int)k.size(2);
  a.dh = (int)q.size(3);
  a.scale = (float)scale;
  if (lse.has_value() && lse->defined()) {
    TORCH_CHECK(lse->scalar_type() == at::kFloat && lse->is_contiguous(), "lse must be f32 [B, H, Sq]");
    a.lse = lse->data_ptr<float>();
  }
  if (kv_lo.has_value() && kv_lo->defined()) a.kv_lo = kv_lo->data_ptr<int>();
  if (kv_hi.has_value() && kv_hi->defined()) a.kv_hi = kv_hi->data_ptr<int>();
  a.err = err_ptr();
  TORCH_CHECK(o_peer.size() <= DFL_MAX_PEERS, "at most 8 output peers");
  a.o_world = (int)o_peer.size();
  for (size_t r = 0; r < o_peer.size(); ++r) a.o_peer[r] = reinterpret_cast<void*>(o_peer[r]);
  a.seg0_len = (int)seg0_len;
  a.seg0_per = (int)seg0_per;
  a.seg1_per = (int)seg1_per;
  a.merge_mode = (int)merge_mode;
  if (merge_mode != 0) {
    TORCH_CHECK(acc_o.has_value() && acc_lse.has_value(), "merge needs acc_o and acc_lse");
    TORCH_CHECK(acc_o->scalar_type() == at::kFloat && acc_o->is_contiguous() &&
                    acc_o->numel() == (int64_t)a.B * a.H * a.Sq * 128, "acc_o must be f32 [B, H, Sq, 128]");
    TORCH_CHECK(acc_lse->scalar_type() == at::kFloat && acc_lse->is_contiguous() &&
                    acc_lse->numel() == (int64_t)a.B * a.H * a.Sq, "acc_lse must be f32 [B, H, Sq]");
    a.acc_o = acc_o->data_ptr<float>();
    a.acc_lse = acc_lse->data_ptr<float>();
  }
  // split-KV partial buffers (stream-ordered allocations, released after the launch)
  at::Tensor split_o, split_lse;
  const int splits = kv_split < 0 ? dfl_attention_plan_splits(&a) : (int)std::max<int64_t>(kv_split, 1);
  if (splits > 1 && merge_mode == 0) {
    const int64_t rows = (int64_t)a.B * a.H * a.Sq;
    split_o = at::empty({splits, rows, 128}, q.options().dtype(at::kFloat));
    split_lse = at::empty({splits, rows}, q.options().dtype(at::kFloat));
    a.kv_splits = splits;
    a.split_o = split_o.data_ptr<float>();
    a.split_lse = split_lse.data_ptr<float>();
  }
  DFL_CHECK_RC(dfl_attention(&a, cur_stream()), "attention");
  return o;
}

at::Tensor error_word(int64_t device) { return error_buffer((int)device); }

// ---------------------------------------------------------------- comm runtime
at::Tensor symm_alloc(int64_t nbytes, int64_t device) {
  const c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)nbytes);
  TORCH_CHECK(e == cudaSuccess, "cudaMalloc(", nbytes, ") failed: ", cudaGetErrorString(e));
  cudaMemset(p, 0, (size_t)nbytes);
  cudaDeviceSynchronize();
  return torch::from_blob(p, {nbytes}, [](void* ptr) { cudaFree(ptr); },
                          at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device));
}

at::Tensor from_ptr(int64_t ptr, int64_t nbytes, int64_t device) {
  return torch::from_blob(reinterpret_cast<void*>(ptr), {nbytes}, [](void*) {},
                          at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device));
}

py::bytes ipc_handle(const at::Tensor& t) {
  char buf[64];
  int rc = dfl_ipc_handle(t.data_ptr(), buf);
  TORCH_CHECK(rc == 0, "cudaIpcGetMemHandle failed: ", rc);
  return py::bytes(buf, 64);
}

int64_t ipc_open(py::bytes handle, int64_t device) {
  const c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
  std::string h = handle;
  TORCH_CHECK(h.size() == 64, "IPC handle must be 64 bytes");
  void* p = nullptr;
  int rc = dfl_ipc_open(h.data(), &p);
  TORCH_CHECK(rc == 0, "cudaIpcOpenMemHandle failed: ", rc);
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) { dfl_ipc_close(reinterpret_cast<void*>(ptr)); }

void tp_reduce(const at::Tensor& slots, int64_t slot_rows, int64_t world, int64_t rows, int64_t N, int64_t row0,
               const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& gate, int64_t rows_per_batch,
               const c10::optional<at::Tensor>& resid, std::vector<int64_t> out, int64_t ldo, int64_t out_row0,
               int64_t resid_row0) {
  TORCH_CHECK(slots.is_cuda() && slots.scalar_type() == at::kBFloat16, "slots must be CUDA bf16");
  TORCH_CHECK(slots.numel() >= world * slot_rows * N, "slots too small");
  TORCH_CHECK(!out.empty() && out.size() <= DFL_MAX_PEERS, "1..8 output pointers");
  const c10::cuda::CUDAGuard guard(slots.device());
  TpReduceArgs a{};
  a.slots = slots.data_ptr();
  a.slot_rows = slot_rows;
  a.world = (int)world;
  a.rows = (int)rows;
  a.N = (int)N;
  a.row0 = row0;
  if (bias.has_value() && bias->defined()) {
    check_bf16_cuda(*bias, "bias");
    a.bias = bias->data_ptr();
  }
  if (gate.has_value() && gate->defined()) {
    TORCH_CHECK(gate->scalar_type() == at::kFloat && gate->stride(1) == 1, "gate must be f32 [B, >=N]");
    TORCH_CHECK(resid.has_value() && resid->defined(), "gate needs resid");
    check_bf16_cuda(*resid, "resid");
    check_rowmajor(*resid, "resid");
    a.gate = gate->data_ptr<float>();
    a.gate_bstride = gate->stride(0);
    a.rows_per_batch = (int)rows_per_batch;
    a.resid = resid->data_ptr();
    a.ldr = resid->stride(0);
    a.resid_row0 = resid_row0;
  }
  a.out_world = (int)out.size();
  for (size_t d = 0; d < out.size(); ++d) a.out[d] = reinterpret_cast<void*>(out[d]);
  a.ldo = ldo;
  a.out_row0 = out_row0;
  DFL_CHECK_RC(dfl_tp_reduce(&a, cur_stream()), "tp_reduce");
}

at::Tensor conv3d(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& bias, int64_t kt,
                  int64_t kh, int64_t kw, bool causal, const c10::optional<at::Tensor>& resid, bool silu,
                  c10::optional<at::Tensor> out, bool valid_t, bool valid_h, bool valid_w) {
  check_bf16_cuda(x, "x");
  check_bf16_cuda(w, "w");
  TORCH_CHECK(x.dim() == 5 && x.is_contiguous(), "x must be contiguous [N, T, H, W, Ci]");
  TORCH_CHECK(w.dim() == 2 && w.is_contiguous() && w.size(1) == kt * kh * kw * x.size(4), "w must be [Co, taps*Ci]");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t Co = w.size(0);
  const int64_t To = valid_t ? x.size(1) - kt + 1 : x.size(1), Ho = valid_h ? x.size(2) - kh + 1 : x.size(2);
  const int64_t Wo = valid_w ? x.size(3) - kw + 1 : x.size(3);
  TORCH_CHECK(To > 0 && Ho > 0 && Wo > 0, "valid convolution of fewer frames / rows / columns than its kernel");
  at::Tensor y = (out.has_value() && out->defined()) ? *out : at::empty({x.size(0), To, Ho, Wo, Co}, x.options());
  TORCH_CHECK(y.is_contiguous() && y.numel() == x.size(0) * To * Ho * Wo * Co,
              "out must be contiguous [N, T_out, H_out, W_out, Co]");
  ConvArgs a{};
  a.x = x.data_ptr();
  a.w = w.data_ptr();
  a.y = y.data_ptr();
  at::Tensor ones;
  if (bias.has_value() && bias->defined()) {
    check_bf16_cuda(*bias, "bias");
    a.bias = bias->data_ptr();
  }
  if (resid.has_value() && resid->defined()) {
    check_bf16_cuda(*resid, "resid");
    TORCH_CHECK(resid->is_contiguous() && resid->numel() == y.numel(), "resid must match out");
    a.resid = resid->data_ptr();
    ones = at::ones({Co}, x.options().dtype(at::kFloat));
    a.ones = ones.data_ptr<float>();
  }
  a.N = (int)x.size(0), a.T = (int)x.size(1), a.H = (int)x.size(2), a.W = (int)x.size(3), a.Ci = (int)x.size(4);
  a.Co = (int)Co;
  a.kt = (int)kt, a.kh = (int)kh, a.kw = (int)kw, a.causal = causal ? 1 : 0, a.silu = silu ? 1 : 0;
  a.valid_t = valid_t ? 1 : 0, a.valid_h = valid_h ? 1 : 0, a.valid_w = valid_w ? 1 : 0;
  a.err = err_ptr();
  DFL_CHECK_RC(dfl_conv3d(&a, cur_stream()), "conv3d");
  return y;
}

// HunyuanVideo-style VAE helpers (vae_gn.cu): channels-last [N, T, H, W, C] bf16 volumes.
at::Tensor gn_stats(const at::Tensor& x, int64_t G, double eps) {
  check_bf16_cuda(x, "x");
  TORCH_CHECK(x.dim() == 5 && x.is_contiguous(), "x must be contiguous [N, T, H, W, C]");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t N = x.size(0), C = x.size(4), P = x.size(1) * x.size(2) * x.size(3);
  int dev = x.device().index();
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int nblk = (int)std::max<int64_t>(1, std::min<int64_t>((int64_t)sms * 4 / std::max<int64_t>(N, 1), P / 64));
  at::Tensor partial = at::empty({nblk, N, G}, x.options().dtype(at::kFloat));
  at::Tensor stats = at::empty({N, G, 2}, x.options().dtype(at::kFloat));
  DFL_CHECK_RC(dfl_gn_stats(x.data_ptr(), (int)N, P, (int)C, (int)G, (float)eps, partial.data_ptr<float>(), nblk,
                            stats.data_ptr<float>(), cur_stream()),
               "gn_stats");
  return stats;
}

void gn_apply(const at::Tensor& x, const at::Tensor& stats, const at::Tensor& gamma, const at::Tensor& beta,
              int64_t G, bool silu, at::Tensor y, int64_t ot, int64_t oh, int64_t ow) {
  check_bf16_cuda(x, "x");
  check_bf16_cuda(y, "y");
  TORCH_CHECK(x.dim() == 5 && x.is_contiguous() && y.dim() == 5 && y.is_contiguous(), "x, y contiguous 5-D");
  TORCH_CHECK(y.size(0) == x.size(0) && y.size(4) == x.size(4), "y must match x in N and C");
  TORCH_CHECK(stats.scalar_type() == at::kFloat && stats.is_contiguous() && stats.numel() == x.size(0) * G * 2,
              "stats f32 [N, G, 2]");
  TORCH_CHECK(gamma.scalar_type() == at::kFloat && beta.scalar_type() == at::kFloat && gamma.is_contiguous() &&
                  beta.is_contiguous() && gamma.numel() == x.size(4) && beta.numel() == x.size(4),
              "gamma / beta f32 [C]");
  const c10::cuda::CUDAGuard guard(x.device());
  GnApplyArgs a{};
  a.x = x.data_ptr(), a.y = y.data_ptr(), a.stats = stats.data_ptr<float>();
  a.gamma = gamma.data_ptr<float>(), a.beta = beta.data_ptr<float>();
  a.N = (int)x.size(0), a.T = (int)x.size(1), a.H = (int)x.size(2), a.W = (int)x.size(3), a.C = (int)x.size(4);
  a.G = (int)G;
  a.Ty = (int)y.size(1), a.Hy = (int)y.size(2), a.Wy = (int)y.size(3);
  a.ot = (int)ot, a.oh = (int)oh, a.ow = (int)ow, a.silu = silu ? 1 : 0;
  DFL_CHECK_RC(dfl_gn_apply(&a, cur_stream()), "gn_apply");
}

void pad_replicate(at::Tensor y, int64_t pt, int64_t ph, int64_t pw, int64_t T, int64_t H, int64_t W) {
  check_bf16_cuda(y, "y");
  TORCH_CHECK(y.dim() == 5 && y.is_contiguous(), "y must be contiguous [N, Ty, Hy, Wy, C]");
  const c10::cuda::CUDAGuard guard(y.device());
  PadArgs a{};
  a.y = y.data_ptr();
  a.N = (int)y.size(0), a.Ty = (int)y.size(1), a.Hy = (int)y.size(2), a.Wy = (int)y.size(3), a.C = (int)y.size(4);
  a.pt = (int)pt, a.ph = (int)ph, a.pw = (int)pw, a.T = (int)T, a.H = (int)H, a.W = (int)W;
  DFL_CHECK_RC(dfl_pad_replicate(&a, cur_stream()), "pad_replicate");
}

void upsample_causal(const at::Tensor& x, bool up_t, at::Tensor y, int64_t ot, int64_t oh, int64_t ow) {
  check_bf16_cuda(x, "x");
  check_bf16_cuda(y, "y");
  TORCH_CHECK(x.dim() == 5 && x.is_contiguous() && y.dim() == 5 && y.is_contiguous(), "x, y contiguous 5-D");
  TORCH_CHECK(y.size(0) == x.size(0) && y.size(4) == x.size(4), "y must match x in N and C");
  const c10::cuda::CUDAGuard guard(x.device());
  UpsampleArgs a{};
  a.x = x.data_ptr(), a.y = y.data_ptr();
  a.N = (int)x.size(0), a.T = (int)x.size(1), a.H = (int)x.size(2), a.W = (int)x.size(3), a.C = (int)x.size(4);
  a.up_t = up_t ? 1 : 0;
  a.Ty = (int)y.size(1), a.Hy = (int)y.size(2), a.Wy = (int)y.size(3);
  a.ot = (int)ot, a.oh = (int)oh, a.ow = (int)ow;
  DFL_CHECK_RC(dfl_upsample_causal(&a, cur_stream()), "upsample_causal");
}

// VAE slab helpers: x [F, Hl, W, C]; y [F, Ho + 2 halo, Wo, C]; up / down = peer pointers (0: none).
static VaeRowArgs vae_args(const at::Tensor& x, const at::Tensor& y, int64_t Ho, int64_t Wo, bool halo, int64_t up,
                           int64_t up_rows, int64_t down, int64_t down_rows) {
  check_bf16_cuda(x, "x");
  check_bf16_cuda(y, "y");
  TORCH_CHECK(x.dim() == 4 && x.is_contiguous() && y.dim() == 4 && y.is_contiguous(), "x / y: contiguous [F, H, W, C]");
  TORCH_CHECK(y.size(0) == x.size(0) && y.size(3) == x.size(3) && y.size(1) == Ho + (halo ? 2 : 0) && y.size(2) == Wo,
              "y must be [F, Ho + 2 halo, Wo, C]");
  VaeRowArgs a{};
  a.x = x.data_ptr();
  a.y = y.data_ptr();
  a.F = (int)x.size(0), a.Ho = (int)Ho, a.Wo = (int)Wo, a.C = (int)x.size(3);
  a.halo = halo ? 1 : 0;
  a.up = reinterpret_cast<void*>(up);
  a.up_rows = (int)up_rows;
  a.down = reinterpret_cast<void*>(down);
  a.down_rows = (int)down_rows;
  return a;
}

void vae_chan_norm(const at::Tensor& x, const at::Tensor& gamma, at::Tensor y, bool silu, bool halo, int64_t up,
                   int64_t up_rows, int64_t down, int64_t down_rows) {
  check_bf16_cuda(gamma, "gamma");
  TORCH_CHECK(gamma.is_contiguous() && gamma.numel() == x.size(3), "gamma must be [C]");
  const c10::cuda::CUDAGuard guard(x.device());
  VaeRowArgs a = vae_args(x, y, x.size(1), x.size(2), halo, up, up_rows, down, down_rows);
  a.gamma = gamma.data_ptr();
  a.silu = silu ? 1 : 0;
  DFL_CHECK_RC(dfl_vae_chan_norm(&a, cur_stream()), "vae_chan_norm");
}

void vae_upsample2x(const at::Tensor& x, at::Tensor y, bool halo, int64_t up, int64_t up_rows, int64_t down,
                    int64_t down_rows) {
  const c10::cuda::CUDAGuard guard(x.device());
  VaeRowArgs a = vae_args(x, y, 2 * x.size(1), 2 * x.size(2), halo, up, up_rows, down, down_rows);
  DFL_CHECK_RC(dfl_vae_upsample2x(&a, cur_stream()), "vae_upsample2x");
}

void memcpy_async(int64_t dst, int64_t src, int64_t nbytes) {
  DFL_CHECK_RC(dfl_memcpy_async(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), nbytes,
                                cur_stream()),
               "memcpy_async");
}

void peer_barrier(std::vector<int64_t> flags, const at::Tensor& counter, int64_t rank, int64_t timeout_cycles) {
  TORCH_CHECK(counter.is_cuda() && counter.scalar_type() == at::kInt, "counter must be a CUDA int32 tensor");
  const c10::cuda::CUDAGuard guard(counter.device());
  BarrierArgs a{};
  a.world = (int)flags.size();
  for (size_t r = 0; r < flags.size(); ++r) a.flags[r] = reinterpret_cast<int*>(flags[r]);
  a.counter = counter.data_ptr<int>();
  a.rank = (int)rank;
  a.timeout_cycles = timeout_cycles;
  a.err = err_ptr();
  DFL_CHECK_RC(dfl_peer_barrier(&a, cur_stream()), "peer_barrier");
}

void peer_put_f32(const at::Tensor& src, std::vector<int64_t> dst, int64_t dst_offset) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == at::kFloat && src.is_contiguous(), "src must be f32 contiguous");
  const c10::cuda::CUDAGuard guard(src.device());
  PeerPutArgs a{};
  a.src = src.data_ptr<float>();
  a.n = src.numel();
  a.world = (int)dst.size();
  for (size_t r = 0; r < dst.size(); ++r) a.dst[r] = reinterpret_cast<float*>(dst[r]);
  a.dst_offset = dst_offset;
  DFL_CHECK_RC(dfl_peer_put_f32(&a, cur_stream()), "peer_put_f32");
}

void cfg_combine(const at::Tensor& mine, int64_t peer_ptr, at::Tensor out, double scale, bool mine_is_cond) {
  check_bf16_cuda(mine, "mine");
  TORCH_CHECK(mine.is_contiguous() && out.is_contiguous() && out.scalar_type() == at::kFloat &&
                  out.numel() == mine.numel(), "mine (bf16) / out (f32) must be contiguous and equal in size");
  const c10::cuda::CUDAGuard guard(mine.device());
  DFL_CHECK_RC(dfl_cfg_combine(mine.data_ptr(), reinterpret_cast<const void*>(peer_ptr), out.data_ptr<float>(),
                               mine.numel(), (float)scale, mine_is_cond ? 1 : 0, cur_stream()),
               "cfg_combine");
}

// TeaCache probe.  Scratch comes from torch's caching allocator, one buffer per
// device, kept (and left ready) between calls.
at::Tensor rel_l1(const at::Tensor& a, const at::Tensor& b) {
  check_bf16_cuda(a, "a");
  check_bf16_cuda(b, "b");
  TORCH_CHECK(a.is_contiguous() && b.is_contiguous() && a.numel() == b.numel(), "a / b must match");
  const c10::cuda::CUDAGuard guard(a.device());
  static at::Tensor scratch[16];
  int dev = c10::cuda::current_device();
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int blocks = dfl_rel_l1_blocks(a.numel(), sms);
  const long long need = dfl_rel_l1_scratch_floats(blocks);
  if (!scratch[dev].defined() || scratch[dev].numel() < need)
    scratch[dev] = at::zeros({need}, a.options().dtype(at::kFloat));
  at::Tensor out = at::empty({1}, a.options().dtype(at::kFloat));
  DFL_CHECK_RC(dfl_rel_l1(a.data_ptr(), b.data_ptr(), a.numel(), scratch[dev].data_ptr<float>(), blocks,
                          out.data_ptr<float>(), cur_stream()),
               "rel_l1");
  return out;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "difflet_b200 native sm_100a kernels";
  m.def("gemm_set_pair_auto", [](bool on) { dfl_gemm_set_pair_auto(on ? 1 : 0); });
  m.def("gemm_set_split_force", [](int64_t s) { dfl_gemm_set_split_force((int)s); });
  m.def("gemm_set_epi_warps", [](int64_t n) { dfl_gemm_set_epi_warps((int)n); });
  m.def("gemm_set_split_workspace", [](const at::Tensor& ws, const at::Tensor& sem) {
    TORCH_CHECK(ws.is_cuda() && sem.is_cuda() && ws.device() == sem.device(), "workspace tensors on one device");
    TORCH_CHECK(ws.scalar_type() == at::kFloat && sem.scalar_type() == at::kInt && ws.is_contiguous() &&
                    sem.is_contiguous(), "ws f32, sem int32, contiguous");
    dfl_gemm_set_split_workspace((int)ws.device().index(), ws.data_ptr(), ws.numel() * 4, sem.data_ptr(),
                                 (int)sem.numel());
  });
  m.def("gemm", &gemm, "tcgen05 GEMM with fused epilogue", py::arg("A"), py::arg("B"),
        py::arg("bias") = py::none(), py::arg("out") = py::none(), py::arg("epi") = 0,
        py::arg("act_lo") = 0, py::arg("act_hi") = -1, py::arg("gate") = py::none(),
        py::arg("rows_per_batch") = 0, py::arg("resid") = py::none(), py::arg("alpha") = 1.0,
        py::arg("out_f32") = false, py::arg("out_peer") = std::vector<int64_t>{}, py::arg("rows_per_rank") = 0,
        py::arg("peer_row_off") = 0, py::arg("ldd") = 0, py::arg("gate_row_map") = py::none(),
        py::arg("cta_mode") = 0, py::arg("qkv_plan") = py::bytes());
  m.def("gemm_group", &gemm_group, "grouped tcgen05 GEMMs (one launch)", py::arg("A"), py::arg("B"),
        py::arg("bias"), py::arg("out"), py::arg("epi"), py::arg("act_lo"), py::arg("act_hi"), py::arg("gate"),
        py::arg("rows_per_batch"), py::arg("resid"), py::arg("qkv_plan"), py::arg("cta_mode") = 0);
  m.def("mx_quantize", &mx_quantize, py::arg("x"), py::arg("blocked") = false);
  m.def("gemm_mx", &gemm_mx, "block-scaled MXFP8 tcgen05 GEMM", py::arg("A"), py::arg("sfa"), py::arg("B"),
        py::arg("sfb"), py::arg("bias") = py::none(), py::arg("out") = py::none(), py::arg("epi") = 0,
        py::arg("act_lo") = 0, py::arg("act_hi") = -1, py::arg("gate") = py::none(),
        py::arg("rows_per_batch") = 0, py::arg("resid") = py::none(), py::arg("alpha") = 1.0,
        py::arg("out_f32") = false, py::arg("out_peer") = std::vector<int64_t>{}, py::arg("rows_per_rank") = 0,
        py::arg("peer_row_off") = 0, py::arg("ldd") = 0, py::arg("gate_row_map") = py::none(),
        py::arg("qkv_plan") = py::bytes());
  m.def("ln_modulate", &ln_modulate, py::arg("x"), py::arg("out") = py::none(),
        py::arg("w") = py::none(), py::arg("b") = py::none(), py::arg("shift") = py::none(),
        py::arg("scale") = py::none(), py::arg("rows_per_batch") = 0, py::arg("eps") = 1e-6,
        py::arg("rms") = false, py::arg("row_map") = py::none(), py::arg("y_peer") = std::vector<int64_t>{},
        py::arg("row0") = 0, py::arg("rows") = -1);
  m.def("qkv_scatter", &qkv_scatter);
  m.def("qkv_plan", &qkv_plan);
  m.def("row_sumsq", &row_sumsq);
  m.def("gemv", &gemv, py::arg("W"), py::arg("x"), py::arg("bias") = py::none(),
        py::arg("out") = py::none(), py::arg("silu_in") = false, py::arg("silu_out") = false);
  m.def("euler_step", &euler_step, py::arg("x32"), py::arg("x16"), py::arg("v"),
        py::arg("cond") = py::none(), py::arg("dt") = 0.0, py::arg("guidance") = 1.0);
  m.def("timestep_embed", &timestep_embed);
  m.def("attention", &attention, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("scale"),
        py::arg("out") = py::none(), py::arg("lse") = py::none(), py::arg("kv_lo") = py::none(),
        py::arg("kv_hi") = py::none(), py::arg("o_peer") = std::vector<int64_t>{},
        py::arg("seg0_len") = 0, py::arg("seg0_per") = 0, py::arg("seg1_per") = 0,
        py::arg("o_strides") = std::vector<int64_t>{}, py::arg("acc_o") = py::none(),
        py::arg("acc_lse") = py::none(), py::arg("merge_mode") = 0, py::arg("kv_split") = -1);
  m.def("error_word", &error_word);
  m.def("symm_alloc", &symm_alloc);
  m.def("from_ptr", &from_ptr);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("memcpy_async", &memcpy_async);
  m.def("conv3d", &conv3d, "implicit-GEMM tcgen05 convolution (channels-last)", py::arg("x"), py::arg("w"),
        py::arg("bias") = py::none(), py::arg("kt") = 3, py::arg("kh") = 3, py::arg("kw") = 3,
        py::arg("causal") = true, py::arg("resid") = py::none(), py::arg("silu") = false, py::arg("out") = py::none(),
        py::arg("valid_t") = false, py::arg("valid_h") = false, py::arg("valid_w") = false);
  m.def("tp_reduce", &tp_reduce, py::arg("slots"), py::arg("slot_rows"), py::arg("world"), py::arg("rows"),
        py::arg("N"), py::arg("row0"), py::arg("bias") = py::none(), py::arg("gate") = py::none(),
        py::arg("rows_per_batch") = 0, py::arg("resid") = py::none(), py::arg("out") = std::vector<int64_t>{},
        py::arg("ldo") = 0, py::arg("out_row0") = 0, py::arg("resid_row0") = 0);
  m.def("peer_barrier", &peer_barrier);
  m.def("peer_put_f32", &peer_put_f32);
  m.def("cfg_combine", &cfg_combine);
  m.def("vae_chan_norm", &vae_chan_norm, py::arg("x"), py::arg("gamma"), py::arg("y"), py::arg("silu"),
        py::arg("halo") = false, py::arg("up") = 0, py::arg("up_rows") = 0, py::arg("down") = 0,
        py::arg("down_rows") = 0);
  m.def("gn_stats", &gn_stats, py::arg("x"), py::arg("G"), py::arg("eps"));
  m.def("gn_apply", &gn_apply, py::arg("x"), py::arg("stats"), py::arg("gamma"), py::arg("beta"), py::arg("G"),
        py::arg("silu"), py::arg("y"), py::arg("ot") = 0, py::arg("oh") = 0, py::arg("ow") = 0);
  m.def("pad_replicate", &pad_replicate, py::arg("y"), py::arg("pt"), py::arg("ph"), py::arg("pw"), py::arg("T"),
        py::arg("H"), py::arg("W"));
  m.def("upsample_causal", &upsample_causal, py::arg("x"), py::arg("up_t"), py::arg("y"), py::arg("ot") = 0,
        py::arg("oh") = 0, py::arg("ow") = 0);
  m.def("vae_upsample2x", &vae_upsample2x, py::arg("x"), py::arg("y"), py::arg("halo") = false, py::arg("up") = 0,
        py::arg("up_rows") = 0, py::arg("down") = 0, py::arg("down_rows") = 0);
  m.def("guided_step", &guided_step, py::arg("a"), py::arg("b_ptr"), py::arg("scale"), py::arg("x"),
        py::arg("x16") = py::none(), py::arg("last") = py::none(), py::arg("m1") = py::none(),
        py::arg("m2") = py::none(), py::arg("m_out") = py::none(), py::arg("coeffs"), py::arg("store_last"),
        py::arg("swap_ab") = false);
  m.def("rel_l1", &rel_l1);
}
