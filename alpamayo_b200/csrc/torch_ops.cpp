// torch_ops.cpp — thin TORCH_LIBRARY shim over the C ABI in include/paro_b200.h.
//
// Registers the ``paro_b200`` operator namespace (CUDA dispatch key only, like
// the reference's ``rotation`` namespace, kernels/paroquant_kernels/src/
// rotation.cu:576-584).  Ops allocate their outputs with the caching
// allocator, launch on the current stream and never synchronise, so they are
// CUDA-graph capturable; the Python package registers fake (meta) kernels so
// torch.compile(fullgraph=True) can trace them.  A non-zero paro_status
// becomes a RuntimeError, as the reference's TORCH_CHECKs do.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <map>
#include <mutex>
#include <utility>
#include <vector>

#include "../../include/paro_b200.h"

namespace {

int to_paro_dtype(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return PARO_F32;
    case at::kHalf: return PARO_F16;
    case at::kBFloat16: return PARO_BF16;
    default: TORCH_CHECK(false, "paro_b200: unsupported dtype ", t, " (Float, Half, BFloat16)");
  }
  return -1;
}

void check_status(int s, const char* what) {
  TORCH_CHECK(s == PARO_OK, "paro_b200::", what, " failed: ", paro_status_string(s),
              (s == PARO_ERR_CUDA ? std::string(" (") + paro_last_cuda_error() + ")" : std::string()));
}

paro_stream_t cur_stream() { return reinterpret_cast<paro_stream_t>(at::cuda::getCurrentCUDAStream().stream()); }

// GEMM workspace: one zero-filled buffer per (device, stream), kept for the
// life of the process (the kernels leave it zero-filled after every call, so
// it is reused without clearing; separate streams get separate buffers so
// concurrent calls do not share it).  It is allocated with at least 16 MiB on
// first use so later, larger calls (and CUDA graphs captured after a warm-up
// call) keep a stable address; it only grows for larger shapes.
std::mutex g_ws_mu;
std::map<std::pair<int, cudaStream_t>, at::Tensor>& ws_cache() {
  static std::map<std::pair<int, cudaStream_t>, at::Tensor> cache;
  return cache;
}

void* workspace_for(const c10::Device& dev, size_t bytes) {
  auto& cache = ws_cache();
  std::lock_guard<std::mutex> lock(g_ws_mu);
  const auto key = std::make_pair((int)dev.index(), at::cuda::getCurrentCUDAStream().stream());
  auto it = cache.find(key);
  if (it == cache.end() || (size_t)it->second.numel() < bytes) {
    const size_t want = std::max(bytes, (size_t)16 << 20);
    at::Tensor t = at::zeros({(int64_t)want}, at::TensorOptions().device(dev).dtype(at::kByte));
    cache[key] = t;
    return t.data_ptr();
  }
  return it->second.data_ptr();
}

void check_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "paro_b200: ", name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), "paro_b200: ", name, " must be contiguous");
}

// rotation::rotate(Tensor x, Tensor idx_ij, Tensor theta, Tensor? scales, int group_size) -> Tensor
at::Tensor rotate(const at::Tensor& x_in, const at::Tensor& idx_ij, const at::Tensor& theta,
                  const c10::optional<at::Tensor>& scales_opt, int64_t group_size) {
  at::Tensor x = x_in.contiguous();
  check_cuda(x, "x");
  check_cuda(idx_ij, "idx_ij");
  check_cuda(theta, "theta");
  TORCH_CHECK(idx_ij.scalar_type() == at::kShort, "idx_ij must be int16");
  TORCH_CHECK(theta.size(0) == idx_ij.size(0), "theta.size(0) must equal idx_ij.size(0)");
  const int64_t K = x.size(-1);
  TORCH_CHECK(K % group_size == 0, "h must be divisible by GROUP_SIZE");
  const void* sp = nullptr;
  at::Tensor sc;
  if (scales_opt.has_value() && scales_opt->defined() && scales_opt->numel() > 0) {
    sc = scales_opt->to(theta.scalar_type()).contiguous();
    check_cuda(sc, "scales");
    sp = sc.data_ptr();
  }
  c10::cuda::CUDAGuard guard(x.device());
  at::Tensor out = at::empty_like(x);
  const int64_t M = x.numel() / K;
  check_status(paro_rotate(x.data_ptr(), to_paro_dtype(x.scalar_type()), M, (int)K, sp, theta.data_ptr(),
                           to_paro_dtype(theta.scalar_type()), idx_ij.data_ptr<int16_t>(), (int)idx_ij.size(0),
                           (int)group_size, out.data_ptr(), cur_stream()),
               "rotate");
  return out;
}

// Validates the pair table and builds the per-channel rotation table
// (synchronises once to read the validation count: load-time only).  The
// uint32 table is returned in an int32 tensor.
at::Tensor prepare_rotation(const at::Tensor& pairs, const at::Tensor& theta, int64_t group_size) {
  check_cuda(pairs, "pairs");
  check_cuda(theta, "theta");
  TORCH_CHECK(pairs.scalar_type() == at::kShort, "pairs must be int16");
  TORCH_CHECK(theta.scalar_type() == at::kHalf, "theta must be float16");
  TORCH_CHECK(theta.size(0) == pairs.size(0) && theta.size(1) * 2 == pairs.size(1), "theta must be [krot, K/2]");
  c10::cuda::CUDAGuard guard(pairs.device());
  at::Tensor out = at::empty(pairs.sizes(), pairs.options().dtype(at::kInt));
  at::Tensor bad = at::empty({1}, pairs.options().dtype(at::kInt));
  check_status(paro_prepare_rotation(pairs.data_ptr<int16_t>(), reinterpret_cast<const uint16_t*>(theta.data_ptr()),
                                     (int)pairs.size(0), (int)pairs.size(1), (int)group_size,
                                     reinterpret_cast<uint32_t*>(out.data_ptr<int32_t>()), bad.data_ptr<int32_t>(),
                                     cur_stream()),
               "prepare_rotation");
  const int nbad = bad.item<int32_t>();
  TORCH_CHECK(nbad == 0, "paro_b200::prepare_rotation: ", nbad,
              " (layer, group) blocks of rotation.pairs are not permutations of 0..", group_size - 1,
              " (Givens pairs of one layer must be disjoint)");
  return out;
}

// The table extended with each group's rotation matrix (load time, one
// launch): int32 [136, K], rows 0-7 the table's words with the matrices flag
// in word 0, rows 8-135 the matrices (paro_prepare_rotation_matrices).
at::Tensor prepare_rotation_matrices(const at::Tensor& rot_table) {
  check_cuda(rot_table, "rot_table");
  TORCH_CHECK(rot_table.scalar_type() == at::kInt && rot_table.dim() == 2 && rot_table.size(0) == 8,
              "rot_table must be the int32 [8, K] tensor from prepare_rotation");
  const int64_t K = rot_table.size(1);
  TORCH_CHECK(K > 0 && K % 128 == 0, "rot_table: K must be a positive multiple of 128");
  c10::cuda::CUDAGuard guard(rot_table.device());
  at::Tensor out = at::empty({(int64_t)(paro_rotation_table_words((int)K, 1) / K), K}, rot_table.options());
  out.narrow(0, 0, 8).copy_(rot_table);
  check_status(paro_prepare_rotation_matrices(reinterpret_cast<uint32_t*>(out.data_ptr<int32_t>()), (int)K,
                                              cur_stream()),
               "prepare_rotation_matrices");
  return out;
}

// A krot-8 table: [8, K], or [136, K] carrying the matrices.
bool rot8_table(const at::Tensor& t, int64_t K) {
  return t.dim() == 2 && t.size(1) == K && (t.size(0) == 8 || t.size(0) == 136);
}

std::tuple<at::Tensor, at::Tensor> rotq_int8(const at::Tensor& x_in, const at::Tensor& rot_table,
                                             const c10::optional<at::Tensor>& scales_opt, int64_t group_size,
                                             bool fp16_round) {
  at::Tensor x = x_in.contiguous();
  check_cuda(x, "x");
  check_cuda(rot_table, "rot_table");
  TORCH_CHECK(rot_table.scalar_type() == at::kInt, "rot_table must be the int32 tensor from prepare_rotation");
  TORCH_CHECK(rot_table.size(-1) == x.size(-1), "rot_table must be [krot, K]");
  const int64_t K = x.size(-1);
  const uint16_t* sp = nullptr;
  at::Tensor sc;
  if (scales_opt.has_value() && scales_opt->defined() && scales_opt->numel() > 0) {
    sc = scales_opt->to(at::kHalf).contiguous();
    check_cuda(sc, "scales");
    sp = reinterpret_cast<const uint16_t*>(sc.data_ptr());
  }
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t M = x.numel() / K;
  at::Tensor q = at::empty(x.sizes(), x.options().dtype(at::kChar));
  auto ssz = x.sizes().vec();
  ssz.back() = 1;
  at::Tensor s = at::empty(ssz, x.options().dtype(at::kFloat));
  // prefill sizes take the two-pass path; its workspace comes from the
  // caching allocator and is released when this call returns
  const size_t wsb = paro_rotq_int8_workspace_size(M, (int)K, fp16_round ? 1 : 0);
  at::Tensor ws;
  if (wsb) ws = at::empty({(int64_t)wsb + 256}, x.options().dtype(at::kByte));
  void* wsp = wsb ? reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(ws.data_ptr()) + 255) & ~(uintptr_t)255)
                  : nullptr;
  check_status(paro_rotq_int8_ws(x.data_ptr(), to_paro_dtype(x.scalar_type()), M, (int)K, sp,
                                 reinterpret_cast<const uint32_t*>(rot_table.data_ptr<int32_t>()),
                                 rot8_table(rot_table, K) ? 8 : (int)rot_table.size(0), (int)group_size,
                                 fp16_round ? 1 : 0, q.data_ptr<int8_t>(),
                                 s.data_ptr<float>(), wsp, wsb, cur_stream()),
               "rotq_int8");
  return {q, s};
}

// per_token_quant_int8 (vllm int8_utils.py:131-156): returns (int8 codes, float32 scales [..., 1])
std::tuple<at::Tensor, at::Tensor> quant_int8(const at::Tensor& x_in) {
  at::Tensor x = x_in.contiguous();
  check_cuda(x, "x");
  const int64_t K = x.size(-1);
  const int64_t M = x.numel() / K;
  c10::cuda::CUDAGuard guard(x.device());
  at::Tensor q = at::empty(x.sizes(), x.options().dtype(at::kChar));
  auto ssz = x.sizes().vec();
  ssz.back() = 1;
  at::Tensor s = at::empty(ssz, x.options().dtype(at::kFloat));
  check_status(paro_quant_int8(x.data_ptr(), to_paro_dtype(x.scalar_type()), M, (int)K, q.data_ptr<int8_t>(),
                               s.data_ptr<float>(), cur_stream()),
               "quant_int8");
  return {q, s};
}

at::Tensor prepare_weights(const at::Tensor& qweight, const at::Tensor& scales, const at::Tensor& scaled_zeros,
                           int64_t N, int64_t K) {
  check_cuda(qweight, "qweight");
  check_cuda(scales, "scales");
  check_cuda(scaled_zeros, "scaled_zeros");
  TORCH_CHECK(qweight.scalar_type() == at::kShort, "qweight must be int16 (WQLinear layout)");
  TORCH_CHECK(scales.scalar_type() == at::kHalf && scaled_zeros.scalar_type() == at::kHalf,
              "scales / scaled_zeros must be float16");
  TORCH_CHECK(qweight.size(0) * 4 == N && qweight.size(1) == K, "qweight must be [N/4, K]");
  TORCH_CHECK(scales.size(1) == N && scaled_zeros.sizes() == scales.sizes(), "scales must be [G_pad, N]");
  c10::cuda::CUDAGuard guard(qweight.device());
  const size_t bytes = paro_packed_weight_bytes((int)N, (int)K);
  TORCH_CHECK(bytes > 0, "paro_b200::prepare_weights: N must be a multiple of 16 and K of 128");
  at::Tensor packed = at::empty({(int64_t)bytes}, qweight.options().dtype(at::kByte));
  check_status(paro_prepare_weights(qweight.data_ptr<int16_t>(), reinterpret_cast<const uint16_t*>(scales.data_ptr()),
                                    reinterpret_cast<const uint16_t*>(scaled_zeros.data_ptr()), (int)N, (int)K,
                                    (int)scales.size(0), packed.data_ptr(), cur_stream()),
               "prepare_weights");
  return packed;
}

at::Tensor prepare_weights_awq(const at::Tensor& qweight, const at::Tensor& scales, const at::Tensor& qzeros,
                               int64_t N, int64_t K) {
  check_cuda(qweight, "qweight");
  check_cuda(scales, "scales");
  check_cuda(qzeros, "qzeros");
  TORCH_CHECK(qweight.scalar_type() == at::kInt && qzeros.scalar_type() == at::kInt, "AWQ buffers must be int32");
  TORCH_CHECK(scales.scalar_type() == at::kHalf, "scales must be float16");
  TORCH_CHECK(qweight.size(0) == K && qweight.size(1) * 8 == N, "qweight must be [K, N/8]");
  c10::cuda::CUDAGuard guard(qweight.device());
  const size_t bytes = paro_packed_weight_bytes((int)N, (int)K);
  TORCH_CHECK(bytes > 0, "paro_b200::prepare_weights_awq: N must be a multiple of 16 and K of 128");
  at::Tensor packed = at::empty({(int64_t)bytes}, qweight.options().dtype(at::kByte));
  check_status(paro_prepare_weights_awq(qweight.data_ptr<int32_t>(),
                                        reinterpret_cast<const uint16_t*>(scales.data_ptr()),
                                        qzeros.data_ptr<int32_t>(), (int)N, (int)K, packed.data_ptr(), cur_stream()),
               "prepare_weights_awq");
  return packed;
}

at::Tensor w4a8_gemm(const at::Tensor& xq_in, const at::Tensor& xscale_in, const at::Tensor& packed, int64_t N,
                     const c10::optional<at::Tensor>& bias_opt, at::ScalarType out_dtype) {
  at::Tensor xq = xq_in.contiguous();
  at::Tensor xscale = xscale_in.contiguous();
  check_cuda(xq, "xq");
  check_cuda(xscale, "xscale");
  check_cuda(packed, "packed");
  TORCH_CHECK(xq.scalar_type() == at::kChar, "xq must be int8");
  TORCH_CHECK(xscale.scalar_type() == at::kFloat, "xscale must be float32");
  const int64_t K = xq.size(-1);
  const int64_t M = xq.numel() / K;
  TORCH_CHECK(xscale.numel() == M, "xscale must hold one scale per token");
  TORCH_CHECK((size_t)packed.numel() == paro_packed_weight_bytes((int)N, (int)K), "packed weight size mismatch");
  const void* bp = nullptr;
  int bdt = PARO_F32;
  at::Tensor bias;
  if (bias_opt.has_value() && bias_opt->defined()) {
    bias = bias_opt->contiguous();
    check_cuda(bias, "bias");
    TORCH_CHECK(bias.numel() == N, "bias must have N elements");
    bp = bias.data_ptr();
    bdt = to_paro_dtype(bias.scalar_type());
  }
  c10::cuda::CUDAGuard guard(xq.device());
  auto osz = xq.sizes().vec();
  osz.back() = N;
  at::Tensor out = at::empty(osz, xq.options().dtype(out_dtype));
  const size_t ws = paro_w4a8_gemm_workspace_size(M, (int)N, (int)K);
  void* wsp = ws ? workspace_for(xq.device(), ws) : nullptr;
  check_status(paro_w4a8_gemm(xq.data_ptr<int8_t>(), xscale.data_ptr<float>(), M, (int)N, (int)K, packed.data_ptr(),
                              bp, bdt, out.data_ptr(), to_paro_dtype(out_dtype), wsp, ws, cur_stream()),
               "w4a8_gemm");
  return out;
}

// One W4A8 rotated linear (paro_w4a8_linear: rotation kernel + GEMM with
// in-prologue quantisation at decode sizes).
at::Tensor linear_w4a8(const at::Tensor& x_in, const at::Tensor& rot_table,
                       const c10::optional<at::Tensor>& channel_scales, const at::Tensor& packed, int64_t N,
                       const c10::optional<at::Tensor>& bias_opt, bool fp16_round, at::ScalarType out_dtype) {
  at::Tensor x = x_in.contiguous();
  check_cuda(x, "x");
  check_cuda(rot_table, "rot_table");
  check_cuda(packed, "packed");
  TORCH_CHECK(rot_table.scalar_type() == at::kInt, "rot_table must be the int32 tensor from prepare_rotation");
  const int64_t K = x.size(-1);
  TORCH_CHECK(rot8_table(rot_table, K), "rot_table must be [8, K] (or [136, K] with the matrices)");
  TORCH_CHECK((size_t)packed.numel() == paro_packed_weight_bytes((int)N, (int)K), "packed weight size mismatch");
  const int64_t M = x.numel() / K;
  const uint16_t* csp = nullptr;
  at::Tensor cs;
  if (channel_scales.has_value() && channel_scales->defined() && channel_scales->numel() > 0) {
    cs = channel_scales->to(at::kHalf).contiguous();
    check_cuda(cs, "channel_scales");
    csp = reinterpret_cast<const uint16_t*>(cs.data_ptr());
  }
  const void* bp = nullptr;
  int bdt = PARO_F32;
  at::Tensor bias;
  if (bias_opt.has_value() && bias_opt->defined()) {
    bias = bias_opt->contiguous();
    check_cuda(bias, "bias");
    TORCH_CHECK(bias.numel() == N, "bias must have N elements");
    bp = bias.data_ptr();
    bdt = to_paro_dtype(bias.scalar_type());
  }
  c10::cuda::CUDAGuard guard(x.device());
  auto osz = x.sizes().vec();
  osz.back() = N;
  at::Tensor out = at::empty(osz, x.options().dtype(out_dtype));
  if (M == 0) return out;
  const size_t wsb = paro_w4a8_linear_workspace_size(M, (int)N, (int)K);
  void* wsp = workspace_for(x.device(), wsb);
  // the scratch needs no initial contents: take it from the caching allocator
  const size_t scb = paro_w4a8_linear_scratch_size(M, (int)N, (int)K, fp16_round ? 1 : 0);
  at::Tensor sct = at::empty({(int64_t)scb + 256}, x.options().dtype(at::kByte));
  void* scp = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(sct.data_ptr()) + 255) & ~(uintptr_t)255);
  check_status(paro_w4a8_linear(x.data_ptr(), to_paro_dtype(x.scalar_type()), M, (int)K, (int)N, csp,
                                reinterpret_cast<const uint32_t*>(rot_table.data_ptr<int32_t>()), fp16_round ? 1 : 0,
                                packed.data_ptr(), bp, bdt, out.data_ptr(), to_paro_dtype(out_dtype), wsp, wsb, scp,
                                scb, cur_stream()),
               "linear_w4a8");
  return out;
}

// One rotated linear with the decoder-layer step before it fused in
// (paro_w4a8_linear_prologue): returns (y, new residual stream); the
// residual output is a fresh tensor (never the input's storage).
std::tuple<at::Tensor, at::Tensor> linear_prologue(int prologue, const at::Tensor& x_in,
                                                   const c10::optional<at::Tensor>& residual_opt,
                                                   const c10::optional<at::Tensor>& norm_weight, double eps,
                                                   const at::Tensor& rot_table,
                                                   const c10::optional<at::Tensor>& channel_scales,
                                                   const at::Tensor& packed, int64_t N,
                                                   const c10::optional<at::Tensor>& bias_opt, bool fp16_round,
                                                   at::ScalarType out_dtype) {
  at::Tensor x = x_in.contiguous();
  check_cuda(x, "x");
  check_cuda(rot_table, "rot_table");
  check_cuda(packed, "packed");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "fused prologue: bf16 input expected");
  TORCH_CHECK(rot_table.scalar_type() == at::kInt, "rot_table must be the int32 tensor from prepare_rotation");
  const bool rms = prologue == PARO_PROLOGUE_ADD_RMSNORM;
  const int64_t K = rms ? x.size(-1) : x.size(-1) / 2;
  TORCH_CHECK(rms || x.size(-1) == 2 * K, "silu prologue: input must be [..., 2K]");
  TORCH_CHECK(rot8_table(rot_table, K), "rot_table must be [8, K] (or [136, K] with the matrices)");
  TORCH_CHECK((size_t)packed.numel() == paro_packed_weight_bytes((int)N, (int)K), "packed weight size mismatch");
  const int64_t M = x.numel() / x.size(-1);
  const uint16_t* csp = nullptr;
  at::Tensor cs;
  if (channel_scales.has_value() && channel_scales->defined() && channel_scales->numel() > 0) {
    cs = channel_scales->to(at::kHalf).contiguous();
    check_cuda(cs, "channel_scales");
    csp = reinterpret_cast<const uint16_t*>(cs.data_ptr());
  }
  const void* bp = nullptr;
  int bdt = PARO_F32;
  at::Tensor bias;
  if (bias_opt.has_value() && bias_opt->defined()) {
    bias = bias_opt->contiguous();
    check_cuda(bias, "bias");
    TORCH_CHECK(bias.numel() == N, "bias must have N elements");
    bp = bias.data_ptr();
    bdt = to_paro_dtype(bias.scalar_type());
  }
  at::Tensor res_in, res_out, w;
  if (rms) {
    TORCH_CHECK(norm_weight.has_value() && norm_weight->defined(), "add_rmsnorm prologue needs the norm weight");
    w = norm_weight->contiguous();
    check_cuda(w, "norm_weight");
    TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.numel() == K, "norm_weight must be bf16 [K]");
    if (residual_opt.has_value() && residual_opt->defined()) {
      res_in = residual_opt->contiguous();
      TORCH_CHECK(res_in.sizes() == x.sizes() && res_in.scalar_type() == at::kBFloat16, "residual must match x");
    }
    res_out = at::empty_like(x);
  }
  c10::cuda::CUDAGuard guard(x.device());
  auto osz = x.sizes().vec();
  osz.back() = N;
  at::Tensor out = at::empty(osz, x.options().dtype(out_dtype));
  if (M == 0) return {out, rms ? res_out : x};
  const size_t wsb = paro_w4a8_linear_workspace_size(M, (int)N, (int)K);
  void* wsp = workspace_for(x.device(), wsb);
  const size_t scb = paro_w4a8_linear_prologue_scratch_size(prologue, M, (int)N, (int)K, fp16_round ? 1 : 0);
  at::Tensor sct = at::empty({(int64_t)scb + 256}, x.options().dtype(at::kByte));
  void* scp = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(sct.data_ptr()) + 255) & ~(uintptr_t)255);
  check_status(paro_w4a8_linear_prologue(prologue, x.data_ptr(), res_in.defined() ? res_in.data_ptr() : nullptr,
                                         rms ? res_out.data_ptr() : nullptr, rms ? w.data_ptr() : nullptr,
                                         (float)eps, M, (int)K, (int)N, csp,
                                         reinterpret_cast<const uint32_t*>(rot_table.data_ptr<int32_t>()),
                                         fp16_round ? 1 : 0, packed.data_ptr(), bp, bdt, out.data_ptr(),
                                         to_paro_dtype(out_dtype), wsp, wsb, scp, scb, cur_stream()),
               "linear_w4a8 (fused prologue)");
  return {out, rms ? res_out : x};
}

std::tuple<at::Tensor, at::Tensor> linear_w4a8_rmsnorm(const at::Tensor& x, const c10::optional<at::Tensor>& residual,
                                                       const at::Tensor& norm_weight, double eps,
                                                       const at::Tensor& rot_table,
                                                       const c10::optional<at::Tensor>& channel_scales,
                                                       const at::Tensor& packed, int64_t N,
                                                       const c10::optional<at::Tensor>& bias, bool fp16_round,
                                                       at::ScalarType out_dtype) {
  return linear_prologue(PARO_PROLOGUE_ADD_RMSNORM, x, residual, norm_weight, eps, rot_table, channel_scales, packed, N,
                         bias, fp16_round, out_dtype);
}

at::Tensor linear_w4a8_silu(const at::Tensor& gate_up, const at::Tensor& rot_table,
                            const c10::optional<at::Tensor>& channel_scales, const at::Tensor& packed, int64_t N,
                            const c10::optional<at::Tensor>& bias, bool fp16_round, at::ScalarType out_dtype) {
  return std::get<0>(linear_prologue(PARO_PROLOGUE_SILU_MUL, gate_up, c10::nullopt, c10::nullopt, 0.0, rot_table,
                                     channel_scales, packed, N, bias, fp16_round, out_dtype));
}

// A group of rotated linears sharing x, one rotation table each, weights
// concatenated along N (paro_w4a8_linear_group): returns ([..., sum N],
// new residual stream or x).
std::tuple<at::Tensor, at::Tensor> linear_w4a8_group(const at::Tensor& x_in, const c10::optional<at::Tensor>& residual,
                                                     const c10::optional<at::Tensor>& norm_weight, double eps,
                                                     int64_t prologue, at::TensorList rot_tables,
                                                     at::TensorList channel_scales, const at::Tensor& packed,
                                                     at::IntArrayRef n_per_table,
                                                     const c10::optional<at::Tensor>& bias_opt, bool fp16_round,
                                                     at::ScalarType out_dtype) {
  at::Tensor x = x_in.contiguous();
  check_cuda(x, "x");
  check_cuda(packed, "packed");
  const int T = (int)rot_tables.size();
  TORCH_CHECK(T >= 1 && T <= 4, "linear group: 1 to 4 rotation tables");
  TORCH_CHECK((int)n_per_table.size() == T, "one output width per table");
  TORCH_CHECK(channel_scales.empty() || (int)channel_scales.size() == T, "one channel-scale vector per table");
  const bool rms = prologue == PARO_PROLOGUE_ADD_RMSNORM, silu = prologue == PARO_PROLOGUE_SILU_MUL;
  const int64_t K = silu ? x.size(-1) / 2 : x.size(-1);
  const int64_t M = x.numel() / x.size(-1);
  std::vector<int> ns(T);
  int64_t N = 0;
  std::vector<const uint32_t*> tabs(T);
  std::vector<const uint16_t*> css(T, nullptr);
  std::vector<at::Tensor> keep;
  for (int t = 0; t < T; ++t) {
    ns[t] = (int)n_per_table[t];
    N += ns[t];
    check_cuda(rot_tables[t], "rot_table");
    TORCH_CHECK(rot_tables[t].scalar_type() == at::kInt && rot8_table(rot_tables[t], K),
                "rot_tables must be int32 [8, K] (or [136, K]) tensors from prepare_rotation");
    tabs[t] = reinterpret_cast<const uint32_t*>(rot_tables[t].data_ptr<int32_t>());
    if (!channel_scales.empty() && channel_scales[t].defined() && channel_scales[t].numel() > 0) {
      at::Tensor c = channel_scales[t].to(at::kHalf).contiguous();
      check_cuda(c, "channel_scales");
      keep.push_back(c);
      css[t] = reinterpret_cast<const uint16_t*>(c.data_ptr());
    }
  }
  TORCH_CHECK((size_t)packed.numel() == paro_packed_weight_bytes((int)N, (int)K), "packed weight size mismatch");
  const void* bp = nullptr;
  int bdt = PARO_F32;
  at::Tensor bias;
  if (bias_opt.has_value() && bias_opt->defined()) {
    bias = bias_opt->contiguous();
    check_cuda(bias, "bias");
    TORCH_CHECK(bias.numel() == N, "bias must have sum(n_per_table) elements");
    bp = bias.data_ptr();
    bdt = to_paro_dtype(bias.scalar_type());
  }
  at::Tensor res_in, res_out, w;
  if (rms) {
    TORCH_CHECK(norm_weight.has_value() && norm_weight->defined(), "add_rmsnorm prologue needs the norm weight");
    w = norm_weight->contiguous();
    TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.numel() == K, "norm_weight must be bf16 [K]");
    if (residual.has_value() && residual->defined()) res_in = residual->contiguous();
    res_out = at::empty_like(x);
  }
  c10::cuda::CUDAGuard guard(x.device());
  auto osz = x.sizes().vec();
  osz.back() = N;
  at::Tensor out = at::empty(osz, x.options().dtype(out_dtype));
  if (M == 0) return {out, rms ? res_out : x};
  const size_t wsb = paro_w4a8_linear_group_workspace_size(M, T, ns.data(), (int)K);
  void* wsp = workspace_for(x.device(), wsb);
  const size_t scb = paro_w4a8_linear_group_scratch_size((int)prologue, M, T, ns.data(), (int)K, fp16_round ? 1 : 0);
  at::Tensor sct = at::empty({(int64_t)scb + 256}, x.options().dtype(at::kByte));
  void* scp = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(sct.data_ptr()) + 255) & ~(uintptr_t)255);
  check_status(paro_w4a8_linear_group((int)prologue, x.data_ptr(), to_paro_dtype(x.scalar_type()),
                                      res_in.defined() ? res_in.data_ptr() : nullptr,
                                      rms ? res_out.data_ptr() : nullptr, rms ? w.data_ptr() : nullptr, (float)eps, M,
                                      (int)K, T, ns.data(), css.data(), tabs.data(), fp16_round ? 1 : 0,
                                      packed.data_ptr(), bp, bdt, out.data_ptr(), to_paro_dtype(out_dtype), wsp, wsb,
                                      scp, scb, cur_stream()),
               "linear_w4a8_group");
  return {out, rms ? res_out : x};
}

// residual add + RMSNorm: returns (normalised, new residual); residual may be
// None (then the new residual is x itself)
std::tuple<at::Tensor, at::Tensor> add_rmsnorm(const at::Tensor& x_in, const c10::optional<at::Tensor>& residual_opt,
                                               const at::Tensor& weight, double eps) {
  at::Tensor x = x_in.contiguous();
  check_cuda(x, "x");
  check_cuda(weight, "weight");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && weight.scalar_type() == at::kBFloat16,
              "add_rmsnorm: bf16 tensors expected");
  const int64_t K = x.size(-1);
  TORCH_CHECK(weight.numel() == K, "weight must have K elements");
  const int64_t M = x.numel() / K;
  c10::cuda::CUDAGuard guard(x.device());
  at::Tensor res;
  void* rp = nullptr;
  if (residual_opt.has_value() && residual_opt->defined()) {
    res = residual_opt->contiguous().clone();
    TORCH_CHECK(res.sizes() == x.sizes() && res.scalar_type() == at::kBFloat16, "residual must match x");
    rp = res.data_ptr();
  }
  at::Tensor out = at::empty_like(x);
  check_status(paro_add_rmsnorm(x.data_ptr(), rp, weight.data_ptr(), M, (int)K, (float)eps, out.data_ptr(),
                                cur_stream()),
               "add_rmsnorm");
  return {out, rp ? res : x};
}

at::Tensor silu_mul(const at::Tensor& x_in) {
  at::Tensor x = x_in.contiguous();
  check_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16, "silu_mul: bf16 expected");
  const int64_t I2 = x.size(-1);
  TORCH_CHECK(I2 % 16 == 0, "silu_mul: last dimension must be 2*I with I % 8 == 0");
  const int64_t M = x.numel() / I2;
  c10::cuda::CUDAGuard guard(x.device());
  auto osz = x.sizes().vec();
  osz.back() = I2 / 2;
  at::Tensor out = at::empty(osz, x.options());
  check_status(paro_silu_mul(x.data_ptr(), M, (int)(I2 / 2), out.data_ptr(), cur_stream()), "silu_mul");
  return out;
}

}  // namespace

// Zero-fill every cached GEMM workspace again (after a kernel's bounded
// wait ran out, an unfinished cross-CTA fix-up may have left partial sums or
// counters in one).  Synchronises the device first, so no kernel is still
// using them.  Returns the number of workspaces cleared, or -1 on a CUDA
// error.
extern "C" int paro_torch_reset_workspaces() {
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  std::lock_guard<std::mutex> lock(g_ws_mu);
  int n = 0;
  for (auto& kv : ws_cache()) {
    c10::cuda::CUDAGuard guard((c10::DeviceIndex)kv.first.first);
    if (cudaMemset(kv.second.data_ptr(), 0, (size_t)kv.second.numel()) != cudaSuccess) return -1;
    ++n;
  }
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  return n;
}

TORCH_LIBRARY(paro_b200, m) {
  m.def("rotate(Tensor x, Tensor idx_ij, Tensor theta, Tensor? scales, int group_size) -> Tensor");
  m.def("prepare_rotation(Tensor pairs, Tensor theta, int group_size) -> Tensor");
  m.def("prepare_rotation_matrices(Tensor rot_table) -> Tensor");
  m.def("rotq_int8(Tensor x, Tensor rot_table, Tensor? scales, int group_size, bool fp16_round) -> (Tensor, Tensor)");
  m.def("quant_int8(Tensor x) -> (Tensor, Tensor)");
  m.def("prepare_weights(Tensor qweight, Tensor scales, Tensor scaled_zeros, int N, int K) -> Tensor");
  m.def("prepare_weights_awq(Tensor qweight, Tensor scales, Tensor qzeros, int N, int K) -> Tensor");
  m.def("w4a8_gemm(Tensor xq, Tensor xscale, Tensor packed, int N, Tensor? bias, ScalarType out_dtype) -> Tensor");
  m.def("linear_w4a8(Tensor x, Tensor rot_table, Tensor? channel_scales, Tensor packed, int N, Tensor? bias, "
        "bool fp16_round, ScalarType out_dtype) -> Tensor");
  m.def("add_rmsnorm(Tensor x, Tensor? residual, Tensor weight, float eps) -> (Tensor, Tensor)");
  m.def("silu_mul(Tensor x) -> Tensor");
  m.def("linear_w4a8_rmsnorm(Tensor x, Tensor? residual, Tensor norm_weight, float eps, Tensor rot_table, "
        "Tensor? channel_scales, Tensor packed, int N, Tensor? bias, bool fp16_round, ScalarType out_dtype) "
        "-> (Tensor, Tensor)");
  m.def("linear_w4a8_group(Tensor x, Tensor? residual, Tensor? norm_weight, float eps, int prologue, "
        "Tensor[] rot_tables, Tensor[] channel_scales, Tensor packed, int[] n_per_table, Tensor? bias, "
        "bool fp16_round, ScalarType out_dtype) -> (Tensor, Tensor)");
  m.def("linear_w4a8_silu(Tensor gate_up, Tensor rot_table, Tensor? channel_scales, Tensor packed, int N, "
        "Tensor? bias, bool fp16_round, ScalarType out_dtype) -> Tensor");
}

TORCH_LIBRARY_IMPL(paro_b200, CUDA, m) {
  m.impl("rotate", &rotate);
  m.impl("prepare_rotation", &prepare_rotation);
  m.impl("prepare_rotation_matrices", &prepare_rotation_matrices);
  m.impl("rotq_int8", &rotq_int8);
  m.impl("quant_int8", &quant_int8);
  m.impl("prepare_weights", &prepare_weights);
  m.impl("prepare_weights_awq", &prepare_weights_awq);
  m.impl("w4a8_gemm", &w4a8_gemm);
  m.impl("linear_w4a8", &linear_w4a8);
  m.impl("add_rmsnorm", &add_rmsnorm);
  m.impl("silu_mul", &silu_mul);
  m.impl("linear_w4a8_rmsnorm", &linear_w4a8_rmsnorm);
  m.impl("linear_w4a8_silu", &linear_w4a8_silu);
  m.impl("linear_w4a8_group", &linear_w4a8_group);
}
