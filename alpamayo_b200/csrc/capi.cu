// capi.cu — the extern "C" entry points declared in include/paro_b200.h.
//
// Each entry point validates its arguments on the host (status codes instead
// of exceptions; the torch shim turns a non-zero status into a RuntimeError,
// mirroring the reference's TORCH_CHECKs in rotation.cu:117-124,456-493),
// then launches asynchronously on the caller's stream.  Nothing here
// allocates device memory or synchronises.
#include <algorithm>
#include <cstring>
#include <string>

#include "tc_ptx.cuh"

namespace paro {
cudaError_t launch_rotate(int x_dtype, int krot, int group, const void* x, int64_t M, int K, const void* scales,
                          const void* theta, int pdt, const int16_t* pairs, void* out, cudaStream_t st);
cudaError_t launch_rotq(int x_dtype, const void* x, int64_t M, int K, const uint16_t* scales, const uint32_t* rtab,
                        int fp16_round, int8_t* q, float* s, cudaStream_t st);
int rotq_max_k();
size_t rotq_rows_workspace(int64_t M, int K);
int rotq_rows_min_m();
cudaError_t launch_rotq_rows(int x_dtype, const void* x, int64_t M, int K, const uint16_t* scales,
                             const uint32_t* rtab, int8_t* q, float* s, void* ws, cudaStream_t st);
cudaError_t launch_quant(int x_dtype, const void* x, int64_t M, int K, int8_t* q, float* s, cudaStream_t st);
cudaError_t launch_prepare_rotation(const int16_t* pairs, const uint16_t* theta, int krot, int K, int group,
                                    uint32_t* out, int32_t* bad, cudaStream_t st);
cudaError_t launch_prepare_rotation_matrices(uint32_t* table, int K, cudaStream_t st);
cudaError_t launch_prepare_wq(const int16_t* qweight, const uint16_t* scales, const uint16_t* scaled_zeros, int N,
                              int K, void* packed, cudaStream_t st);
cudaError_t launch_prepare_awq(const int32_t* qweight, const uint16_t* scales, const int32_t* qzeros, int N, int K,
                               void* packed, cudaStream_t st);
cudaError_t launch_gemm_decode(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                               const void* bias, int bias_dtype, void* out, int out_dtype, void* ws,
                               cudaStream_t st);
size_t gemm_decode_workspace(int64_t M, int N);
cudaError_t launch_add_rmsnorm(const void* x, void* residual, const void* weight, int64_t M, int K, float eps,
                               void* out, cudaStream_t st);
cudaError_t launch_silu_mul(const void* x, int64_t M, int I, void* out, cudaStream_t st);
size_t linear_decode_workspace(int64_t M, int N, int K, int T);
size_t linear_decode_scratch(int64_t M, int K, int T);
cudaError_t launch_linear_decode_tables(const void* x, int x_dtype, const RotTables& tabs, int T, const int* tab_nb,
                                        int64_t M, int N, int K, const void* packed, const void* bias, int bias_dtype,
                                        void* out, int out_dtype, void* ws, void* scratch, int pro_kind,
                                        const RotPro& pro, cudaStream_t st);
cudaError_t launch_linear_decode(const void* x, int x_dtype, const uint16_t* cscale, const uint32_t* rtab, int64_t M,
                                 int N, int K, const void* packed, const void* bias, int bias_dtype, void* out,
                                 int out_dtype, void* ws, void* scratch, int pro_kind, const RotPro& pro,
                                 cudaStream_t st);
int gemm_tc_supported(int64_t M, int N, int K);
size_t gemm_tc_workspace(int64_t M, int N, int K);
size_t gemm_tc_workspace_tile(int64_t M, int N, int K, int bt);
cudaError_t launch_gemm_rows(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                             const void* bias, int bias_dtype, void* out, int out_dtype, void* ws, uint32_t* amax,
                             const int* gsum, int gsum_mp, cudaStream_t st, int any_shape);
cudaError_t launch_gemm_tc_tile(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                                const void* bias, int bias_dtype, void* out, int out_dtype, void* workspace,
                                size_t workspace_bytes, int T, const int* tab_nb, int bt, cudaStream_t st,
                                uint32_t* zero_after, int zero_n, int out_mc);
cudaError_t launch_selftest_wait(long long limit_cycles, cudaStream_t st);
cudaError_t launch_gemm_tc(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                           const void* bias, int bias_dtype, void* out, int out_dtype, void* ws, size_t ws_bytes,
                           cudaStream_t st);
cudaError_t launch_gemm_tc_sets(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                                const void* bias, int bias_dtype, void* out, int out_dtype, void* workspace,
                                size_t workspace_bytes, int T, const int* tab_nb, cudaStream_t st);
int gemm_tc_sets_ok(int T, const int* tab_nb);
}  // namespace paro

#include <map>
#include <mutex>

namespace paro {
uint32_t error_word_decode(int clear);
uint32_t error_word_tc(int clear);
uint32_t error_word_rtc(int clear);
uint32_t error_word_rows(int clear);

cudaError_t ensure_smem_limit(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  int& have = done[std::make_pair(kernel, dev)];
  if (have >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) have = bytes;
  return e;
}
}  // namespace paro

using namespace paro;

namespace {
thread_local std::string g_last_cuda_error;

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return PARO_OK;
  g_last_cuda_error = cudaGetErrorString(e);
  return PARO_ERR_CUDA;
}

bool valid_dtype(int d) { return d == PARO_F32 || d == PARO_F16 || d == PARO_BF16; }

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int device_check() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PARO_ERR_DEVICE;
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return PARO_ERR_DEVICE;
  return major == 10 ? PARO_OK : PARO_ERR_DEVICE;
}
}  // namespace

extern "C" {

const char* paro_status_string(int s) {
  switch (s) {
    case PARO_OK: return "ok";
    case PARO_ERR_INVALID_ARGUMENT: return "invalid argument";
    case PARO_ERR_SHAPE: return "unsupported shape";
    case PARO_ERR_UNSUPPORTED: return "unsupported configuration";
    case PARO_ERR_MISALIGNED: return "misaligned pointer";
    case PARO_ERR_CUDA: return "CUDA error";
    case PARO_ERR_WORKSPACE: return "workspace too small";
    case PARO_ERR_DEVICE: return "current device is not an sm_100 GPU";
    case PARO_ERR_TOO_LARGE: return "size beyond compiled limit";
  }
  return "unknown status";
}

int paro_version(void) { return 100; }

const char* paro_last_cuda_error(void) { return g_last_cuda_error.c_str(); }

int paro_prepare_rotation(const int16_t* pairs, const uint16_t* theta, int krot, int K, int group,
                          uint32_t* out_table, int32_t* bad, paro_stream_t stream) {
  if (!pairs || !theta || !out_table || !bad || krot <= 0 || K <= 0) return PARO_ERR_INVALID_ARGUMENT;
  if (group != 128) return PARO_ERR_UNSUPPORTED;
  if (K % group) return PARO_ERR_SHAPE;
  if (int d = device_check()) return d;
  return cuda_status(launch_prepare_rotation(pairs, theta, krot, K, group, out_table, bad, (cudaStream_t)stream));
}

size_t paro_rotation_table_words(int K, int with_matrices) {
  if (K <= 0 || K % kGroup) return 0;
  return (size_t)(with_matrices ? 8 + 128 : 8) * (size_t)K;
}

int paro_prepare_rotation_matrices(uint32_t* table, int K, paro_stream_t stream) {
  if (!table || K <= 0) return PARO_ERR_INVALID_ARGUMENT;
  if (K % kGroup) return PARO_ERR_SHAPE;
  if (!aligned(table, 16)) return PARO_ERR_MISALIGNED;
  if (int d = device_check()) return d;
  return cuda_status(launch_prepare_rotation_matrices(table, K, (cudaStream_t)stream));
}

int paro_rotate(const void* x, int x_dtype, int64_t M, int K, const void* scales, const void* theta,
                int param_dtype, const int16_t* pairs, int krot, int group, void* out, paro_stream_t stream) {
  if (M == 0 && K > 0) return PARO_OK;
  if (!x || !theta || !pairs || !out || K <= 0 || M < 0) return PARO_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(x_dtype) || !valid_dtype(param_dtype)) return PARO_ERR_UNSUPPORTED;
  if (group != 64 && group != 128) return PARO_ERR_UNSUPPORTED;
  if (krot != 1 && krot != 2 && krot != 4 && krot != 8 && krot != 16) return PARO_ERR_UNSUPPORTED;
  if (K % group) return PARO_ERR_SHAPE;
  if (!aligned(pairs, 4)) return PARO_ERR_MISALIGNED;
  if (M == 0) return PARO_OK;
  if (int d = device_check()) return d;
  return cuda_status(
      launch_rotate(x_dtype, krot, group, x, M, K, scales, theta, param_dtype, pairs, out, (cudaStream_t)stream));
}

int paro_rotq_int8(const void* x, int x_dtype, int64_t M, int K, const uint16_t* scales, const uint32_t* rot_table,
                   int krot, int group, int fp16_round, int8_t* out_q, float* out_scale, paro_stream_t stream) {
  if (M == 0 && K > 0) return PARO_OK;
  if (!x || !rot_table || !out_q || !out_scale || K <= 0 || M < 0) return PARO_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(x_dtype)) return PARO_ERR_UNSUPPORTED;
  if (krot != 8 || group != 128) return PARO_ERR_UNSUPPORTED;  // Rotation supports only these (rotation_linear.py:18-19)
  if (K % group) return PARO_ERR_SHAPE;
  if (K > rotq_max_k()) return PARO_ERR_TOO_LARGE;
  if (!aligned(x, x_dtype == PARO_F32 ? 4 : 2) || (scales && !aligned(scales, 2)) || !aligned(rot_table, 4))
    return PARO_ERR_MISALIGNED;
  if (M == 0) return PARO_OK;
  if (int d = device_check()) return d;
  return cuda_status(
      launch_rotq(x_dtype, x, M, K, scales, rot_table, fp16_round ? 1 : 0, out_q, out_scale, (cudaStream_t)stream));
}

size_t paro_rotq_int8_workspace_size(int64_t M, int K, int fp16_round) {
  if (M < rotq_rows_min_m() || K <= 0 || K % kGroup || !fp16_round) return 0;
  return rotq_rows_workspace(M, K);
}

int paro_rotq_int8_ws(const void* x, int x_dtype, int64_t M, int K, const uint16_t* scales,
                      const uint32_t* rot_table, int krot, int group, int fp16_round, int8_t* out_q,
                      float* out_scale, void* workspace, size_t workspace_bytes, paro_stream_t stream) {
  const size_t need = paro_rotq_int8_workspace_size(M, K, fp16_round);
  if (need == 0)
    return paro_rotq_int8(x, x_dtype, M, K, scales, rot_table, krot, group, fp16_round, out_q, out_scale, stream);
  if (!x || !rot_table || !out_q || !out_scale) return PARO_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(x_dtype)) return PARO_ERR_UNSUPPORTED;
  if (krot != 8 || group != 128) return PARO_ERR_UNSUPPORTED;
  if (!aligned(x, x_dtype == PARO_F32 ? 4 : 2) || (scales && !aligned(scales, 2)) || !aligned(rot_table, 4))
    return PARO_ERR_MISALIGNED;
  if (!workspace || workspace_bytes < need) return PARO_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return PARO_ERR_MISALIGNED;
  if (int d = device_check()) return d;
  return cuda_status(launch_rotq_rows(x_dtype, x, M, K, scales, rot_table, out_q, out_scale, workspace,
                                      (cudaStream_t)stream));
}

int paro_quant_int8(const void* x, int x_dtype, int64_t M, int K, int8_t* out_q, float* out_scale,
                    paro_stream_t stream) {
  if (M == 0 && K > 0) return PARO_OK;
  if (!x || !out_q || !out_scale || K <= 0 || M < 0) return PARO_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(x_dtype)) return PARO_ERR_UNSUPPORTED;
  if (M == 0) return PARO_OK;
  if (int d = device_check()) return d;
  return cuda_status(launch_quant(x_dtype, x, M, K, out_q, out_scale, (cudaStream_t)stream));
}

size_t paro_packed_weight_bytes(int N, int K) {
  if (N <= 0 || K <= 0 || N % kRecRows || K % kGroup) return 0;
  return (size_t)(N / kRecRows) * (K / kGroup) * kRecBytes;
}

int paro_prepare_weights(const int16_t* qweight, const uint16_t* scales, const uint16_t* scaled_zeros, int N, int K,
                         int G_pad, void* packed, paro_stream_t stream) {
  if (!qweight || !scales || !scaled_zeros || !packed || N <= 0 || K <= 0) return PARO_ERR_INVALID_ARGUMENT;
  if (N % kRecRows || K % kGroup || G_pad < K / kGroup) return PARO_ERR_SHAPE;
  if (!aligned(packed, 16)) return PARO_ERR_MISALIGNED;
  if (int d = device_check()) return d;
  return cuda_status(launch_prepare_wq(qweight, scales, scaled_zeros, N, K, packed, (cudaStream_t)stream));
}

int paro_prepare_weights_awq(const int32_t* awq_qweight, const uint16_t* awq_scales, const int32_t* awq_qzeros, int N,
                             int K, void* packed, paro_stream_t stream) {
  if (!awq_qweight || !awq_scales || !awq_qzeros || !packed || N <= 0 || K <= 0) return PARO_ERR_INVALID_ARGUMENT;
  if (N % kRecRows || K % kGroup) return PARO_ERR_SHAPE;
  if (!aligned(packed, 16)) return PARO_ERR_MISALIGNED;
  if (int d = device_check()) return d;
  return cuda_status(launch_prepare_awq(awq_qweight, awq_scales, awq_qzeros, N, K, packed, (cudaStream_t)stream));
}

int paro_w4a8_gemm_path(int64_t M, int N, int K) { return gemm_tc_supported(M, N, K) ? 1 : 0; }

size_t paro_w4a8_gemm_workspace_size(int64_t M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0 || N % kRecRows || K % kGroup) return 0;
  return gemm_tc_supported(M, N, K) ? gemm_tc_workspace(M, N, K) : gemm_decode_workspace(M, N);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// one rotated W4A8 linear (activation + GEMM)
// ---------------------------------------------------------------------------
namespace {
constexpr int64_t kLinearFusedMaxM = 64;
size_t al256(size_t b) { return (b + 255) & ~(size_t)255; }
// scratch of the two-kernel route: int8 rows, token scales, activation workspace
size_t linear_unfused_scratch(int64_t M, int K, int fp16_round) {
  return al256((size_t)M * K) + al256((size_t)M * sizeof(float)) + paro_rotq_int8_workspace_size(M, K, fp16_round);
}
}  // namespace

extern "C" {

size_t paro_w4a8_linear_workspace_size(int64_t M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0 || N % kRecRows || K % kGroup) return 0;
  size_t ws = paro_w4a8_gemm_workspace_size(M, N, K);
  if (M <= kLinearFusedMaxM) ws = std::max(ws, linear_decode_workspace(M, N, K, 1));
  return ws;
}

size_t paro_w4a8_linear_scratch_size(int64_t M, int N, int K, int fp16_round) {
  if (M <= 0 || N <= 0 || K <= 0 || N % kRecRows || K % kGroup) return 0;
  size_t sc = linear_unfused_scratch(M, K, fp16_round);
  if (M <= kLinearFusedMaxM) sc = std::max(sc, linear_decode_scratch(M, K, 1));
  return sc;
}

int paro_w4a8_linear(const void* x, int x_dtype, int64_t M, int K, int N, const uint16_t* channel_scales,
                     const uint32_t* rot_table, int fp16_round, const void* packed, const void* bias, int bias_dtype,
                     void* out, int out_dtype, void* workspace, size_t workspace_bytes, void* scratch,
                     size_t scratch_bytes, paro_stream_t stream) {
  if (M == 0 && N > 0 && K > 0) return PARO_OK;
  if (!x || !rot_table || !packed || !out || M < 0 || N <= 0 || K <= 0) return PARO_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(x_dtype) || !valid_dtype(out_dtype) || (bias && !valid_dtype(bias_dtype)))
    return PARO_ERR_UNSUPPORTED;
  if (N % kRecRows || K % kGroup) return PARO_ERR_SHAPE;
  if (!aligned(x, x_dtype == PARO_F32 ? 4 : 2) || (channel_scales && !aligned(channel_scales, 2)) ||
      !aligned(rot_table, 4) || !aligned(packed, 16))
    return PARO_ERR_MISALIGNED;
  if (workspace_bytes < paro_w4a8_linear_workspace_size(M, N, K) ||
      scratch_bytes < paro_w4a8_linear_scratch_size(M, N, K, fp16_round) || !workspace || !scratch)
    return PARO_ERR_WORKSPACE;
  if (!aligned(workspace, 256) || !aligned(scratch, 256)) return PARO_ERR_MISALIGNED;
  if (int d = device_check()) return d;
  cudaStream_t st = (cudaStream_t)stream;
  // decode sizes: rotation kernel + quantiser + GEMM, chained by
  // programmatic dependent launch (measured on B200 faster than the
  // activation kernel + GEMM pair, whose single-pass activation kernel
  // spreads a row over one 8-CTA cluster)
  if (M <= kLinearFusedMaxM && fp16_round) {
    const cudaError_t e = launch_linear_decode(x, x_dtype, channel_scales, rot_table, M, N, K, packed, bias,
                                               bias_dtype, out, out_dtype, workspace, scratch, kProNone, RotPro{},
                                               st);
    if (e != cudaErrorNotSupported) return cuda_status(e);
  }
  // two kernels: activation into the scratch, then the GEMM
  uint8_t* sp = static_cast<uint8_t*>(scratch);
  int8_t* xq = reinterpret_cast<int8_t*>(sp);
  float* xs = reinterpret_cast<float*>(sp + al256((size_t)M * K));
  void* aws = sp + al256((size_t)M * K) + al256((size_t)M * sizeof(float));
  const size_t aws_bytes = paro_rotq_int8_workspace_size(M, K, fp16_round);
  int rc = paro_rotq_int8_ws(x, x_dtype, M, K, channel_scales, rot_table, 8, kGroup, fp16_round, xq, xs,
                             aws_bytes ? aws : nullptr, aws_bytes, stream);
  if (rc != PARO_OK) return rc;
  return paro_w4a8_gemm(xq, xs, M, N, K, packed, bias, bias_dtype, out, out_dtype, workspace, workspace_bytes,
                        stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// one rotated linear with the decoder-layer step before it fused in
// ---------------------------------------------------------------------------
namespace {
bool overlaps(const void* a, size_t an, const void* b, size_t bn) {
  const uintptr_t pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b);
  return pa < pb + bn && pb < pa + an;
}
}  // namespace

extern "C" {

size_t paro_w4a8_linear_prologue_scratch_size(int prologue, int64_t M, int N, int K, int fp16_round) {
  if (prologue < PARO_PROLOGUE_NONE || prologue > PARO_PROLOGUE_SILU_MUL) return 0;
  const size_t lin = paro_w4a8_linear_scratch_size(M, N, K, fp16_round);
  if (!lin) return 0;
  // the unfused route (prefill sizes) keeps the prologue's bf16 output
  return prologue == PARO_PROLOGUE_NONE ? lin : al256((size_t)M * K * 2) + lin;
}

int paro_w4a8_linear_prologue(int prologue, const void* x, const void* residual_in, void* residual_out,
                              const void* norm_weight, float eps, int64_t M, int K, int N,
                              const uint16_t* channel_scales, const uint32_t* rot_table, int fp16_round,
                              const void* packed, const void* bias, int bias_dtype, void* out, int out_dtype,
                              void* workspace, size_t workspace_bytes, void* scratch, size_t scratch_bytes,
                              paro_stream_t stream) {
  if (prologue == PARO_PROLOGUE_NONE)
    return paro_w4a8_linear(x, PARO_BF16, M, K, N, channel_scales, rot_table, fp16_round, packed, bias, bias_dtype,
                            out, out_dtype, workspace, workspace_bytes, scratch, scratch_bytes, stream);
  if (prologue != PARO_PROLOGUE_ADD_RMSNORM && prologue != PARO_PROLOGUE_SILU_MUL) return PARO_ERR_UNSUPPORTED;
  if (M == 0 && N > 0 && K > 0) return PARO_OK;
  if (!x || !rot_table || !packed || !out || M < 0 || N <= 0 || K <= 0) return PARO_ERR_INVALID_ARGUMENT;
  const bool rms = prologue == PARO_PROLOGUE_ADD_RMSNORM;
  if (rms && (!residual_out || !norm_weight)) return PARO_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(out_dtype) || (bias && !valid_dtype(bias_dtype))) return PARO_ERR_UNSUPPORTED;
  if (N % kRecRows || K % kGroup) return PARO_ERR_SHAPE;
  if (!aligned(x, 16) || (rms && (!aligned(norm_weight, 16) || !aligned(residual_out, 16))) ||
      (residual_in && !aligned(residual_in, 16)) || (channel_scales && !aligned(channel_scales, 2)) ||
      !aligned(rot_table, 4) || !aligned(packed, 16))
    return PARO_ERR_MISALIGNED;
  const size_t row_bytes = (size_t)M * K * 2;
  // every CTA of a row reads the whole input row while others write their
  // channels of the residual output: the two must be separate buffers
  if (rms && (overlaps(residual_out, row_bytes, x, row_bytes) ||
              (residual_in && overlaps(residual_out, row_bytes, residual_in, row_bytes))))
    return PARO_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < paro_w4a8_linear_workspace_size(M, N, K) ||
      scratch_bytes < paro_w4a8_linear_prologue_scratch_size(prologue, M, N, K, fp16_round) || !workspace ||
      !scratch)
    return PARO_ERR_WORKSPACE;
  if (!aligned(workspace, 256) || !aligned(scratch, 256)) return PARO_ERR_MISALIGNED;
  if (int d = device_check()) return d;
  cudaStream_t st = (cudaStream_t)stream;
  if (M <= kLinearFusedMaxM && fp16_round) {
    RotPro pro{};
    pro.res_in = static_cast<const __nv_bfloat16*>(residual_in);
    pro.res_out = static_cast<__nv_bfloat16*>(residual_out);
    pro.w = static_cast<const __nv_bfloat16*>(norm_weight);
    pro.eps = eps;
    const cudaError_t e =
        launch_linear_decode(x, PARO_BF16, channel_scales, rot_table, M, N, K, packed, bias, bias_dtype, out, out_dtype,
                             workspace, scratch, rms ? kProAddRmsnorm : kProSiluMul, pro, st);
    if (e != cudaErrorNotSupported) return cuda_status(e);
  }
  // prefill sizes: the prologue's own kernel into the scratch, then the linear
  uint8_t* h = static_cast<uint8_t*>(scratch);
  cudaError_t e;
  if (rms) {
    // the separate kernel updates the residual in place: copy it over first
    const void* src = residual_in ? residual_in : x;
    e = cudaMemcpyAsync(residual_out, src, row_bytes, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_status(e);
    e = launch_add_rmsnorm(residual_in ? x : residual_out, residual_in ? residual_out : nullptr, norm_weight, M, K,
                           eps, h, st);
  } else {
    e = launch_silu_mul(x, M, K, h, st);
  }
  if (e != cudaSuccess) return cuda_status(e);
  return paro_w4a8_linear(h, PARO_BF16, M, K, N, channel_scales, rot_table, fp16_round, packed, bias, bias_dtype, out,
                          out_dtype, workspace, workspace_bytes, h + al256(row_bytes), scratch_bytes - al256(row_bytes),
                          stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// a group of rotated linears sharing their input, one rotation table each
// ---------------------------------------------------------------------------
namespace {
size_t elem_bytes(int dtype) { return dtype == PARO_F32 ? 4 : 2; }

int group_check(int T, const int* n_per_table, int K, int* n_total, int* nb_start) {
  if (T < 1 || T > kMaxTables || !n_per_table) return PARO_ERR_INVALID_ARGUMENT;
  int n = 0;
  for (int t = 0; t < T; ++t) {
    if (n_per_table[t] <= 0) return PARO_ERR_INVALID_ARGUMENT;
    if (n_per_table[t] % kRecRows) return PARO_ERR_SHAPE;
    nb_start[t] = n / kRecRows;
    n += n_per_table[t];
  }
  if (K <= 0 || K % kGroup) return PARO_ERR_SHAPE;
  *n_total = n;
  return PARO_OK;
}
}  // namespace

extern "C" {

size_t paro_w4a8_linear_group_workspace_size(int64_t M, int T, const int* n_per_table, int K) {
  int nt = 0, nb[kMaxTables];
  if (M <= 0 || group_check(T, n_per_table, K, &nt, nb)) return 0;
  size_t ws = M <= kLinearFusedMaxM ? linear_decode_workspace(M, nt, K, T) : 0;
  if (gemm_tc_supported(M, nt, K)) ws = std::max(ws, gemm_tc_workspace(M, nt, K));
  for (int t = 0; t < T; ++t) ws = std::max(ws, paro_w4a8_linear_workspace_size(M, n_per_table[t], K));
  return ws;
}

size_t paro_w4a8_linear_group_scratch_size(int prologue, int64_t M, int T, const int* n_per_table, int K,
                                           int fp16_round) {
  int nt = 0, nb[kMaxTables];
  if (M <= 0 || group_check(T, n_per_table, K, &nt, nb)) return 0;
  if (prologue < PARO_PROLOGUE_NONE || prologue > PARO_PROLOGUE_SILU_MUL) return 0;
  size_t sc = M <= kLinearFusedMaxM && fp16_round ? linear_decode_scratch(M, K, T) : 0;
  // per-table route: the prologue's output, one table's output in fp32 and
  // that linear's scratch
  size_t per = 0;
  for (int t = 0; t < T; ++t)
    per = std::max(per, al256((size_t)M * n_per_table[t] * 4) +
                            paro_w4a8_linear_scratch_size(M, n_per_table[t], K, fp16_round));
  // prefill route with every table on a 256-row tile: T activation sets,
  // then one tensor-core GEMM
  const size_t sets = al256((size_t)T * M * K) + al256((size_t)T * M * 4) + paro_rotq_int8_workspace_size(M, K, fp16_round);
  per = std::max(per, sets);
  per += prologue == PARO_PROLOGUE_NONE ? 0 : al256((size_t)M * K * 2);
  return std::max(sc, per);
}

int paro_w4a8_linear_group(int prologue, const void* x, int x_dtype, const void* residual_in, void* residual_out,
                           const void* norm_weight, float eps, int64_t M, int K, int T, const int* n_per_table,
                           const uint16_t* const* channel_scales, const uint32_t* const* rot_tables, int fp16_round,
                           const void* packed, const void* bias, int bias_dtype, void* out, int out_dtype,
                           void* workspace, size_t workspace_bytes, void* scratch, size_t scratch_bytes,
                           paro_stream_t stream) {
  int N = 0, nb[kMaxTables];
  if (int rc = group_check(T, n_per_table, K, &N, nb)) return rc;
  if (prologue < PARO_PROLOGUE_NONE || prologue > PARO_PROLOGUE_SILU_MUL) return PARO_ERR_UNSUPPORTED;
  if (M == 0) return PARO_OK;
  if (!x || !rot_tables || !packed || !out || M < 0) return PARO_ERR_INVALID_ARGUMENT;
  for (int t = 0; t < T; ++t) {
    if (!rot_tables[t]) return PARO_ERR_INVALID_ARGUMENT;
    if (!aligned(rot_tables[t], 4) || (channel_scales && channel_scales[t] && !aligned(channel_scales[t], 2)))
      return PARO_ERR_MISALIGNED;
  }
  const bool rms = prologue == PARO_PROLOGUE_ADD_RMSNORM;
  if (!valid_dtype(x_dtype) || !valid_dtype(out_dtype) || (bias && !valid_dtype(bias_dtype)))
    return PARO_ERR_UNSUPPORTED;
  if (prologue != PARO_PROLOGUE_NONE && x_dtype != PARO_BF16) return PARO_ERR_UNSUPPORTED;
  if (rms && (!residual_out || !norm_weight)) return PARO_ERR_INVALID_ARGUMENT;
  const size_t row_bytes = (size_t)M * K * 2;
  if (rms && (overlaps(residual_out, row_bytes, x, row_bytes) ||
              (residual_in && overlaps(residual_out, row_bytes, residual_in, row_bytes))))
    return PARO_ERR_INVALID_ARGUMENT;
  if (!aligned(x, 16) || !aligned(packed, 16) || !aligned(out, 16) || (residual_in && !aligned(residual_in, 16)) ||
      (rms && (!aligned(residual_out, 16) || !aligned(norm_weight, 16))))
    return PARO_ERR_MISALIGNED;
  if (!workspace || !scratch || workspace_bytes < paro_w4a8_linear_group_workspace_size(M, T, n_per_table, K) ||
      scratch_bytes < paro_w4a8_linear_group_scratch_size(prologue, M, T, n_per_table, K, fp16_round))
    return PARO_ERR_WORKSPACE;
  if (!aligned(workspace, 256) || !aligned(scratch, 256)) return PARO_ERR_MISALIGNED;
  if (int d = device_check()) return d;
  cudaStream_t st = (cudaStream_t)stream;
  RotPro pro{};
  if (rms) {
    pro.res_in = static_cast<const __nv_bfloat16*>(residual_in);
    pro.res_out = static_cast<__nv_bfloat16*>(residual_out);
    pro.w = static_cast<const __nv_bfloat16*>(norm_weight);
    pro.eps = eps;
  }
  if (M <= kLinearFusedMaxM && fp16_round) {
    // one rotation kernel and one quantiser over all T tables, one GEMM over
    // the concatenated weights
    RotTables tabs = {};
    for (int t = 0; t < T; ++t) {
      tabs.rtab[t] = rot_tables[t];
      tabs.cs[t] = channel_scales ? channel_scales[t] : nullptr;
    }
    const int pk = prologue == PARO_PROLOGUE_NONE ? kProNone : rms ? kProAddRmsnorm : kProSiluMul;
    const cudaError_t e = launch_linear_decode_tables(x, x_dtype, tabs, T, nb, M, N, K, packed, bias, bias_dtype,
                                                      out, out_dtype, workspace, scratch, pk, pro, st);
    if (e != cudaErrorNotSupported) return cuda_status(e);
  }
  // otherwise one linear per table into the scratch, copied into its columns
  uint8_t* sp = static_cast<uint8_t*>(scratch);
  const void* xin = x;
  int xdt = x_dtype;
  if (prologue != PARO_PROLOGUE_NONE) {
    cudaError_t e;
    if (rms) {
      const void* src = residual_in ? residual_in : x;
      e = cudaMemcpyAsync(residual_out, src, row_bytes, cudaMemcpyDeviceToDevice, st);
      if (e != cudaSuccess) return cuda_status(e);
      e = launch_add_rmsnorm(residual_in ? x : residual_out, residual_in ? residual_out : nullptr, norm_weight, M, K,
                             eps, sp, st);
    } else {
      e = launch_silu_mul(x, M, K, sp, st);
    }
    if (e != cudaSuccess) return cuda_status(e);
    xin = sp;
    xdt = PARO_BF16;
    sp += al256(row_bytes);
  }
  if (gemm_tc_supported(M, N, K) && gemm_tc_sets_ok(T, nb) && aligned(out, 16)) {
    // every table starts on a 256-row tile: one activation set per table,
    // then one tensor-core GEMM over the concatenated weights
    int8_t* xq = reinterpret_cast<int8_t*>(sp);
    float* xs = reinterpret_cast<float*>(sp + al256((size_t)T * M * K));
    uint8_t* aws = sp + al256((size_t)T * M * K) + al256((size_t)T * M * 4);
    const size_t awb = paro_rotq_int8_workspace_size(M, K, fp16_round);
    for (int t = 0; t < T; ++t) {
      const int rc = paro_rotq_int8_ws(xin, xdt, M, K, channel_scales ? channel_scales[t] : nullptr, rot_tables[t], 8,
                                       kGroup, fp16_round, xq + (size_t)t * M * K, xs + (size_t)t * M,
                                       awb ? aws : nullptr, awb, stream);
      if (rc != PARO_OK) return rc;
    }
    const size_t tcb = gemm_tc_workspace(M, N, K);
    return cuda_status(launch_gemm_tc_sets(xq, xs, M, N, K, packed, bias, bias_dtype, out, out_dtype,
                                           tcb ? workspace : nullptr, tcb, T, nb, st));
  }
  const size_t rec_bytes_per_nb = (size_t)(K / kGroup) * kRecBytes;
  const size_t oe = elem_bytes(out_dtype);
  for (int t = 0; t < T; ++t) {
    const int nt = n_per_table[t], n0 = nb[t] * kRecRows;
    const size_t tmp_bytes = al256((size_t)M * nt * 4);
    const uint8_t* pk = static_cast<const uint8_t*>(packed) + (size_t)nb[t] * rec_bytes_per_nb;
    const void* bt = bias ? static_cast<const uint8_t*>(bias) + (size_t)n0 * elem_bytes(bias_dtype) : nullptr;
    int rc = paro_w4a8_linear(xin, xdt, M, K, nt, channel_scales ? channel_scales[t] : nullptr, rot_tables[t],
                              fp16_round, pk, bt, bias_dtype, sp, out_dtype, workspace, workspace_bytes,
                              sp + tmp_bytes, scratch_bytes - (size_t)(sp - static_cast<uint8_t*>(scratch)) - tmp_bytes,
                              stream);
    if (rc != PARO_OK) return rc;
    const cudaError_t e = cudaMemcpy2DAsync(static_cast<uint8_t*>(out) + (size_t)n0 * oe, (size_t)N * oe, sp,
                                            (size_t)nt * oe, (size_t)nt * oe, (size_t)M, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_status(e);
  }
  return PARO_OK;
}

}  // extern "C"

extern "C" {

int paro_add_rmsnorm(const void* x, void* residual, const void* weight, int64_t M, int K, float eps, void* out,
                     paro_stream_t stream) {
  if (M == 0 && K > 0) return PARO_OK;
  if (!x || !weight || !out || M < 0 || K <= 0) return PARO_ERR_INVALID_ARGUMENT;
  if (K % 8) return PARO_ERR_SHAPE;
  if (!aligned(x, 16) || !aligned(weight, 16) || !aligned(out, 16) || (residual && !aligned(residual, 16)))
    return PARO_ERR_MISALIGNED;
  if (int d = device_check()) return d;
  return cuda_status(launch_add_rmsnorm(x, residual, weight, M, K, eps, out, (cudaStream_t)stream));
}

int paro_silu_mul(const void* x, int64_t M, int I, void* out, paro_stream_t stream) {
  if (M == 0 && I > 0) return PARO_OK;
  if (!x || !out || M < 0 || I <= 0) return PARO_ERR_INVALID_ARGUMENT;
  if (I % 8) return PARO_ERR_SHAPE;
  if (!aligned(x, 16) || !aligned(out, 16)) return PARO_ERR_MISALIGNED;
  if (int d = device_check()) return d;
  return cuda_status(launch_silu_mul(x, M, I, out, (cudaStream_t)stream));
}

int paro_device_error_word(int clear) {
  const uint32_t a = error_word_decode(clear), b = error_word_tc(clear), c = error_word_rtc(clear),
                 d = error_word_rows(clear);
  if (a == ~0u || b == ~0u || c == ~0u || d == ~0u) return -1;
  return (int)(a | b | c | d);
}

int paro_selftest_wait_timeout(long long limit_cycles, paro_stream_t stream) {
  if (limit_cycles < 1 || limit_cycles > 2000000000LL) return PARO_ERR_INVALID_ARGUMENT;
  if (int d = device_check()) return d;
  return cuda_status(launch_selftest_wait(limit_cycles, (cudaStream_t)stream));
}

int paro_w4a8_gemm(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                   const void* bias, int bias_dtype, void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                   paro_stream_t stream) {
  if (M == 0 && N > 0 && K > 0) return PARO_OK;
  if (!xq || !xscale || !packed || !out || M < 0 || N <= 0 || K <= 0) return PARO_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(out_dtype) || (bias && !valid_dtype(bias_dtype))) return PARO_ERR_UNSUPPORTED;
  if (N % kRecRows || K % kGroup) return PARO_ERR_SHAPE;
  if (!aligned(packed, 16) || !aligned(xq, 16)) return PARO_ERR_MISALIGNED;
  if (M == 0) return PARO_OK;
  if (int d = device_check()) return d;
  if (gemm_tc_supported(M, N, K)) {
    if (!aligned(out, 16)) return PARO_ERR_MISALIGNED;
    if (workspace_bytes < gemm_tc_workspace(M, N, K) || (gemm_tc_workspace(M, N, K) && !workspace))
      return PARO_ERR_WORKSPACE;
    return cuda_status(launch_gemm_tc(xq, xscale, M, N, K, packed, bias, bias_dtype, out, out_dtype, workspace,
                                      workspace_bytes, (cudaStream_t)stream));
  }
  const size_t need = gemm_decode_workspace(M, N);
  if (!workspace || workspace_bytes < need) return PARO_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return PARO_ERR_MISALIGNED;
  return cuda_status(launch_gemm_decode(xq, xscale, M, N, K, packed, bias, bias_dtype, out, out_dtype, workspace,
                                        (cudaStream_t)stream));
}

int paro_w4a8_gemm_multicast(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                             const void* bias, int bias_dtype, void* out_multicast, paro_stream_t stream) {
  if (M == 0 && N > 0 && K > 0) return PARO_OK;
  if (!xq || !xscale || !packed || !out_multicast || M < 0 || N <= 0 || K <= 0) return PARO_ERR_INVALID_ARGUMENT;
  if (bias && !valid_dtype(bias_dtype)) return PARO_ERR_UNSUPPORTED;
  if (N % kRecRows || K % kGroup) return PARO_ERR_SHAPE;
  if (!aligned(packed, 16) || !aligned(xq, 16) || !aligned(out_multicast, 16)) return PARO_ERR_MISALIGNED;
  if (int d = device_check()) return d;
  const int nb0 = 0;
  return cuda_status(launch_gemm_tc_tile(xq, xscale, M, N, K, packed, bias, bias_dtype, out_multicast, PARO_BF16,
                                         nullptr, 0, 1, &nb0, 0, (cudaStream_t)stream, nullptr, 0, 1));
}

// tokens the streaming decode kernel is built and tuned for
constexpr int64_t kStreamMaxTokens = 64;
// ... and the one-row-block-per-warp decode kernel
constexpr int64_t kRowsMaxTokens = 16;

size_t paro_w4a8_gemm_route_workspace_size(int route, int64_t M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0 || N % kRecRows || K % kGroup) return 0;
  switch (route) {
    case PARO_ROUTE_AUTO: return paro_w4a8_gemm_workspace_size(M, N, K);
    case PARO_ROUTE_STREAM: return M <= kStreamMaxTokens ? gemm_decode_workspace(M, N) : 0;
    case PARO_ROUTE_ROWS: return M <= kRowsMaxTokens ? gemm_decode_workspace(M, N) : 0;
    case PARO_ROUTE_TC256: return gemm_tc_workspace_tile(M, N, K, 256);
    case PARO_ROUTE_TC64: return gemm_tc_workspace_tile(M, N, K, 64);
  }
  return 0;
}

int paro_w4a8_gemm_route(int route, const int8_t* xq, const float* xscale, int64_t M, int N, int K,
                         const void* packed, const void* bias, int bias_dtype, void* out, int out_dtype,
                         void* workspace, size_t workspace_bytes, paro_stream_t stream) {
  if (route == PARO_ROUTE_AUTO)
    return paro_w4a8_gemm(xq, xscale, M, N, K, packed, bias, bias_dtype, out, out_dtype, workspace,
                          workspace_bytes, stream);
  if (route != PARO_ROUTE_STREAM && route != PARO_ROUTE_TC256 && route != PARO_ROUTE_TC64 && route != PARO_ROUTE_ROWS)
    return PARO_ERR_INVALID_ARGUMENT;
  if (M == 0 && N > 0 && K > 0) return PARO_OK;
  if (!xq || !xscale || !packed || !out || M < 0 || N <= 0 || K <= 0) return PARO_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(out_dtype) || (bias && !valid_dtype(bias_dtype))) return PARO_ERR_UNSUPPORTED;
  if (N % kRecRows || K % kGroup) return PARO_ERR_SHAPE;
  if (!aligned(packed, 16) || !aligned(xq, 16)) return PARO_ERR_MISALIGNED;
  if (int d = device_check()) return d;
  if (route == PARO_ROUTE_ROWS) {
    if (M > kRowsMaxTokens) return PARO_ERR_TOO_LARGE;
    const size_t need = gemm_decode_workspace(M, N);
    if (!workspace || workspace_bytes < need) return PARO_ERR_WORKSPACE;
    if (!aligned(workspace, 256)) return PARO_ERR_MISALIGNED;
    const cudaError_t e = launch_gemm_rows(xq, xscale, M, N, K, packed, bias, bias_dtype, out, out_dtype, workspace,
                                           nullptr, nullptr, 0, (cudaStream_t)stream, 1);
    return e == cudaErrorNotSupported ? PARO_ERR_UNSUPPORTED : cuda_status(e);
  }
  if (route == PARO_ROUTE_STREAM) {
    if (M > kStreamMaxTokens) return PARO_ERR_TOO_LARGE;
    const size_t need = gemm_decode_workspace(M, N);
    if (!workspace || workspace_bytes < need) return PARO_ERR_WORKSPACE;
    if (!aligned(workspace, 256)) return PARO_ERR_MISALIGNED;
    return cuda_status(launch_gemm_decode(xq, xscale, M, N, K, packed, bias, bias_dtype, out, out_dtype, workspace,
                                          (cudaStream_t)stream));
  }
  const int bt = route == PARO_ROUTE_TC64 ? 64 : 256;
  if (!aligned(out, 16)) return PARO_ERR_MISALIGNED;
  const size_t need = gemm_tc_workspace_tile(M, N, K, bt);
  if (workspace_bytes < need || (need && !workspace)) return PARO_ERR_WORKSPACE;
  const int nb0 = 0;
  return cuda_status(launch_gemm_tc_tile(xq, xscale, M, N, K, packed, bias, bias_dtype, out, out_dtype, workspace,
                                         workspace_bytes, 1, &nb0, bt, (cudaStream_t)stream, nullptr, 0, 0));
}

}  // extern "C"

// ---------------------------------------------------------------------------
// paro_w4a8_gemm_noalloc: the GEMM with its scratch in a fixed array compiled
// into this library, for callers that may not allocate device memory.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_noalloc_scratch[PARO_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoallocMaxDevices];  // device address of the array, per device

// Set-up, once per device and with that device current: look up the array's
// device address.  Nothing is allocated.
int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoallocMaxDevices) return PARO_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e);
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return PARO_OK;
}
}  // namespace

extern "C" {

int paro_w4a8_gemm_noalloc(const int8_t* xq, const float* xscale, int64_t M, int N, int K, const void* packed,
                           const void* bias, int bias_dtype, void* out, int out_dtype, paro_stream_t stream) {
  if (M == 0 && N > 0 && K > 0) return PARO_OK;
  if (!xq || !xscale || !packed || !out || M < 0 || N <= 0 || K <= 0) return PARO_ERR_INVALID_ARGUMENT;
  if (!valid_dtype(out_dtype) || (bias && !valid_dtype(bias_dtype))) return PARO_ERR_UNSUPPORTED;
  if (N % kRecRows || K % kGroup) return PARO_ERR_SHAPE;
  if (!aligned(packed, 16) || !aligned(xq, 16)) return PARO_ERR_MISALIGNED;
  if (int d = device_check()) return d;
  if (gemm_tc_supported(M, N, K)) {
    if (!aligned(out, 16)) return PARO_ERR_MISALIGNED;
    // split-K partial sums go to the fixed array when they fit (the same
    // kernel and splits as paro_w4a8_gemm, so the same bits); beyond the
    // array the kernel runs unsplit, which needs no scratch
    const size_t tcb = gemm_tc_workspace(M, N, K);
    void* tws = nullptr;
    if (tcb && tcb <= (size_t)PARO_NOALLOC_SCRATCH_BYTES) {
      if (int st = noalloc_scratch(&tws)) return st;
      const cudaError_t e = cudaMemsetAsync(tws, 0, tcb, (cudaStream_t)stream);
      if (e != cudaSuccess) return cuda_status(e);
    }
    return cuda_status(launch_gemm_tc(xq, xscale, M, N, K, packed, bias, bias_dtype, out, out_dtype, tws,
                                      tws ? tcb : 0, (cudaStream_t)stream));
  }
  const size_t need = gemm_decode_workspace(M, N);
  if (need > (size_t)PARO_NOALLOC_SCRATCH_BYTES) return PARO_ERR_TOO_LARGE;
  void* scratch = nullptr;
  if (int st = noalloc_scratch(&scratch)) return st;
  // the decode kernel expects a zero-filled workspace; the array holds
  // whatever the previous call left, so clear the part this call uses
  cudaError_t e = cudaMemsetAsync(scratch, 0, need, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_status(e);
  return cuda_status(launch_gemm_decode(xq, xscale, M, N, K, packed, bias, bias_dtype, out, out_dtype, scratch,
                                        (cudaStream_t)stream));
}

}  // extern "C"
