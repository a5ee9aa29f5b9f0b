/*
 * paro_b200.h — C ABI of the B200 (sm_100a) ParoQuant W4A8 rotated-linear
 * kernels.
 *
 * Every entry point takes raw device pointers, sizes and a CUDA stream,
 * launches asynchronously on that stream, never synchronises, never
 * allocates, and returns a paro_status code (0 = success).  Outputs are
 * written only on success.  No torch types appear here: the torch operator
 * shim (alpamayo_b200/csrc/torch_ops.cpp) and any FFI binding (ctypes, cgo,
 * JNI) call these functions directly.
 *
 * Reference interfaces replaced (paths relative to the reference project):
 *   rotation::rotate            kernels/paroquant_kernels/src/rotation.cu:456-493,576-584
 *   rotation::rotate_and_quant  kernels/paroquant_kernels/src/rotation.cu:495-536 (the
 *                               build's fused quantiser is per-token int8, the format
 *                               the W4A8 path consumes, not NVFP4)
 *   per_token_quant_int8        vllm/model_executor/layers/quantization/utils/int8_utils.py:131-156
 *   marlin_gemm (uint4 x int8)  vllm/_custom_ops.py:1277-1318 via
 *                               src/alpamayo_r1/utils/quantization/paroquant_marlin_w4a8.py:314-333
 *   WQLinear -> Marlin repack   src/alpamayo_r1/utils/quantization/paroquant_marlin_w4a8.py:95-209,274-312
 */
#ifndef PARO_B200_H_
#define PARO_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t; NULL means the legacy default stream. */
typedef struct CUstream_st* paro_stream_t;

typedef enum paro_status {
  PARO_OK = 0,
  PARO_ERR_INVALID_ARGUMENT = 1, /* null pointer where one is required, size <= 0   */
  PARO_ERR_SHAPE = 2,            /* K % group != 0, N % 16 != 0, ...                */
  PARO_ERR_UNSUPPORTED = 3,      /* krot / group / dtype combination not built      */
  PARO_ERR_MISALIGNED = 4,       /* pointer not aligned as the entry point requires */
  PARO_ERR_CUDA = 5,             /* a CUDA runtime call or launch failed            */
  PARO_ERR_WORKSPACE = 6,        /* workspace smaller than *_workspace_size()       */
  PARO_ERR_DEVICE = 7,           /* current device is not sm_100                    */
  PARO_ERR_TOO_LARGE = 8         /* size beyond a compiled limit                    */
} paro_status;

typedef enum paro_dtype {
  PARO_F32 = 0,
  PARO_F16 = 1,
  PARO_BF16 = 2
} paro_dtype;

/* Human-readable name of a status code (static storage). */
const char* paro_status_string(int status);

/* Library ABI version (major * 100 + minor). */
int paro_version(void);

/* Last CUDA error string seen by the library on this thread ("" if none). */
const char* paro_last_cuda_error(void);

/* ------------------------------------------------------------------------
 * Rotation tables
 * ------------------------------------------------------------------------ */

/*
 * Validate the Givens pair table and build the per-channel rotation table
 * the fused activation kernel reads.
 *   pairs     : int16 [krot, K] group-local channel indices; entries 2p, 2p+1
 *               of each group form pair p (reference layout,
 *               rotation_linear.py:32-44, read by rotation.cuh:280-297).
 *   theta     : fp16 [krot, K/2] angle of each pair.
 *   out_table : uint32 [krot, K] indexed by channel: partner channel (bits
 *               0-6, group-local), role (bit 7: 0 = first element of its
 *               pair, 1 = second), a shared-memory exchange slot (bits 8-14:
 *               a permutation of the group's channels under which each
 *               32-channel warp's writes and its partners' reads fall in 32
 *               different banks) and the pair's fp16 angle bits (16-31).
 *   bad       : device int32, set to the number of (layer, group) blocks that
 *               are not a permutation of 0..group-1 (must be zero before the
 *               table is trusted: overlapping pairs make a layer
 *               order-dependent and leave table entries unwritten).
 * group must be 128 (Rotation supports only krot 8 / group 128,
 * rotation_linear.py:18-19; any krot is accepted here).  The reference has no
 * validator; this guards the disjointness invariant rotation.cu:48-54 relies on.
 */
int paro_prepare_rotation(const int16_t* pairs, const uint16_t* theta, int krot, int K,
                          int group, uint32_t* out_table, int32_t* bad,
                          paro_stream_t stream);

/*
 * Words of a rotation table for K channels: 8·K (krot 8, group 128), or
 * 136·K with with_matrices = 1.  0 when K is not a positive multiple of 128.
 */
size_t paro_rotation_table_words(int K, int with_matrices);

/*
 * Load-time, optional: extends a krot-8, group-128 table with each group's
 * 128 x 128 rotation matrix (the eight Givens layers applied to the unit
 * vectors, fp32, channel scales not included), so that the prefill
 * activation path (paro_rotq_int8_ws and the linears from
 * paro_rotq_int8_workspace_size tokens on, bf16 x) loads the matrix instead
 * of building it in every CTA.  Every result is bit-identical with and
 * without the matrices; the decode path ignores them.  The reference builds
 * nothing ahead of time (its rotate kernel applies the layers one by one,
 * rotation.cuh:280-334).
 *   table : uint32 [136, K], 16-byte aligned; rows 0-7 from
 *           paro_prepare_rotation (krot 8), rows 8-135 written here.  Bit 15
 *           of word 0 (which paro_prepare_rotation never sets) is set to mark
 *           the table as carrying the matrices: a table so marked must be
 *           136·K words long.
 */
int paro_prepare_rotation_matrices(uint32_t* table, int K, paro_stream_t stream);

/* ------------------------------------------------------------------------
 * Activation kernels
 * ------------------------------------------------------------------------ */

/*
 * rotation::rotate (rotation.cu:456-493): out = R_krot...R_1 (x * scales)
 * per group, float32 math, stored in x's dtype.
 *   x, out       : [M, K] of x_dtype (F32 / F16 / BF16), row-major.
 *   scales       : [K] of param_dtype or NULL (no scaling).
 *   theta        : [krot, K/2] of param_dtype.
 *   pairs        : int16 [krot, K].
 *   krot in {1,2,4,8,16}, group in {64,128}.
 */
int paro_rotate(const void* x, int x_dtype, int64_t M, int K,
                const void* scales, const void* theta, int param_dtype,
                const int16_t* pairs, int krot, int group,
                void* out, paro_stream_t stream);

/*
 * Fused channel scale + Givens rotation + per-token symmetric int8
 * quantisation: the activation half of one W4A8 linear, replacing
 * rotation::rotate (rotation.cu:15-60) followed by per_token_quant_int8
 * (int8_utils.py:106-128).
 *   x            : [M, K] of x_dtype (F32 / F16 / BF16).
 *   scales       : fp16 [K] channel scales or NULL.
 *   rot_table    : uint32 [krot, K] from paro_prepare_rotation (or [136, K]
 *                  with paro_prepare_rotation_matrices).
 *   fp16_round   : 1 = round the rotated value to fp16 before quantising,
 *                  as the reference does (its rotate kernel stores fp16,
 *                  rotation.cuh:333-334); 0 = quantise the float32 value.
 *   out_q        : int8 [M, K];  out_scale : float32 [M] (= absmax / 127).
 */
int paro_rotq_int8(const void* x, int x_dtype, int64_t M, int K,
                   const uint16_t* scales, const uint32_t* rot_table, int krot,
                   int group, int fp16_round, int8_t* out_q, float* out_scale,
                   paro_stream_t stream);

/*
 * paro_rotq_int8 for many tokens: from paro_rotq_int8_workspace_size(M, K,
 * fp16_round) > 0 tokens on (prefill sizes, fp16_round = 1), a two-pass path
 * (rotation into an fp16 workspace with per-row maxima, then quantisation)
 * that keeps the GPU busy where the single-pass cluster kernel cannot; the
 * codes match paro_rotq_int8's within the code tolerance (rare 1-step
 * differences from packed float arithmetic).  Below that size, or
 * with a size of 0, it is paro_rotq_int8.
 *   workspace : at least paro_rotq_int8_workspace_size(...) bytes (about
 *               2 * M * K), 256-byte aligned; no initial contents required.
 *               Calls that may run concurrently need separate workspaces.
 */
size_t paro_rotq_int8_workspace_size(int64_t M, int K, int fp16_round);

int paro_rotq_int8_ws(const void* x, int x_dtype, int64_t M, int K,
                      const uint16_t* scales, const uint32_t* rot_table, int krot,
                      int group, int fp16_round, int8_t* out_q, float* out_scale,
                      void* workspace, size_t workspace_bytes, paro_stream_t stream);

/*
 * per_token_quant_int8 (int8_utils.py:131-156): absmax = max(max|x|, 1e-10),
 * scale = absmax / 127, q = round_half_away(x * (127 / absmax)).
 *   x : [M, K] of x_dtype;  out_q : int8 [M, K];  out_scale : float32 [M].
 */
int paro_quant_int8(const void* x, int x_dtype, int64_t M, int K,
                    int8_t* out_q, float* out_scale, paro_stream_t stream);

/* ------------------------------------------------------------------------
 * Weights
 * ------------------------------------------------------------------------ */

/*
 * Size in bytes of the packed weight buffer for an N x K layer.  The layout
 * ("tile records"): for each block of 16 output rows and each 128-channel
 * group one 1072-byte record = 16 rows x 64 bytes of int4 codes, then the
 * 16 fp16 group scales, then the 16 uint8 zero points.
 */
size_t paro_packed_weight_bytes(int N, int K);

/*
 * WQLinear checkpoint buffers -> packed tile records.
 *   qweight       : int16 [N/4, K] (qmodule.py:39-78 layout).
 *   scales        : fp16 [G_pad, N];  scaled_zeros : fp16 [G_pad, N] (= -s*z),
 *                   G_pad >= K/128 (qmodule.py:123-142).
 *   zero points are recovered as clamp(round(-sz / s), 0, 15) with |s| < 1e-10
 *   treated as 1 (paroquant_marlin_w4a8.py:197-204).
 *   packed        : paro_packed_weight_bytes(N, K) bytes, 16-byte aligned.
 * Requires N % 16 == 0, K % 128 == 0.
 */
int paro_prepare_weights(const int16_t* qweight, const uint16_t* scales,
                         const uint16_t* scaled_zeros, int N, int K, int G_pad,
                         void* packed, paro_stream_t stream);

/*
 * AWQ int32 buffers (the input of MarlinW4A8Linear.load_from_awq,
 * paroquant_marlin_w4a8.py:274-312) -> packed tile records.
 *   awq_qweight : int32 [K, N/8], nibble order [0,2,4,6,1,3,5,7] (:149-164).
 *   awq_scales  : fp16 [K/128, N];  awq_qzeros : int32 [K/128, N/8].
 */
int paro_prepare_weights_awq(const int32_t* awq_qweight, const uint16_t* awq_scales,
                             const int32_t* awq_qzeros, int N, int K,
                             void* packed, paro_stream_t stream);

/* ------------------------------------------------------------------------
 * The int4 x int8 GEMM
 * ------------------------------------------------------------------------ */

/*
 * y[m, n] = xscale[m] * sum_g s[g, n] * sum_{k in g} (q[k, n] - z[g, n]) * xq[m, k]
 *           (+ bias[n]),
 * int32-exact per 128-channel group, float32 across groups, stored in
 * out_dtype (F16 / BF16 / F32).  Replaces marlin_gemm as called by
 * apply_awq_marlin_linear (vllm/.../marlin_utils.py:577-630).
 *   xq        : int8 [M, K];  xscale : float32 [M].
 *   packed    : tile records from paro_prepare_weights*.
 *   bias      : [N] of bias_dtype (F16 / BF16 / F32) or NULL.
 *   out       : [M, N] of out_dtype.
 *   workspace : at least paro_w4a8_gemm_workspace_size(M, N, K) bytes,
 *               256-byte aligned, ZERO-FILLED before its first use.  Every
 *               call leaves it zero-filled again (the kernels clear what they
 *               use), so one buffer serves all calls on one stream; calls that
 *               may run concurrently need separate workspaces.
 * Requires N % 16 == 0, K % 128 == 0, M >= 1.  From 24 tokens (13 for
 * K >= 8192, 17 for layers with at least 0.8 x SMs 256-row tiles), and
 * always above 64, the tensor-core kernel runs (paro_w4a8_gemm_path), with
 * 64-token tiles up to 64 tokens and the tile its cost estimate prefers
 * beyond; it writes `out` with 16-byte stores, so `out` must then be
 * 16-byte aligned.
 */
size_t paro_w4a8_gemm_workspace_size(int64_t M, int N, int K);

int paro_w4a8_gemm(const int8_t* xq, const float* xscale, int64_t M, int N, int K,
                   const void* packed, const void* bias, int bias_dtype,
                   void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                   paro_stream_t stream);

/* ------------------------------------------------------------------------
 * Decoder-layer glue (bf16), used by the decoder-stack benchmark
 * ------------------------------------------------------------------------ */

/*
 * Residual add + Qwen3VLTextRMSNorm (src/alpamayo_r1/models/qwen3_vl/
 * modeling_qwen3_vl.py:340-357): if residual is not NULL it becomes
 * bf16(x + residual) and is normalised; otherwise x is.  out = bf16(weight *
 * bf16(s * rsqrt(mean(s^2) + eps))), float32 math.  All bf16 [M, K] / [K],
 * K % 8 == 0, 16-byte aligned.
 */
int paro_add_rmsnorm(const void* x, void* residual, const void* weight, int64_t M, int K,
                     float eps, void* out, paro_stream_t stream);

/* SiLU(gate) * up on a fused gate_up output: x bf16 [M, 2I] (gate columns
 * first), out bf16 [M, I] = bf16(bf16(silu(gate)) * up).  I % 8 == 0. */
int paro_silu_mul(const void* x, int64_t M, int I, void* out, paro_stream_t stream);

/* Error bits kernels raise instead of hanging (1 = a pipeline wait timed
 * out, 2 = tensor-memory allocation failed, 4 = a wait for the other CTAs of
 * the same launch timed out); synchronises with the device to
 * read them.  clear != 0 resets the word.  Returns -1 if it cannot be read.
 *
 * Recovery: a kernel whose wait ran out stops where it was, so the outputs
 * of the calls made since the last clean read are invalid, and the
 * workspaces those calls used (paro_w4a8_gemm, paro_w4a8_linear) may hold
 * partial sums or unit counters of an unfinished cross-CTA fix-up.  After a
 * non-zero word, zero-fill every such workspace again before its next use
 * (the torch operators do this for the workspaces they own when
 * alpamayo_b200.ops.device_error_word() sees a non-zero word). */
int paro_device_error_word(int clear);

/* Diagnostics (no counterpart in the reference, which has no bounded
 * waits): launches one thread that waits, through the same bounded
 * mbarrier wait every pipelined kernel here uses, on a barrier nothing
 * arrives on, with a limit of limit_cycles SM clocks (1 .. 2e9).  No copy
 * is in flight, so the wait runs out, sets bit 1 of the device error word
 * and the kernel returns; the context stays usable.  Lets a deployment
 * check that its error polling sees a timed-out wait without breaking
 * anything. */
int paro_selftest_wait_timeout(long long limit_cycles, paro_stream_t stream);

/*
 * One rotated W4A8 linear: y = paro_w4a8_gemm(paro_rotq_int8(x)), the whole
 * forward of RotateLinearInt4 / BF16RotateLinearWrapper
 * (src/alpamayo_r1/utils/quantization/paroquant_marlin_w4a8.py:47-71 with
 * rotation_linear.py:53-139).  Up to 64 tokens with fp16_round = 1 it is
 * three chained kernels: one rotates the activations into the scratch
 * (fp16, one CTA per (128-channel group, token)) and records each row's
 * |max|, one quantises the rows to int8, and the GEMM (the streaming kernel,
 * launched behind them with programmatic dependent launch so that its weight
 * stream starts early; or, where paro_w4a8_gemm_path picks it, the
 * tensor-core kernel with 64-token tiles).  Otherwise it is the activation kernel(s)
 * followed by the GEMM.
 *   x             : [M, K] of x_dtype;  channel_scales : fp16 [K] or NULL.
 *   rot_table     : uint32 [8, K] from paro_prepare_rotation (group 128), or
 *                   [136, K] with paro_prepare_rotation_matrices.
 *   workspace     : paro_w4a8_linear_workspace_size(M, N, K) bytes, 256-byte
 *                   aligned, ZERO-FILLED before first use and left zero-filled
 *                   by every call (as paro_w4a8_gemm's).
 *   scratch       : paro_w4a8_linear_scratch_size(M, N, K, fp16_round) bytes,
 *                   256-byte aligned, no initial contents required.
 * Calls that may run concurrently need separate workspaces and scratches.
 */
size_t paro_w4a8_linear_workspace_size(int64_t M, int N, int K);
size_t paro_w4a8_linear_scratch_size(int64_t M, int N, int K, int fp16_round);

int paro_w4a8_linear(const void* x, int x_dtype, int64_t M, int K, int N,
                     const uint16_t* channel_scales, const uint32_t* rot_table, int fp16_round,
                     const void* packed, const void* bias, int bias_dtype,
                     void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                     void* scratch, size_t scratch_bytes, paro_stream_t stream);

/*
 * paro_w4a8_linear with the decoder-layer step in front of it fused into
 * the activation kernel: the residual add + Qwen3VLTextRMSNorm before qkv
 * and gate_up (src/alpamayo_r1/models/qwen3_vl/modeling_qwen3_vl.py:340-357,
 * the decoder layer's `residual + hidden_states`), or SiLU(gate) * up before
 * down (src/alpamayo_r1/utils/system/patches.py:540-547,
 * `down_proj(act_fn(gate) * up)`).
 *   PARO_PROLOGUE_ADD_RMSNORM: x bf16 [M, K]; residual_in bf16 [M, K] or
 *     NULL; residual_out bf16 [M, K] receives bf16(x + residual_in) (x when
 *     NULL) and must not overlap x or residual_in; norm_weight bf16 [K]; the
 *     linear's input is bf16(w * bf16(s * rsqrt(mean(s^2) + eps))).
 *   PARO_PROLOGUE_SILU_MUL: x bf16 [M, 2K], gate columns first; the linear's
 *     input is bf16(bf16(silu(gate)) * up).  residual_* / norm_weight unused.
 *   PARO_PROLOGUE_NONE: paro_w4a8_linear on bf16 x.
 * Up to 64 tokens (fp16_round = 1) the step runs inside the rotation kernel
 * (one kernel fewer per linear; same bits as the separate kernels:
 * paro_add_rmsnorm / paro_silu_mul, then paro_w4a8_linear); above, the
 * separate kernel writes into the scratch and the linear follows.  16-byte
 * aligned bf16 buffers; other arguments as paro_w4a8_linear, with
 * scratch_bytes >= paro_w4a8_linear_prologue_scratch_size().
 */
typedef enum paro_prologue {
  PARO_PROLOGUE_NONE = 0,
  PARO_PROLOGUE_ADD_RMSNORM = 1,
  PARO_PROLOGUE_SILU_MUL = 2
} paro_prologue;

size_t paro_w4a8_linear_prologue_scratch_size(int prologue, int64_t M, int N, int K, int fp16_round);

int paro_w4a8_linear_prologue(int prologue, const void* x, const void* residual_in, void* residual_out,
                              const void* norm_weight, float eps, int64_t M, int K, int N,
                              const uint16_t* channel_scales, const uint32_t* rot_table, int fp16_round,
                              const void* packed, const void* bias, int bias_dtype,
                              void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                              void* scratch, size_t scratch_bytes, paro_stream_t stream);

/*
 * A group of T (1..4) rotated linears that read the same input, each with
 * its own rotation: q / k / v after input_layernorm, gate / up after
 * post_attention_layernorm, as a real checkpoint holds them (the reference
 * loads them unfused, each its own RotateLinearInt4 with its own tables:
 * src/alpamayo_r1/utils/quantization/paroquant_marlin_w4a8.py:455-460).
 * y = [linear_0(x) | linear_1(x) | ...], the fused-projection layout
 * (patches.py:144-263).
 *   n_per_table   : host array of T output widths (each a multiple of 16).
 *   rot_tables    : host array of T device tables from paro_prepare_rotation
 *                   (each [8, K], or [136, K] with the matrices).
 *   channel_scales: host array of T device fp16 [K] pointers (entries may be
 *                   NULL), or NULL.
 *   packed        : the T layers' tile records concatenated (records are
 *                   row-block major, so this is their byte concatenation).
 *   bias          : [sum n] of bias_dtype or NULL;  out : [M, sum n].
 *   prologue      : as paro_w4a8_linear_prologue (x bf16 for the fused
 *                   steps; the residual output is written once).
 * Up to 64 tokens (fp16_round = 1): one rotation kernel and one quantiser
 * for all T tables (the table index is a grid dimension) and one GEMM over
 * the concatenated weights, each row block reading its table's activations.
 * Otherwise one paro_w4a8_linear per table into the scratch, copied into its
 * columns of out.  Workspace (zero-filled, left so) and scratch as sized.
 */
size_t paro_w4a8_linear_group_workspace_size(int64_t M, int T, const int* n_per_table, int K);
size_t paro_w4a8_linear_group_scratch_size(int prologue, int64_t M, int T, const int* n_per_table, int K,
                                           int fp16_round);
int paro_w4a8_linear_group(int prologue, const void* x, int x_dtype, const void* residual_in, void* residual_out,
                           const void* norm_weight, float eps, int64_t M, int K, int T, const int* n_per_table,
                           const uint16_t* const* channel_scales, const uint32_t* const* rot_tables,
                           int fp16_round, const void* packed, const void* bias, int bias_dtype,
                           void* out, int out_dtype, void* workspace, size_t workspace_bytes,
                           void* scratch, size_t scratch_bytes, paro_stream_t stream);

/* Which GEMM kernel paro_w4a8_gemm would launch for this shape
 * (0 = streaming decode kernel, 1 = tcgen05 tensor-core kernel). */
int paro_w4a8_gemm_path(int64_t M, int N, int K);

/* ---- GEMM with an explicit kernel (no counterpart in the reference) ------
 * paro_w4a8_gemm with the kernel named instead of picked by shape, for tests
 * that hold the kernels to one another and for measuring where one
 * overtakes another:
 *   PARO_ROUTE_AUTO    the kernel paro_w4a8_gemm picks;
 *   PARO_ROUTE_STREAM  the streaming decode kernel (M <= 64, else
 *                      PARO_ERR_TOO_LARGE);
 *   PARO_ROUTE_TC256   the tensor-core kernel with 256-token tiles;
 *   PARO_ROUTE_TC64    the tensor-core kernel with 64-token tiles;
 *   PARO_ROUTE_ROWS    the decode kernel with one row block per warp (M <= 16,
 *                      else PARO_ERR_TOO_LARGE; PARO_ERR_UNSUPPORTED where its
 *                      shared memory plan does not fit), which no automatic
 *                      choice uses unless the environment sets
 *                      PARO_DECODE_GEMM=rows.
 * The tensor-core routes want `out` 16-byte aligned.  Workspace: at least
 * paro_w4a8_gemm_route_workspace_size(route, M, N, K) bytes, zero-filled
 * before the first call and left zero by every call.  Results of the two
 * tensor-core routes are equal bit for bit when neither splits K (which
 * happens when the shape's tiles fill the GPU's CTA pairs); the int32 group
 * sums are exact on every route, and routes otherwise differ only in the
 * order float32 partial sums are added. */
typedef enum paro_route {
  PARO_ROUTE_AUTO = 0,
  PARO_ROUTE_STREAM = 1,
  PARO_ROUTE_TC256 = 2,
  PARO_ROUTE_TC64 = 3,
  PARO_ROUTE_ROWS = 4
} paro_route;

size_t paro_w4a8_gemm_route_workspace_size(int route, int64_t M, int N, int K);

int paro_w4a8_gemm_route(int route, const int8_t* xq, const float* xscale, int64_t M, int N, int K,
                         const void* packed, const void* bias, int bias_dtype, void* out, int out_dtype,
                         void* workspace, size_t workspace_bytes, paro_stream_t stream);

/* ---- GEMM into every rank's copy of a buffer (no counterpart in the
 * reference) --------------------------------------------------------------
 * The tensor-core GEMM with bf16 output stored through an NVLink multicast
 * address (multimem.st): every GPU whose memory is bound to the multicast
 * object receives the [M, N] result at the same offset, so a column-sharded
 * linear's blocks reach every rank from the GEMM's own epilogue, with no
 * separate gather.  out_multicast: the multicast address of this rank's
 * [M, N] block (16-byte aligned), e.g. a torch symmetric-memory buffer's
 * multicast pointer plus the block's byte offset.  No split-K (no
 * workspace).  The stores are ordered before whatever follows on the stream
 * at system scope; the caller's cross-rank barrier then makes the whole
 * buffer valid on every rank.  Arguments are otherwise those of
 * paro_w4a8_gemm. */
int paro_w4a8_gemm_multicast(const int8_t* xq, const float* xscale, int64_t M, int N, int K,
                             const void* packed, const void* bias, int bias_dtype,
                             void* out_multicast, paro_stream_t stream);

/* ---- Allocation-free GEMM (no counterpart in the reference) --------------
 * paro_w4a8_gemm without a caller-provided workspace, for callers that may
 * not allocate device memory when they run a layer: an engine whose memory
 * pool already owns the whole device, a latency-critical loop that cannot
 * afford cudaMalloc's implicit device-wide synchronisation, or a foreign
 * binding with no device allocator of its own.  It allocates nothing: no
 * cudaMalloc / cudaFree and no allocating library routine.
 *
 * The decode kernel's scratch lives in one fixed array of
 * PARO_NOALLOC_SCRATCH_BYTES compiled into this library (one copy per
 * device).
 *  - Set-up: the first call on a device, with that device current, looks
 *    up the array's device address (cudaGetSymbolAddress).  Make that first
 *    call before any stream capture.
 *  - Limit: a shape uses paro_w4a8_gemm_workspace_size(M, N, K) bytes of
 *    the array (about 8 * M * N where it is not 0).  Shapes for which
 *    paro_w4a8_gemm_path returns 0 (the streaming kernel) and that need
 *    more than PARO_NOALLOC_SCRATCH_BYTES return PARO_ERR_TOO_LARGE and
 *    launch nothing.  Shapes for which it returns 1 (the tensor-core
 *    kernel) always run: with split-K through the array when their size
 *    fits (then bit for bit the result of paro_w4a8_gemm), otherwise
 *    without split-K, which needs no scratch but is slower on small layers
 *    at 65 to about 1,300 tokens and rounds the cross-group sums in float32
 *    instead of 64-bit fixed point (results agree to float32 rounding).
 *  - State: the array keeps whatever the previous call left, so every call
 *    first clears the part it uses (cudaMemsetAsync on `stream`).
 *  - Concurrency: all calls on a device share the one array.  Calls whose
 *    work can overlap on the GPU (different streams with no ordering between
 *    them) race on it and give wrong results; order them on one stream, or
 *    use paro_w4a8_gemm with a workspace per stream.
 * Arguments, results and errors are otherwise those of paro_w4a8_gemm.
 */
#define PARO_NOALLOC_SCRATCH_BYTES (8u << 20)

int paro_w4a8_gemm_noalloc(const int8_t* xq, const float* xscale, int64_t M, int N, int K,
                           const void* packed, const void* bias, int bias_dtype,
                           void* out, int out_dtype, paro_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* PARO_B200_H_ */
