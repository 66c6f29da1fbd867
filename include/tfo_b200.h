/*
 * tfo_b200.h — C ABI of the B200 (sm_100a) fused transformer-op library.
 *
 * Every entry point takes raw device pointers, element counts and dtype
 * codes (no framework types), launches on the given CUDA stream (NULL = the
 * legacy default stream), never synchronises the host, and returns a status
 * code. On a non-zero status, tfo_last_error() returns a message for the
 * calling thread. Inputs are read-only; outputs are caller-allocated.
 *
 * Each function names the reference interface it replaces
 * (LessUp/triton-fused-ops, paths inside that project).
 */
#ifndef TFO_B200_H
#define TFO_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TFO_API __attribute__((visibility("default")))
#else
#define TFO_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes */
#define TFO_DTYPE_F16 0
#define TFO_DTYPE_BF16 1
#define TFO_DTYPE_F32 2
#define TFO_DTYPE_U8 3   /* reference 8-bit codec: u = int8(q) + 128 */
#define TFO_DTYPE_E4M3 4 /* float8 e4m3fn bytes */

/* status codes */
#define TFO_OK 0
#define TFO_ERR_INVALID 1 /* bad pointer, size or shape */
#define TFO_ERR_DTYPE 2   /* unsupported dtype combination */
#define TFO_ERR_CUDA 3    /* CUDA runtime error (message has the details) */
#define TFO_ERR_DEVICE 4  /* a kernel recorded a device-side error */

/* gated-MLP activations */
#define TFO_ACT_SILU 0      /* x * sigmoid(x) */
#define TFO_ACT_GELU 1      /* erf form: 0.5 x (1 + erf(x / sqrt 2)) */
#define TFO_ACT_GELU_TANH 2 /* tanh approximation */

/* layout of the B operand of tfo_fp8_gemm */
#define TFO_B_KN 0 /* b is [K, N] row-major (reference fp8_gemm convention) */
#define TFO_B_NK 1 /* b is [N, K] row-major (nn.Linear weight convention) */

/* Library version string. */
TFO_API const char* tfo_version(void);

/* Number of kernels (and memsets) this library has launched in this process,
 * over all devices and threads. No counterpart in the reference. */
TFO_API unsigned long long tfo_kernel_launches(void);

/* Message of the last failing call on this thread ("" if none). */
TFO_API const char* tfo_last_error(void);

/* Synchronises the current device, then reads (and if `clear`, resets) the
 * device error word that kernels set when a bounded wait expires. */
TFO_API int tfo_device_error_flags(uint32_t* flags, int clear);

/* The launch configuration the library picks for a problem shape: the static,
 * shape-keyed table that replaces the reference's autotuner
 * (triton_ops/autotuner/tuner.py; its ops launch fixed block sizes).
 *   op TFO_OP_FP8_GEMM:     M, N, K, aux = TFO_DTYPE_U8 or _E4M3 ([K, N] B,
 *                           16-byte-aligned operands);
 *                           out = {tile rows, tile columns, CTAs per MMA,
 *                           pipeline stages, K splits, group_m}
 *   op TFO_OP_GATED_MLP:    M, N, K (16-bit operands); out as above
 *   op TFO_OP_RMSNORM_ROPE: M = rows, N = hidden, K = head_dim, aux = x dtype
 *                           (16-byte-aligned x/out, heads = hidden / head_dim);
 *                           out = {kernel (0 generic, 1 CTA per row, 2 warp per
 *                           row), threads per CTA or rows per CTA, 16-byte
 *                           vectors per thread or lane, all columns rotated,
 *                           dynamic shared bytes, 0}
 * Writes min(n_out, 6) values. Needs no GPU when the device cannot be
 * queried (148 SMs are assumed). No counterpart in the reference. */
#define TFO_OP_FP8_GEMM 0
#define TFO_OP_GATED_MLP 1
#define TFO_OP_RMSNORM_ROPE 2
TFO_API int tfo_select_tile(int op, int64_t M, int64_t N, int64_t K, int aux, int32_t* out, int n_out);

/* Launches a one-thread kernel that waits on a barrier nothing will complete,
 * giving up after budget_cycles SM cycles (<= 2^32) and setting the
 * wait-timeout bit of the device error word, exactly as a GEMM pipeline wait
 * would. Lets tests exercise the failure path without hanging a GPU.
 * No counterpart in the reference (its kernels have no device-side waits). */
TFO_API int tfo_selftest_bounded_wait(int64_t budget_cycles, void* stream);

/* Fused RMSNorm + rotate-half RoPE over x [batch, seq_len, hidden] (contiguous).
 * weight [hidden]; cos/sin indexed as cos[pos * cs_stride_seq + i * cs_stride_dim]
 * for pos < seq_len, i < head_dim / 2. Columns >= num_heads * head_dim are
 * normalised but not rotated. out has x's shape and dtype.
 * Replaces: triton_ops/kernels/rmsnorm_rope.py:238-302 (fused_rmsnorm_rope)
 * and its kernel :138-235. */
TFO_API int tfo_rmsnorm_rope(const void* x, const void* weight, const void* cos, const void* sin, void* out, int64_t batch,
                     int64_t seq_len, int64_t hidden, int64_t head_dim, int64_t num_heads, int64_t cs_stride_seq,
                     int64_t cs_stride_dim, double eps, int x_dtype, int w_dtype, int cos_dtype, int sin_dtype,
                     void* stream);

/* RMSNorm + RoPE as tfo_rmsnorm_rope, with the output as 8-bit codes
 * (code_dtype TFO_DTYPE_U8: the reference codec; TFO_DTYPE_E4M3): codes and
 * scale equal tfo_fp8_quantize of the tfo_rmsnorm_rope output byte for byte.
 * The rows are written to the workspace and encoded from there. With scale
 * == NULL (dynamic per-tensor scale 448 / max|output|, written to scale_out)
 * the row pass also records one max per CTA when tfo_rmsnorm_rope runs its
 * warp-per-row kernel on the shape (tfo_select_tile(TFO_OP_RMSNORM_ROPE,
 * batch * seq_len, ...) kernel 2, 16-byte-aligned x, one cos/sin dtype), so
 * the encode pass derives the scale without a separate read of the rows.
 * Workspace: tfo_rmsnorm_rope_quantize_workspace_bytes (the rows plus a few
 * KB). No counterpart in the reference: this is the RMSNorm+RoPE -> FP8
 * fusion its roadmap lists for FusedRMSNormRoPE -> FP8Linear chains. */
TFO_API size_t tfo_rmsnorm_rope_quantize_workspace_bytes(int64_t batch, int64_t seq_len, int64_t hidden, int x_dtype);
TFO_API int tfo_rmsnorm_rope_quantize(const void* x, const void* weight, const void* cos, const void* sin, void* codes,
                                      int64_t batch, int64_t seq_len, int64_t hidden, int64_t head_dim,
                                      int64_t num_heads, int64_t cs_stride_seq, int64_t cs_stride_dim, double eps,
                                      int x_dtype, int w_dtype, int cos_dtype, int sin_dtype, const float* scale,
                                      float* scale_out, int code_dtype, void* workspace, size_t workspace_bytes,
                                      void* stream);

/* Bytes of workspace needed by the dynamic-scale codec calls for numel elements. */
TFO_API size_t tfo_fp8_scale_workspace_bytes(int64_t numel);

/* Per-tensor dynamic scale: scale = fp32(448 / double(max|x|)), 1 if max|x| == 0.
 * Writes one fp32 to scale_out (device). No host synchronisation.
 * Replaces: triton_ops/models.py:282-299 (FP8Format.compute_scale). */
TFO_API int tfo_fp8_compute_scale(const void* x, int64_t numel, int x_dtype, float* scale_out, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Quantize numel elements of x (f16/bf16/f32) to out_dtype TFO_DTYPE_U8 (the
 * reference codec, bit-exact) or TFO_DTYPE_E4M3. If `scale` is non-NULL it is
 * used; otherwise the dynamic scale is computed on the device (needs
 * `workspace`) and written to scale_out.
 * Replaces: triton_ops/kernels/fp8_quantize.py:128-173 (quantize_fp8) and
 * :21-59 (quantize_fp8_kernel). */
TFO_API int tfo_fp8_quantize(const void* x, int64_t numel, int x_dtype, const float* scale, float* scale_out, void* out,
                     int out_dtype, void* workspace, size_t workspace_bytes, void* stream);

/* tfo_fp8_quantize with a dynamic scale, for callers that cannot allocate
 * device memory: code running inside another framework's memory pool or a
 * fixed-budget serving process that owns every byte of the GPU, or a plugin
 * whose host has no allocator to lend it. It calls no cudaMalloc, cudaFree or
 * allocating library routine and takes no workspace: its scratch (the per-block
 * amax partials) is a static 16 KiB device array inside this library, which
 * every GPU that loads the library keeps until the process exits. Limit: a
 * call may need at most 4096 partial slots (one per amax block, at most
 * 4 x the SM count, i.e. 592 on a 148-SM B200); larger needs are rejected with
 * TFO_ERR_INVALID and an explanatory message. The first call in each CUDA
 * context (per device, and again after cudaDeviceReset or in another context
 * made current through the driver API) looks up the scratch address in that
 * context, so make it before any stream capture. All
 * calls share the scratch: calls that overlap on the GPU (different streams,
 * same device) race and must be serialised by the caller.
 * No counterpart in the reference; same results as tfo_fp8_quantize with a
 * NULL scale. */
TFO_API int tfo_fp8_quantize_noalloc(const void* x, int64_t numel, int x_dtype, float* scale_out, void* out,
                                     int out_dtype, void* stream);

/* Dequantize numel codes (TFO_DTYPE_U8 reference codec or TFO_DTYPE_E4M3) to
 * out_dtype: out = dec(q) / scale.
 * Replaces: triton_ops/kernels/fp8_quantize.py:176-211 (dequantize_fp8) and
 * :62-98 (dequantize_fp8_kernel). */
TFO_API int tfo_fp8_dequantize(const void* q, int64_t numel, int q_dtype, const float* scale, void* out, int out_dtype,
                       void* stream);

/* Workspace bytes tfo_fp8_gemm needs for these sizes (an upper bound over
 * operand alignments; 0 when the product is empty). */
TFO_API size_t tfo_fp8_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int ab_dtype, int b_layout);

/* C[M, N] = dec(a)[M, K] . dec(b)[K, N] / (a_scale * b_scale) on tcgen05.
 * a: [M, K] row-major codes; b: [K, N] (TFO_B_KN) or [N, K] (TFO_B_NK) codes;
 * both TFO_DTYPE_U8 (reference codec, exact int8 products, int32 accumulation)
 * or both TFO_DTYPE_E4M3 (fp32 accumulation). a_scale / b_scale: one fp32 each
 * on the device. out_dtype: f16 / bf16 / f32. K <= 131072.
 * Replaces: triton_ops/kernels/fp8_gemm.py:123-187 (fp8_gemm) and its kernel
 * :21-120; TFO_B_NK serves FP8Linear (:272-310) without the per-call transpose. */
TFO_API int tfo_fp8_gemm(const void* a, const void* b, const float* a_scale, const float* b_scale, void* c, int64_t M,
                         int64_t N, int64_t K, int ab_dtype, int b_layout, int out_dtype, void* workspace,
                         size_t workspace_bytes, void* stream);

/* Per-token / per-channel scales (extension; the reference's quantize_fp8
 * reads one scale, its FP8Format.compute_scale_per_channel,
 * triton_ops/models.py:301-314, computes per-channel ones in torch):
 * tfo_fp8_compute_scale_rows: scales[r] = 448 / max|x[r, :]| (a zero max
 *   counts as 1) for a contiguous [rows, cols] x, with torch's rounding of
 *   compute_scale_per_channel(x, dim=-1) in x's dtype (reciprocal, then
 *   * 448), stored as fp32;
 * tfo_fp8_quantize_rows / tfo_fp8_dequantize_rows: the per-tensor codec with
 *   scales[r] for row r;
 * tfo_fp8_gemm_scaled: tfo_fp8_gemm with a per-row A scale vector [M]
 *   (a_per_row = 1, else a_scales[0]) and/or a per-column B scale vector [N]
 *   (b_per_col = 1), applied in the epilogue; workspace
 *   tfo_fp8_gemm_scaled_workspace_bytes. */
TFO_API int tfo_fp8_compute_scale_rows(const void* x, int64_t rows, int64_t cols, int x_dtype, float* scales,
                                       void* stream);
TFO_API int tfo_fp8_quantize_rows(const void* x, int64_t rows, int64_t cols, int x_dtype, const float* scales, void* out,
                                  int out_dtype, void* stream);
/* Per-token dynamic quantize in one launch (extension): for a contiguous
 * [rows, cols] x, scales_out[r] (x's dtype) = the value
 * FP8Format.compute_scale_per_channel(x, dim=-1) returns for row r
 * (triton_ops/models.py:301-314: 448 / max|x[r, :]|, a zero max counting as
 * 1, rounded in x's dtype), and out = the codes quantize_fp8(x, scales)
 * produces with those per-row scales (triton_ops/kernels/fp8_quantize.py:
 * 128-173 with a per-row scale): the bytes of tfo_fp8_compute_scale_rows
 * followed by tfo_fp8_quantize_rows, from one read of x. out_dtype: U8 or
 * E4M3. */
TFO_API int tfo_fp8_quantize_per_token(const void* x, int64_t rows, int64_t cols, int x_dtype, void* scales_out,
                                       void* out, int out_dtype, void* stream);
TFO_API int tfo_fp8_dequantize_rows(const void* q, int64_t rows, int64_t cols, int q_dtype, const float* scales,
                                    void* out, int out_dtype, void* stream);
TFO_API size_t tfo_fp8_gemm_scaled_workspace_bytes(int64_t M, int64_t N, int64_t K, int ab_dtype, int b_layout);
TFO_API int tfo_fp8_gemm_scaled(const void* a, const void* b, const float* a_scales, int a_per_row,
                                const float* b_scales, int b_per_col, void* c, int64_t M, int64_t N, int64_t K,
                                int ab_dtype, int b_layout, int out_dtype, void* workspace, size_t workspace_bytes,
                                void* stream);

/* FP8Linear's forward GEMM: out[M, N] = round_to(gemm_dtype)(x_codes @ w_codesᵀ
 * decoded and scaled, as tfo_fp8_gemm with b_layout TFO_B_NK) + bias[N], the sum
 * in fp32 and stored as out_dtype: exactly the reference's
 * `fp8_gemm(..., output_dtype=x.dtype)` followed by `output + self.bias`
 * (triton_ops/kernels/fp8_gemm.py:293-309), with the bias added in the GEMM's
 * epilogue instead of a separate pass. bias == NULL: tfo_fp8_gemm with
 * out_dtype = gemm_dtype. Workspace: tfo_fp8_gemm_workspace_bytes(M, N, K,
 * ab_dtype, TFO_B_NK). No separate counterpart in the reference. */
TFO_API int tfo_fp8_linear(const void* x_codes, const void* w_codes, const float* x_scale, const float* w_scale,
                           const void* bias, int bias_dtype, void* out, int64_t M, int64_t N, int64_t K, int ab_dtype,
                           int gemm_dtype, int out_dtype, void* workspace, size_t workspace_bytes, void* stream);

/* The prepared form of a reference-codec (TFO_DTYPE_U8) weight w_codes[N, K]
 * for tfo_fp8_linear_prepared: w_s8[n, k] = w_codes[n, k] ^ 0x80 (the int8
 * value u - 128, N x K bytes) and w_sums[n] = the sum over k of w_s8[n, :].
 * K % 16 == 0 and all pointers 16-byte aligned. The result stays valid while
 * the weight does: prepare once per weight, not per call.
 * No counterpart in the reference (its fp8_gemm re-reads the uint8 codes on
 * every call). */
TFO_API int tfo_fp8_prepare_weight(const void* w_codes, int64_t N, int64_t K, void* w_s8, int32_t* w_sums,
                                   void* stream);

/* tfo_fp8_linear for reference-codec operands with the weight prepared by
 * tfo_fp8_prepare_weight: the same output bits, with no per-call operand
 * preparation (tfo_fp8_linear sign-flips the smaller operand and sums it on
 * every call, a pass over the weight when M > N). x_codes [M, K] uint8,
 * K % 16 == 0, 16-byte-aligned pointers; bias may be NULL (then out_dtype
 * must equal gemm_dtype). Workspace: tfo_fp8_gemm_workspace_bytes(M, N, K,
 * TFO_DTYPE_U8, TFO_B_NK).
 * Replaces: FP8Linear.forward's GEMM + bias (triton_ops/kernels/fp8_gemm.py:293-309). */
TFO_API int tfo_fp8_linear_prepared(const void* x_codes, const void* w_s8, const int32_t* w_sums,
                                    const float* x_scale, const float* w_scale, const void* bias, int bias_dtype,
                                    void* out, int64_t M, int64_t N, int64_t K, int gemm_dtype, int out_dtype,
                                    void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes tfo_gated_mlp needs (non-zero only when an fp32 copy of an
 * operand is required, i.e. mixed or fp32 dtypes). */
TFO_API size_t tfo_gated_mlp_workspace_bytes(int64_t M, int64_t N, int64_t K, int x_dtype, int w_dtype);

/* out[M, N] = (x . w_gate^T) * act(x . w_up^T), x [M, K], w_gate / w_up [N, K],
 * all row-major; fp32 accumulation; out has x's dtype. activation: TFO_ACT_*.
 * Replaces: triton_ops/kernels/gated_mlp.py:149-218 (fused_gated_mlp) and its
 * kernel :31-146. */
TFO_API int tfo_gated_mlp(const void* x, const void* w_gate, const void* w_up, void* out, int64_t M, int64_t N,
                          int64_t K, int x_dtype, int w_dtype, int activation, void* workspace,
                          size_t workspace_bytes, void* stream);

/* The gated MLP with its output as 8-bit codes (code_dtype TFO_DTYPE_U8: the
 * reference codec; TFO_DTYPE_E4M3) for an FP8 down-projection: codes and scale
 * equal tfo_fp8_quantize of the tfo_gated_mlp output byte for byte. Given
 * scale on the tcgen05 path: the epilogue rounds each output to x's dtype
 * and writes its code directly (no output rows in memory, no encode pass).
 * scale == NULL: the epilogue writes the rows to the workspace and one max
 * per epilogue warp, and the encode pass derives the scale from those (no
 * separate amax read). CUDA-core shapes run the two ops. Workspace:
 * tfo_gated_mlp_quantize_workspace_bytes with the same pointers and
 * has_scale = (scale != NULL). No counterpart in the reference: the MLP ->
 * FP8 down-projection chain of its roadmap. */
TFO_API size_t tfo_gated_mlp_quantize_workspace_bytes(const void* x, const void* w_gate, const void* w_up, int64_t M,
                                                      int64_t N, int64_t K, int x_dtype, int w_dtype, int has_scale);
TFO_API int tfo_gated_mlp_quantize(const void* x, const void* w_gate, const void* w_up, void* codes, int64_t M,
                                   int64_t N, int64_t K, int x_dtype, int w_dtype, int activation, const float* scale,
                                   float* scale_out, int code_dtype, void* workspace, size_t workspace_bytes,
                                   void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TFO_B200_H */
