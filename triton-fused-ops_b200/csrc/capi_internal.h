// Internal launch interfaces between the C-ABI layer (capi.cu) and the
// kernel translation units. Nothing here is exported.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <algorithm>
#include <utility>

namespace tfo {

// Records `msg` as this thread's last error (read by tfo_last_error) and returns `code`.
int report_error(int code, const char* msg);

// Counts kernel launches made by this library (reported by tfo_kernel_launches).
void note_launch(int n = 1);

// Device address of the current device's error word (cached per device).
uint32_t* error_word_ptr();
// Number of SMs of the current device (cached per device).
int num_sms();
// cudaOccupancyMaxActiveBlocksPerMultiprocessor, cached per (kernel, block, smem).
int cached_occupancy(const void* kernel, int block, size_t smem);
// Raises the kernel's dynamic shared-memory limit to at least `smem` bytes on
// the current device; the attribute call is made once per (kernel, device, size).
cudaError_t ensure_smem_attr(const void* kernel, size_t smem);
// For a persistent GEMM kernel (`threads` threads, `smem` bytes of dynamic
// shared memory, raised on first use): how many work units can be resident at
// once on the current device, a unit being one CTA (cg == 1) or one cluster of
// two CTAs (cg == 2). Cached per (kernel, smem, cg, device); 0 on error.
int gemm_resident_units(const void* kernel, int threads, size_t smem, int cg);

// Two-CTA (cta_group::2) GEMM tiles are used where they apply unless the
// environment sets TFO_B200_PAIR_MMA=0 (read once per process).
bool pair_mma_enabled();

// Launches a GEMM kernel (`threads` threads) on `grid` CTAs as clusters of
// `cluster` consecutive CTAs (1 = no cluster).
template <typename... KArgs, typename... Args>
cudaError_t launch_gemm_grid(void (*kernel)(KArgs...), int threads, int grid, int cluster, size_t smem,
                             cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (cluster > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = static_cast<unsigned>(cluster);
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  // the kernel's setup may overlap the previous kernel (it waits before touching global memory)
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = 1;
  ++na;
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Launches an ordinary kernel as a programmatic dependent of the previous
// kernel on the stream: it may be scheduled while that kernel runs and must
// execute griddepcontrol.wait before touching global memory.
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kernel)(KArgs...), int grid, int block, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(block));
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Launches a persistent GEMM kernel: `units` work units (see above) of
// `threads` threads, as clusters of two CTAs when cg == 2.
template <typename... KArgs, typename... Args>
cudaError_t launch_gemm_units(void (*kernel)(KArgs...), int threads, int cg, int units, size_t smem,
                              cudaStream_t st, Args&&... args) {
  return launch_gemm_grid(kernel, threads, units * cg, cg, smem, st, std::forward<Args>(args)...);
}

struct RmsNormRopeArgs {
  const void* x;
  const void* weight;
  const void* cos;
  const void* sin;
  void* out;
  int64_t batch, seq_len, hidden, head_dim, num_heads;
  int64_t cs_stride_seq, cs_stride_dim;
  float eps;
  int x_dtype, w_dtype, cos_dtype, sin_dtype;
};
cudaError_t rmsnorm_rope_launch(const RmsNormRopeArgs& a, cudaStream_t st);
// Extra output of the warp-per-row RMSNorm+RoPE kernel for a fused quantize:
// one max |output value| per CTA.
struct RowQuantArgs {
  uint32_t* parts_out;
};
// RMSNorm+RoPE rows to a.out plus one amax partial per CTA to q.parts_out
// (mode 3; *nparts receives their count). Returns cudaErrorNotSupported unless
// tfo_rmsnorm_rope would run its warp-per-row kernel on this shape (same
// kernel, so the rows are bit-identical); the caller then runs the two ops.
cudaError_t rmsnorm_rope_quant_launch(const RmsNormRopeArgs& a, int mode, const RowQuantArgs& q, int* nparts,
                                      cudaStream_t st);
// Upper bound on the amax partials of mode 3 (one per CTA).
int rmsnorm_rope_quant_max_parts();
// Launch choice of tfo_rmsnorm_rope (see rmsnorm_rope_plan in rmsnorm_rope.cu).
struct RmsPlan {
  int kind;     // 0 generic, 1 CTA per row, 2 warp per row
  int threads;  // kind 1: threads per CTA; kind 2: warps (rows) per CTA
  int vec;      // kind 1: 16-byte vectors per thread; kind 2: per lane
  bool full;    // every column belongs to a rotated head
  int cs_stride;
  size_t smem;
};
RmsPlan rmsnorm_rope_plan(int64_t rows, int64_t hidden, int64_t head_dim, int64_t num_heads, int esz, bool vec_ok);

// FP8 codec (fp8_codec.cu)
int amax_partials_count(int64_t n);
cudaError_t amax_partials_launch(const void* x, int64_t n, int x_dtype, uint32_t* partials, int nparts,
                                 cudaStream_t st);
cudaError_t finalize_scale_launch(const uint32_t* partials, int nparts, float* scale_out, cudaStream_t st);
// Encodes x with either a given scale (scale_in) or the dynamic scale reduced
// from `partials` (then scale_out, if non-null, receives it).
cudaError_t encode_launch(const void* x, int64_t n, int x_dtype, const float* scale_in, const uint32_t* partials,
                          int nparts, float* scale_out, void* out, int out_dtype, cudaStream_t st);
cudaError_t dequantize_launch(const void* q, int64_t n, int q_dtype, const float* scale, void* out, int out_dtype,
                              cudaStream_t st);
// Per-row (per-token / per-channel) scales of a [rows, cols] matrix.
cudaError_t row_scales_launch(const void* x, int64_t rows, int64_t cols, int x_dtype, float* scales, cudaStream_t st);
// Per-token dynamic quantize in one launch: scales_out[r] (x's dtype) and the codes of row r.
cudaError_t quantize_rows_dynamic_launch(const void* x, int64_t rows, int64_t cols, int x_dtype, void* scales_out,
                                         void* out, int out_dtype, cudaStream_t st);
cudaError_t encode_rows_launch(const void* x, int64_t rows, int64_t cols, int x_dtype, const float* scales, void* out,
                               int out_dtype, cudaStream_t st);
cudaError_t decode_rows_launch(const void* q, int64_t rows, int64_t cols, int q_dtype, const float* scales, void* out,
                               int out_dtype, cudaStream_t st);
// Workspace of the one-kernel dynamic-scale quantize: a grid-barrier counter
// and the running max at bytes 0-7 (zeroed by quantize_dynamic_launch).
size_t quantize_dynamic_workspace_bytes();
cudaError_t quantize_dynamic_launch(const void* x, int64_t n, int x_dtype, float* scale_out, void* out, int out_dtype,
                                    void* ws, size_t ws_bytes, cudaStream_t st);

// FP8 GEMM (fp8_gemm.cu). b_layout: 0 = [K, N] row-major, 1 = [N, K] row-major.
struct Fp8GemmArgs {
  const void* a;
  const void* b;
  const float* sa;
  const float* sb;
  void* c;
  int64_t M, N, K;
  int ab_dtype, b_layout, out_dtype;
  void* ws;
  size_t ws_bytes;
  // FP8Linear: bias[N] added after rounding the product to round_dtype
  // (< 0: no rounding step), result stored as out_dtype
  const void* bias = nullptr;
  int bias_dtype = -1;
  int round_dtype = -1;
  // per-token / per-channel scales: sa_rows[M] replaces sa, sb_cols[N] replaces sb
  const float* sa_rows = nullptr;
  const float* sb_cols = nullptr;
  // reference codec, B given as [N, K] int8 values u - 128 (a prepared
  // constant weight) with b_s8_sums[n] = their sum over k: A is used raw and
  // no operand is prepared per call
  const int32_t* b_s8_sums = nullptr;
};
// The prepared form of a [rows, K] reference-codec weight: dst = codes ^ 0x80
// (int8 u - 128), sums[r] = the row's sum of those values.
cudaError_t fp8_prepare_rows_launch(const void* codes, int64_t rows, int64_t K, void* dst, int32_t* sums,
                                    cudaStream_t st);
size_t fp8_gemm_workspace_bytes(const Fp8GemmArgs& g);
// Launch choice of tfo_fp8_gemm for 16-byte-aligned operands: out = {rows
// per tile, columns per tile, CTAs per MMA, stages, K splits, group_m}.
void fp8_gemm_tile(int64_t M, int64_t N, int64_t K, int ab_dtype, int b_layout, int32_t out[6]);
// Same for tfo_gated_mlp with 16-bit operands.
void gated_mlp_tile(int64_t M, int64_t N, int64_t K, int32_t out[6]);
cudaError_t fp8_gemm_launch(const Fp8GemmArgs& g, cudaStream_t st);

// Gated MLP (gated_mlp.cu): out[M, N] = (x Wg^T) * act(x Wu^T), x [M, K], W [N, K].
struct GatedMlpArgs {
  const void* x;
  const void* wg;
  const void* wu;
  void* out;
  int64_t M, N, K;
  int x_dtype, w_dtype, act;
  void* ws;
  size_t ws_bytes;
  // 8-bit output (tfo_gated_mlp_quantize): codes of the outputs rounded to x's
  // dtype with the given scale (out may then be NULL), and/or one max |output|
  // per epilogue warp (4 per CTA) to amax_parts
  uint8_t* codes = nullptr;
  const float* scale = nullptr;
  int e4m3 = 0;
  uint32_t* amax_parts = nullptr;
  int* ctas_out = nullptr;  // receives the tcgen05 kernel's CTA count (4 amax partials each)
};
size_t gated_mlp_workspace_bytes(const GatedMlpArgs& g);
cudaError_t gated_mlp_launch(const GatedMlpArgs& g, cudaStream_t st);
// True when gated_mlp_launch runs the tcgen05 kernel (which supports the 8-bit
// output); otherwise it runs the CUDA-core kernel.
bool gated_mlp_tensor_path(const GatedMlpArgs& g);
// Upper bound on the CTAs of the tcgen05 kernel (amax partials: 4 per CTA).
int gated_mlp_max_ctas();
}  // namespace tfo
