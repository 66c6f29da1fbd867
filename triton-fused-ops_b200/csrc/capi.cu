// C-ABI layer: argument checks, status/error reporting, device caches and
// dispatch into the kernel translation units.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <string>
#include <tuple>
#include <map>

#include "capi_internal.h"
#include "common.cuh"
#include "tfo_b200.h"

namespace tfo {

__device__ uint32_t g_error_word = 0;

namespace {
thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(TFO_ERR_CUDA, std::string(where) + ": " + cudaGetErrorName(e) + ": " + cudaGetErrorString(e));
}

bool is_float_dtype(int d) { return d == F16 || d == BF16 || d == F32; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

std::mutex g_cache_mu;
std::map<int, int> g_sm_count;
std::map<std::tuple<const void*, int, size_t, int>, int> g_occ;
}  // namespace

int report_error(int code, const char* msg) { return fail(code, msg); }

static std::atomic<unsigned long long> g_launches{0};
void note_launch(int n) { g_launches.fetch_add(static_cast<unsigned long long>(n), std::memory_order_relaxed); }

uint32_t* error_word_ptr() {
  int dev = 0;
  cudaGetDevice(&dev);
  static std::mutex mu;
  static std::map<int, uint32_t*> ptrs;
  std::lock_guard<std::mutex> lk(mu);
  auto it = ptrs.find(dev);
  if (it != ptrs.end()) return it->second;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_error_word) != cudaSuccess) p = nullptr;
  ptrs[dev] = static_cast<uint32_t*>(p);
  return static_cast<uint32_t*>(p);
}

int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_cache_mu);
  auto it = g_sm_count.find(dev);
  if (it != g_sm_count.end()) return it->second;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  g_sm_count[dev] = n;
  return n;
}

int cached_occupancy(const void* kernel, int block, size_t smem) {
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(kernel, block, smem, dev);
  {
    std::lock_guard<std::mutex> lk(g_cache_mu);
    auto it = g_occ.find(key);
    if (it != g_occ.end()) return it->second;
  }
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, block, smem) != cudaSuccess || occ <= 0) occ = 1;
  std::lock_guard<std::mutex> lk(g_cache_mu);
  g_occ[key] = occ;
  return occ;
}

bool pair_mma_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("TFO_B200_PAIR_MMA");
    return !(v != nullptr && v[0] == '0');
  }();
  return on;
}

int gemm_resident_units(const void* kernel, int threads, size_t smem, int cg) {
  int dev = 0;
  cudaGetDevice(&dev);
  static std::mutex mu;
  static std::map<std::tuple<const void*, int, size_t, int, int>, int> cache;
  const auto key = std::make_tuple(kernel, threads, smem, cg, dev);
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
    return 0;
  int units = 0;
  if (cg == 1) {
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, threads, smem) != cudaSuccess) return 0;
    units = occ * num_sms();
  } else {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * num_sms());
    cfg.blockDim = dim3(static_cast<unsigned>(threads));
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&units, kernel, &cfg) != cudaSuccess) return 0;
  }
  cache[key] = units;
  return units;
}

cudaError_t ensure_smem_attr(const void* kernel, size_t smem) {
  if (smem <= 48 * 1024) return cudaSuccess;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> done;
  std::lock_guard<std::mutex> lk(mu);
  size_t& have = done[std::make_pair(kernel, dev)];
  if (have >= smem) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e == cudaSuccess) have = smem;
  return e;
}

size_t scale_workspace_bytes(int64_t numel) {
  return std::max(static_cast<size_t>(amax_partials_count(numel)) * sizeof(uint32_t),
                  quantize_dynamic_workspace_bytes());
}

// Waits on an mbarrier that nothing ever arrives on, with the given cycle
// budget, to exercise the bounded-wait error path end to end.
__global__ void selftest_bounded_wait_kernel(long long budget, uint32_t* err) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const long long t0 = clock64();
    while (!mbar_try_wait(&bar, 0)) {
      if (clock64() - t0 > budget) {
        set_error(err, ERR_WAIT_TIMEOUT_OTHER);
        break;
      }
    }
  }
}

}  // namespace tfo

using namespace tfo;

extern "C" {

unsigned long long tfo_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

const char* tfo_version(void) { return "tfo_b200 0.1.0 (sm_100a)"; }

const char* tfo_last_error(void) { return g_last_error.c_str(); }

int tfo_device_error_flags(uint32_t* flags, int clear) {
  if (flags == nullptr) return fail(TFO_ERR_INVALID, "tfo_device_error_flags: flags is NULL");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "tfo_device_error_flags: synchronize");
  e = cudaMemcpyFromSymbol(flags, g_error_word, sizeof(uint32_t));
  if (e != cudaSuccess) return cuda_fail(e, "tfo_device_error_flags: read");
  if (clear) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(g_error_word, &zero, sizeof(uint32_t));
    if (e != cudaSuccess) return cuda_fail(e, "tfo_device_error_flags: clear");
  }
  return TFO_OK;
}

int tfo_rmsnorm_rope(const void* x, const void* weight, const void* cos, const void* sin, void* out, int64_t batch,
                     int64_t seq_len, int64_t hidden, int64_t head_dim, int64_t num_heads, int64_t cs_stride_seq,
                     int64_t cs_stride_dim, double eps, int x_dtype, int w_dtype, int cos_dtype, int sin_dtype,
                     void* stream) {
  if (!is_float_dtype(x_dtype) || !is_float_dtype(w_dtype) || !is_float_dtype(cos_dtype) ||
      !is_float_dtype(sin_dtype))
    return fail(TFO_ERR_DTYPE, "tfo_rmsnorm_rope: dtypes must be f16, bf16 or f32");
  if (batch < 0 || seq_len < 0 || hidden <= 0 || head_dim <= 0 || num_heads < 0)
    return fail(TFO_ERR_INVALID, "tfo_rmsnorm_rope: negative or zero dimension");
  if (head_dim % 2 != 0) return fail(TFO_ERR_INVALID, "tfo_rmsnorm_rope: head_dim must be even");
  if (num_heads * head_dim > hidden)
    return fail(TFO_ERR_INVALID, "tfo_rmsnorm_rope: num_heads * head_dim exceeds hidden");
  if (hidden > (1 << 20) || seq_len > (1ll << 31) - 1)
    return fail(TFO_ERR_INVALID, "tfo_rmsnorm_rope: hidden or seq_len too large");
  if (batch == 0 || seq_len == 0) return TFO_OK;
  if (!x || !weight || !cos || !sin || !out) return fail(TFO_ERR_INVALID, "tfo_rmsnorm_rope: NULL pointer");
  RmsNormRopeArgs a{x,         weight,    cos,           sin,           out,       batch,
                    seq_len,   hidden,    head_dim,      num_heads,     cs_stride_seq,
                    cs_stride_dim, static_cast<float>(eps), x_dtype, w_dtype,  cos_dtype, sin_dtype};
  cudaError_t e = rmsnorm_rope_launch(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tfo_rmsnorm_rope");
  return TFO_OK;
}

size_t tfo_fp8_scale_workspace_bytes(int64_t numel) { return scale_workspace_bytes(numel); }

size_t tfo_rmsnorm_rope_quantize_workspace_bytes(int64_t batch, int64_t seq_len, int64_t hidden, int x_dtype) {
  // the rows, then the amax partials or the quantize's own workspace
  const int64_t n = std::max<int64_t>(0, batch) * std::max<int64_t>(0, seq_len) * std::max<int64_t>(0, hidden);
  const size_t y_bytes = (static_cast<size_t>(n) * (x_dtype == F32 ? 4 : 2) + 255) / 256 * 256;
  const size_t parts = sizeof(uint32_t) * static_cast<size_t>(rmsnorm_rope_quant_max_parts());
  return y_bytes + std::max(parts, scale_workspace_bytes(n));
}

int tfo_rmsnorm_rope_quantize(const void* x, const void* weight, const void* cos, const void* sin, void* codes,
                              int64_t batch, int64_t seq_len, int64_t hidden, int64_t head_dim, int64_t num_heads,
                              int64_t cs_stride_seq, int64_t cs_stride_dim, double eps, int x_dtype, int w_dtype,
                              int cos_dtype, int sin_dtype, const float* scale, float* scale_out, int code_dtype,
                              void* workspace, size_t workspace_bytes, void* stream) {
  const char* fn = "tfo_rmsnorm_rope_quantize";
  if (!is_float_dtype(x_dtype) || !is_float_dtype(w_dtype) || !is_float_dtype(cos_dtype) ||
      !is_float_dtype(sin_dtype))
    return fail(TFO_ERR_DTYPE, std::string(fn) + ": dtypes must be f16, bf16 or f32");
  if (code_dtype != U8 && code_dtype != E4M3) return fail(TFO_ERR_DTYPE, std::string(fn) + ": codes must be U8 or E4M3");
  if (batch < 0 || seq_len < 0 || hidden <= 0 || head_dim <= 0 || num_heads < 0)
    return fail(TFO_ERR_INVALID, std::string(fn) + ": negative or zero dimension");
  if (head_dim % 2 != 0) return fail(TFO_ERR_INVALID, std::string(fn) + ": head_dim must be even");
  if (num_heads * head_dim > hidden)
    return fail(TFO_ERR_INVALID, std::string(fn) + ": num_heads * head_dim exceeds hidden");
  if (hidden > (1 << 20) || seq_len > (1ll << 31) - 1)
    return fail(TFO_ERR_INVALID, std::string(fn) + ": hidden or seq_len too large");
  if (scale == nullptr && scale_out == nullptr)
    return fail(TFO_ERR_INVALID, std::string(fn) + ": a dynamic scale needs scale_out");
  const int64_t rows = batch * seq_len;
  auto st = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    if (scale != nullptr) return TFO_OK;
    // no elements: the dynamic scale of an empty tensor (1.0), from one zero partial
    if (!workspace || workspace_bytes < sizeof(uint32_t))
      return fail(TFO_ERR_INVALID, std::string(fn) + ": workspace too small");
    uint32_t* parts = static_cast<uint32_t*>(workspace);
    cudaError_t e = amax_partials_launch(x, 0, x_dtype, parts, 1, st);
    if (e == cudaSuccess) e = finalize_scale_launch(parts, 1, scale_out, st);
    return e == cudaSuccess ? TFO_OK : cuda_fail(e, fn);
  }
  if (!x || !weight || !cos || !sin || !codes) return fail(TFO_ERR_INVALID, std::string(fn) + ": NULL pointer");
  if (!workspace || workspace_bytes < tfo_rmsnorm_rope_quantize_workspace_bytes(batch, seq_len, hidden, x_dtype))
    return fail(TFO_ERR_INVALID, std::string(fn) + ": workspace too small");
  // rows in the workspace, then the 8-bit encode of the rows
  const size_t y_bytes = (static_cast<size_t>(rows * hidden) * (x_dtype == F32 ? 4 : 2) + 255) / 256 * 256;
  void* tail = static_cast<char*>(workspace) + y_bytes;
  const size_t tail_bytes = workspace_bytes - y_bytes;
  RmsNormRopeArgs a{x,         weight,    cos,           sin,           workspace, batch,
                    seq_len,   hidden,    head_dim,      num_heads,     cs_stride_seq,
                    cs_stride_dim, static_cast<float>(eps), x_dtype, w_dtype,  cos_dtype, sin_dtype};
  cudaError_t e = cudaErrorNotSupported;
  if (scale == nullptr) {
    // dynamic scale: the row pass also records one max |row value| per CTA,
    // and the encode kernel reduces those to the scale (no separate amax pass)
    RowQuantArgs q{static_cast<uint32_t*>(tail)};
    int nparts = 0;
    e = rmsnorm_rope_quant_launch(a, 3, q, &nparts, st);
    if (e == cudaSuccess)
      e = encode_launch(workspace, rows * hidden, x_dtype, nullptr, q.parts_out, nparts, scale_out, codes, code_dtype,
                        st);
  }
  if (e == cudaErrorNotSupported) {
    (void)cudaGetLastError();
    e = rmsnorm_rope_launch(a, st);
    if (e == cudaSuccess) {
      e = (scale == nullptr)
              ? quantize_dynamic_launch(workspace, rows * hidden, x_dtype, scale_out, codes, code_dtype, tail, tail_bytes,
                                        st)
              : encode_launch(workspace, rows * hidden, x_dtype, scale, nullptr, 0, nullptr, codes, code_dtype, st);
    }
  }
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return TFO_OK;
}



int tfo_select_tile(int op, int64_t M, int64_t N, int64_t K, int aux, int32_t* out, int n_out) {
  if (!out || n_out < 0) return fail(TFO_ERR_INVALID, "tfo_select_tile: NULL output");
  if (M < 0 || N < 0 || K < 0) return fail(TFO_ERR_INVALID, "tfo_select_tile: negative size");
  int32_t v[6] = {0, 0, 0, 0, 0, 0};
  if (op == TFO_OP_FP8_GEMM) {
    if (aux != U8 && aux != E4M3) return fail(TFO_ERR_DTYPE, "tfo_select_tile: fp8_gemm takes U8 or E4M3");
    fp8_gemm_tile(M, N, K, aux, 0, v);
  } else if (op == TFO_OP_GATED_MLP) {
    gated_mlp_tile(M, N, K, v);
  } else if (op == TFO_OP_RMSNORM_ROPE) {
    if (!is_float_dtype(aux)) return fail(TFO_ERR_DTYPE, "tfo_select_tile: rmsnorm_rope x must be f16, bf16 or f32");
    if (K <= 0) return fail(TFO_ERR_INVALID, "tfo_select_tile: head_dim must be positive");
    const RmsPlan p = rmsnorm_rope_plan(M, N, K, N / K, aux == F32 ? 4 : 2, true);
    v[0] = p.kind;
    v[1] = p.threads;
    v[2] = p.vec;
    v[3] = p.full ? 1 : 0;
    v[4] = static_cast<int32_t>(p.smem);
  } else {
    return fail(TFO_ERR_INVALID, "tfo_select_tile: unknown op");
  }
  for (int i = 0; i < std::min(n_out, 6); ++i) out[i] = v[i];
  return TFO_OK;
}

int tfo_fp8_compute_scale(const void* x, int64_t numel, int x_dtype, float* scale_out, void* workspace,
                          size_t workspace_bytes, void* stream) {
  if (!is_float_dtype(x_dtype)) return fail(TFO_ERR_DTYPE, "tfo_fp8_compute_scale: x must be f16, bf16 or f32");
  if (numel < 0) return fail(TFO_ERR_INVALID, "tfo_fp8_compute_scale: negative numel");
  if (!scale_out || (numel > 0 && !x)) return fail(TFO_ERR_INVALID, "tfo_fp8_compute_scale: NULL pointer");
  const int nparts = amax_partials_count(numel);
  if (!workspace || workspace_bytes < static_cast<size_t>(nparts) * sizeof(uint32_t))
    return fail(TFO_ERR_INVALID, "tfo_fp8_compute_scale: workspace too small");
  auto st = static_cast<cudaStream_t>(stream);
  uint32_t* parts = static_cast<uint32_t*>(workspace);
  cudaError_t e = amax_partials_launch(x, numel, x_dtype, parts, nparts, st);
  if (e == cudaSuccess) e = finalize_scale_launch(parts, nparts, scale_out, st);
  if (e != cudaSuccess) return cuda_fail(e, "tfo_fp8_compute_scale");
  return TFO_OK;
}

int tfo_fp8_quantize(const void* x, int64_t numel, int x_dtype, const float* scale, float* scale_out, void* out,
                     int out_dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (!is_float_dtype(x_dtype)) return fail(TFO_ERR_DTYPE, "tfo_fp8_quantize: x must be f16, bf16 or f32");
  if (out_dtype != U8 && out_dtype != E4M3) return fail(TFO_ERR_DTYPE, "tfo_fp8_quantize: out must be U8 or E4M3");
  if (numel < 0) return fail(TFO_ERR_INVALID, "tfo_fp8_quantize: negative numel");
  auto st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  if (scale == nullptr) {
    if (!scale_out) return fail(TFO_ERR_INVALID, "tfo_fp8_quantize: dynamic scale needs scale_out");
    const int nparts = amax_partials_count(numel);
    if (!workspace || workspace_bytes < static_cast<size_t>(nparts) * sizeof(uint32_t))
      return fail(TFO_ERR_INVALID, "tfo_fp8_quantize: workspace too small");
    uint32_t* parts = static_cast<uint32_t*>(workspace);
    if (numel == 0) {
      e = amax_partials_launch(x, 0, x_dtype, parts, nparts, st);
      if (e == cudaSuccess) e = finalize_scale_launch(parts, nparts, scale_out, st);
      if (e != cudaSuccess) return cuda_fail(e, "tfo_fp8_quantize");
      return TFO_OK;
    }
    if (!x || !out) return fail(TFO_ERR_INVALID, "tfo_fp8_quantize: NULL pointer");
    if (workspace_bytes < quantize_dynamic_workspace_bytes())
      return fail(TFO_ERR_INVALID, "tfo_fp8_quantize: workspace too small");
    e = quantize_dynamic_launch(x, numel, x_dtype, scale_out, out, out_dtype, workspace, workspace_bytes, st);
  } else {
    if (numel == 0) return TFO_OK;
    if (!x || !out) return fail(TFO_ERR_INVALID, "tfo_fp8_quantize: NULL pointer");
    e = encode_launch(x, numel, x_dtype, scale, nullptr, 0, nullptr, out, out_dtype, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, "tfo_fp8_quantize");
  return TFO_OK;
}

int tfo_fp8_dequantize(const void* q, int64_t numel, int q_dtype, const float* scale, void* out, int out_dtype,
                       void* stream) {
  if (q_dtype != U8 && q_dtype != E4M3) return fail(TFO_ERR_DTYPE, "tfo_fp8_dequantize: q must be U8 or E4M3");
  if (!is_float_dtype(out_dtype)) return fail(TFO_ERR_DTYPE, "tfo_fp8_dequantize: out must be f16, bf16 or f32");
  if (numel < 0) return fail(TFO_ERR_INVALID, "tfo_fp8_dequantize: negative numel");
  if (numel == 0) return TFO_OK;
  if (!q || !scale || !out) return fail(TFO_ERR_INVALID, "tfo_fp8_dequantize: NULL pointer");
  cudaError_t e = dequantize_launch(q, numel, q_dtype, scale, out, out_dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tfo_fp8_dequantize");
  return TFO_OK;
}

size_t tfo_fp8_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int ab_dtype, int b_layout) {
  Fp8GemmArgs g{};
  g.M = M; g.N = N; g.K = K; g.ab_dtype = ab_dtype; g.b_layout = b_layout;
  return (M <= 0 || N <= 0 || K <= 0) ? 0 : fp8_gemm_workspace_bytes(g);
}

int tfo_fp8_gemm(const void* a, const void* b, const float* a_scale, const float* b_scale, void* c, int64_t M,
                 int64_t N, int64_t K, int ab_dtype, int b_layout, int out_dtype, void* workspace,
                 size_t workspace_bytes, void* stream) {
  if (ab_dtype != U8 && ab_dtype != E4M3) return fail(TFO_ERR_DTYPE, "tfo_fp8_gemm: operands must be U8 or E4M3");
  if (!is_float_dtype(out_dtype)) return fail(TFO_ERR_DTYPE, "tfo_fp8_gemm: output must be f16, bf16 or f32");
  if (b_layout != TFO_B_KN && b_layout != TFO_B_NK) return fail(TFO_ERR_INVALID, "tfo_fp8_gemm: bad b_layout");
  if (M < 0 || N < 0 || K < 0) return fail(TFO_ERR_INVALID, "tfo_fp8_gemm: negative dimension");
  if (M > INT32_MAX || N > INT32_MAX || K > 131072)
    return fail(TFO_ERR_INVALID, "tfo_fp8_gemm: M, N must fit in int32 and K <= 131072 (exact int32 accumulation)");
  if (M == 0 || N == 0) return TFO_OK;
  if (!c || !a_scale || !b_scale) return fail(TFO_ERR_INVALID, "tfo_fp8_gemm: NULL pointer");
  auto st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (K == 0) {
    const size_t esz = out_dtype == F32 ? 4 : 2;
    e = cudaMemsetAsync(c, 0, static_cast<size_t>(M) * N * esz, st);
    note_launch();
    if (e != cudaSuccess) return cuda_fail(e, "tfo_fp8_gemm");
    return TFO_OK;
  }
  if (!a || !b) return fail(TFO_ERR_INVALID, "tfo_fp8_gemm: NULL operand");
  Fp8GemmArgs g{a, b, a_scale, b_scale, c, M, N, K, ab_dtype, b_layout, out_dtype, workspace, workspace_bytes};
  if (workspace_bytes < fp8_gemm_workspace_bytes(g) || !workspace)
    return fail(TFO_ERR_INVALID, "tfo_fp8_gemm: workspace smaller than tfo_fp8_gemm_workspace_bytes()");
  e = fp8_gemm_launch(g, st);
  if (e != cudaSuccess) return cuda_fail(e, "tfo_fp8_gemm");
  return TFO_OK;
}

int tfo_fp8_linear(const void* x_codes, const void* w_codes, const float* x_scale, const float* w_scale,
                   const void* bias, int bias_dtype, void* out, int64_t M, int64_t N, int64_t K, int ab_dtype,
                   int gemm_dtype, int out_dtype, void* workspace, size_t workspace_bytes, void* stream) {
  const char* fn = "tfo_fp8_linear";
  if (bias == nullptr)
    return tfo_fp8_gemm(x_codes, w_codes, x_scale, w_scale, out, M, N, K, ab_dtype, TFO_B_NK, gemm_dtype, workspace,
                        workspace_bytes, stream);
  if (ab_dtype != U8 && ab_dtype != E4M3) return fail(TFO_ERR_DTYPE, std::string(fn) + ": operands must be U8 or E4M3");
  if (!is_float_dtype(gemm_dtype) || !is_float_dtype(out_dtype) || !is_float_dtype(bias_dtype))
    return fail(TFO_ERR_DTYPE, std::string(fn) + ": gemm, bias and output dtypes must be f16, bf16 or f32");
  if (M < 0 || N < 0 || K <= 0) return fail(TFO_ERR_INVALID, std::string(fn) + ": bad dimension (K must be positive)");
  if (M > INT32_MAX || N > INT32_MAX || K > 131072)
    return fail(TFO_ERR_INVALID, std::string(fn) + ": M, N must fit in int32 and K <= 131072");
  if (M == 0 || N == 0) return TFO_OK;
  if (!x_codes || !w_codes || !x_scale || !w_scale || !out) return fail(TFO_ERR_INVALID, std::string(fn) + ": NULL pointer");
  Fp8GemmArgs g{x_codes, w_codes, x_scale, w_scale, out, M, N, K, ab_dtype, TFO_B_NK, out_dtype, workspace,
                workspace_bytes};
  g.bias = bias;
  g.bias_dtype = bias_dtype;
  g.round_dtype = gemm_dtype;
  if (workspace_bytes < fp8_gemm_workspace_bytes(g) || !workspace)
    return fail(TFO_ERR_INVALID, std::string(fn) + ": workspace smaller than tfo_fp8_gemm_workspace_bytes()");
  const cudaError_t e = fp8_gemm_launch(g, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return TFO_OK;
}

int tfo_fp8_prepare_weight(const void* w_codes, int64_t N, int64_t K, void* w_s8, int32_t* w_sums, void* stream) {
  const char* fn = "tfo_fp8_prepare_weight";
  if (N < 0 || K <= 0 || K % 16 != 0) return fail(TFO_ERR_INVALID, std::string(fn) + ": need N >= 0 and K a positive multiple of 16");
  if (N == 0) return TFO_OK;
  if (!w_codes || !w_s8 || !w_sums) return fail(TFO_ERR_INVALID, std::string(fn) + ": NULL pointer");
  if (!aligned16(w_codes) || !aligned16(w_s8)) return fail(TFO_ERR_INVALID, std::string(fn) + ": pointers must be 16-byte aligned");
  const cudaError_t e = fp8_prepare_rows_launch(w_codes, N, K, w_s8, w_sums, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return TFO_OK;
}

int tfo_fp8_linear_prepared(const void* x_codes, const void* w_s8, const int32_t* w_sums, const float* x_scale,
                            const float* w_scale, const void* bias, int bias_dtype, void* out, int64_t M, int64_t N,
                            int64_t K, int gemm_dtype, int out_dtype, void* workspace, size_t workspace_bytes,
                            void* stream) {
  const char* fn = "tfo_fp8_linear_prepared";
  if (!is_float_dtype(gemm_dtype) || !is_float_dtype(out_dtype) || (bias != nullptr && !is_float_dtype(bias_dtype)))
    return fail(TFO_ERR_DTYPE, std::string(fn) + ": gemm, bias and output dtypes must be f16, bf16 or f32");
  if (bias == nullptr && out_dtype != gemm_dtype)
    return fail(TFO_ERR_DTYPE, std::string(fn) + ": without a bias the output dtype is gemm_dtype");
  if (M < 0 || N < 0 || K <= 0 || K % 16 != 0)
    return fail(TFO_ERR_INVALID, std::string(fn) + ": bad dimension (K must be a positive multiple of 16)");
  if (M > INT32_MAX || N > INT32_MAX || K > 131072)
    return fail(TFO_ERR_INVALID, std::string(fn) + ": M, N must fit in int32 and K <= 131072");
  if (M == 0 || N == 0) return TFO_OK;
  if (!x_codes || !w_s8 || !w_sums || !x_scale || !w_scale || !out)
    return fail(TFO_ERR_INVALID, std::string(fn) + ": NULL pointer");
  if (!aligned16(x_codes) || !aligned16(w_s8)) return fail(TFO_ERR_INVALID, std::string(fn) + ": operands must be 16-byte aligned");
  Fp8GemmArgs g{x_codes, w_s8, x_scale, w_scale, out, M, N, K, U8, TFO_B_NK, out_dtype, workspace, workspace_bytes};
  g.bias = bias;
  g.bias_dtype = bias != nullptr ? bias_dtype : -1;
  g.round_dtype = bias != nullptr ? gemm_dtype : -1;
  g.b_s8_sums = w_sums;
  if (workspace_bytes < fp8_gemm_workspace_bytes(g) || !workspace)
    return fail(TFO_ERR_INVALID, std::string(fn) + ": workspace smaller than tfo_fp8_gemm_workspace_bytes()");
  const cudaError_t e = fp8_gemm_launch(g, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return TFO_OK;
}

int tfo_fp8_compute_scale_rows(const void* x, int64_t rows, int64_t cols, int x_dtype, float* scales, void* stream) {
  const char* fn = "tfo_fp8_compute_scale_rows";
  if (!is_float_dtype(x_dtype)) return fail(TFO_ERR_DTYPE, std::string(fn) + ": x must be f16, bf16 or f32");
  if (rows < 0 || cols <= 0) return fail(TFO_ERR_INVALID, std::string(fn) + ": bad shape");
  if (rows == 0) return TFO_OK;
  if (!x || !scales) return fail(TFO_ERR_INVALID, std::string(fn) + ": NULL pointer");
  const cudaError_t e = row_scales_launch(x, rows, cols, x_dtype, scales, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TFO_OK : cuda_fail(e, fn);
}

int tfo_fp8_quantize_rows(const void* x, int64_t rows, int64_t cols, int x_dtype, const float* scales, void* out,
                          int out_dtype, void* stream) {
  const char* fn = "tfo_fp8_quantize_rows";
  if (!is_float_dtype(x_dtype)) return fail(TFO_ERR_DTYPE, std::string(fn) + ": x must be f16, bf16 or f32");
  if (out_dtype != U8 && out_dtype != E4M3) return fail(TFO_ERR_DTYPE, std::string(fn) + ": out must be U8 or E4M3");
  if (rows < 0 || cols <= 0) return fail(TFO_ERR_INVALID, std::string(fn) + ": bad shape");
  if (rows == 0) return TFO_OK;
  if (!x || !scales || !out) return fail(TFO_ERR_INVALID, std::string(fn) + ": NULL pointer");
  const cudaError_t e = encode_rows_launch(x, rows, cols, x_dtype, scales, out, out_dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TFO_OK : cuda_fail(e, fn);
}

int tfo_fp8_quantize_per_token(const void* x, int64_t rows, int64_t cols, int x_dtype, void* scales_out, void* out,
                               int out_dtype, void* stream) {
  const char* fn = "tfo_fp8_quantize_per_token";
  if (!is_float_dtype(x_dtype)) return fail(TFO_ERR_DTYPE, std::string(fn) + ": x must be f16, bf16 or f32");
  if (out_dtype != U8 && out_dtype != E4M3) return fail(TFO_ERR_DTYPE, std::string(fn) + ": out must be U8 or E4M3");
  if (rows < 0 || cols <= 0) return fail(TFO_ERR_INVALID, std::string(fn) + ": bad shape");
  if (rows == 0) return TFO_OK;
  if (!x || !scales_out || !out) return fail(TFO_ERR_INVALID, std::string(fn) + ": NULL pointer");
  const cudaError_t e = quantize_rows_dynamic_launch(x, rows, cols, x_dtype, scales_out, out, out_dtype,
                                                     static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TFO_OK : cuda_fail(e, fn);
}

int tfo_fp8_dequantize_rows(const void* q, int64_t rows, int64_t cols, int q_dtype, const float* scales, void* out,
                            int out_dtype, void* stream) {
  const char* fn = "tfo_fp8_dequantize_rows";
  if (q_dtype != U8 && q_dtype != E4M3) return fail(TFO_ERR_DTYPE, std::string(fn) + ": codes must be U8 or E4M3");
  if (!is_float_dtype(out_dtype)) return fail(TFO_ERR_DTYPE, std::string(fn) + ": out must be f16, bf16 or f32");
  if (rows < 0 || cols <= 0) return fail(TFO_ERR_INVALID, std::string(fn) + ": bad shape");
  if (rows == 0) return TFO_OK;
  if (!q || !scales || !out) return fail(TFO_ERR_INVALID, std::string(fn) + ": NULL pointer");
  const cudaError_t e = decode_rows_launch(q, rows, cols, q_dtype, scales, out, out_dtype, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TFO_OK : cuda_fail(e, fn);
}

size_t tfo_fp8_gemm_scaled_workspace_bytes(int64_t M, int64_t N, int64_t K, int ab_dtype, int b_layout) {
  return tfo_fp8_gemm_workspace_bytes(M, N, K, ab_dtype, b_layout) +
         ((4 * static_cast<size_t>(std::max<int64_t>(0, M) + std::max<int64_t>(0, N)) + 255) / 256) * 256;
}

int tfo_fp8_gemm_scaled(const void* a, const void* b, const float* a_scales, int a_per_row, const float* b_scales,
                        int b_per_col, void* c, int64_t M, int64_t N, int64_t K, int ab_dtype, int b_layout,
                        int out_dtype, void* workspace, size_t workspace_bytes, void* stream) {
  const char* fn = "tfo_fp8_gemm_scaled";
  if (ab_dtype != U8 && ab_dtype != E4M3) return fail(TFO_ERR_DTYPE, std::string(fn) + ": operands must be U8 or E4M3");
  if (!is_float_dtype(out_dtype)) return fail(TFO_ERR_DTYPE, std::string(fn) + ": output must be f16, bf16 or f32");
  if (b_layout != TFO_B_KN && b_layout != TFO_B_NK) return fail(TFO_ERR_INVALID, std::string(fn) + ": bad b_layout");
  if (M < 0 || N < 0 || K <= 0) return fail(TFO_ERR_INVALID, std::string(fn) + ": bad dimension (K must be positive)");
  if (M > INT32_MAX || N > INT32_MAX || K > 131072)
    return fail(TFO_ERR_INVALID, std::string(fn) + ": M, N must fit in int32 and K <= 131072");
  if (M == 0 || N == 0) return TFO_OK;
  if (!a || !b || !a_scales || !b_scales || !c) return fail(TFO_ERR_INVALID, std::string(fn) + ": NULL pointer");
  Fp8GemmArgs g{a, b, a_scales, b_scales, c, M, N, K, ab_dtype, b_layout, out_dtype, workspace, workspace_bytes};
  g.sa_rows = a_per_row ? a_scales : nullptr;
  g.sb_cols = b_per_col ? b_scales : nullptr;
  if (!a_per_row && !b_per_col) g.sa_rows = nullptr;
  if (!workspace || workspace_bytes < tfo_fp8_gemm_scaled_workspace_bytes(M, N, K, ab_dtype, b_layout))
    return fail(TFO_ERR_INVALID, std::string(fn) + ": workspace smaller than tfo_fp8_gemm_scaled_workspace_bytes()");
  const cudaError_t e = fp8_gemm_launch(g, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TFO_OK : cuda_fail(e, fn);
}

size_t tfo_gated_mlp_workspace_bytes(int64_t M, int64_t N, int64_t K, int x_dtype, int w_dtype) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  GatedMlpArgs g{};
  g.M = M; g.N = N; g.K = K; g.x_dtype = x_dtype; g.w_dtype = w_dtype;
  // alignment-independent upper bound: pretend every pointer is aligned
  g.x = g.wg = g.wu = reinterpret_cast<const void*>(uintptr_t(256));
  g.out = reinterpret_cast<void*>(uintptr_t(256));
  return gated_mlp_workspace_bytes(g);
}

int tfo_gated_mlp(const void* x, const void* w_gate, const void* w_up, void* out, int64_t M, int64_t N, int64_t K,
                  int x_dtype, int w_dtype, int activation, void* workspace, size_t workspace_bytes, void* stream) {
  if (!is_float_dtype(x_dtype) || !is_float_dtype(w_dtype))
    return fail(TFO_ERR_DTYPE, "tfo_gated_mlp: dtypes must be f16, bf16 or f32");
  if (activation < TFO_ACT_SILU || activation > TFO_ACT_GELU_TANH)
    return fail(TFO_ERR_INVALID, "tfo_gated_mlp: unknown activation");
  if (M < 0 || N < 0 || K < 0) return fail(TFO_ERR_INVALID, "tfo_gated_mlp: negative dimension");
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(TFO_ERR_INVALID, "tfo_gated_mlp: dimensions must fit in int32");
  if (M == 0 || N == 0) return TFO_OK;
  if (!out) return fail(TFO_ERR_INVALID, "tfo_gated_mlp: NULL output");
  auto st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (K == 0) {
    const size_t esz = x_dtype == F32 ? 4 : 2;
    e = cudaMemsetAsync(out, 0, static_cast<size_t>(M) * N * esz, st);
    note_launch();
    if (e != cudaSuccess) return cuda_fail(e, "tfo_gated_mlp");
    return TFO_OK;
  }
  if (!x || !w_gate || !w_up) return fail(TFO_ERR_INVALID, "tfo_gated_mlp: NULL operand");
  GatedMlpArgs g{x, w_gate, w_up, out, M, N, K, x_dtype, w_dtype, activation, workspace, workspace_bytes};
  if (workspace_bytes < gated_mlp_workspace_bytes(g))
    return fail(TFO_ERR_INVALID, "tfo_gated_mlp: workspace smaller than tfo_gated_mlp_workspace_bytes()");
  e = gated_mlp_launch(g, st);
  if (e != cudaSuccess) return cuda_fail(e, "tfo_gated_mlp");
  return TFO_OK;
}

namespace {
inline size_t round256(size_t v) { return (v + 255) / 256 * 256; }
// Workspace layout of tfo_gated_mlp_quantize: [MLP workspace][rows][partials / quantize workspace]
struct MlpQuantLayout {
  size_t mlp, rows, tail, total;
  bool tensor, one_pass;
};
MlpQuantLayout mlp_quant_layout(const void* x, const void* wg, const void* wu, int64_t M, int64_t N, int64_t K,
                                int x_dtype, int w_dtype, bool has_scale) {
  GatedMlpArgs g{x, wg, wu, nullptr, M, N, K, x_dtype, w_dtype, 0, nullptr, 0};
  MlpQuantLayout l{};
  l.mlp = round256(gated_mlp_workspace_bytes(g));
  l.tensor = gated_mlp_tensor_path(g);
  l.one_pass = has_scale && l.tensor;
  const int64_t n = M * N;
  l.rows = l.one_pass ? 0 : round256(static_cast<size_t>(n) * (x_dtype == F32 ? 4 : 2));
  l.tail = std::max(sizeof(uint32_t) * 4 * static_cast<size_t>(gated_mlp_max_ctas()), scale_workspace_bytes(n));
  l.total = l.mlp + l.rows + l.tail;
  return l;
}
}  // namespace

size_t tfo_gated_mlp_quantize_workspace_bytes(const void* x, const void* w_gate, const void* w_up, int64_t M,
                                              int64_t N, int64_t K, int x_dtype, int w_dtype, int has_scale) {
  if (M <= 0 || N <= 0 || K <= 0) return 16;
  return mlp_quant_layout(x, w_gate, w_up, M, N, K, x_dtype, w_dtype, has_scale != 0).total;
}

int tfo_gated_mlp_quantize(const void* x, const void* w_gate, const void* w_up, void* codes, int64_t M, int64_t N,
                           int64_t K, int x_dtype, int w_dtype, int activation, const float* scale, float* scale_out,
                           int code_dtype, void* workspace, size_t workspace_bytes, void* stream) {
  const char* fn = "tfo_gated_mlp_quantize";
  if (!is_float_dtype(x_dtype) || !is_float_dtype(w_dtype))
    return fail(TFO_ERR_DTYPE, std::string(fn) + ": dtypes must be f16, bf16 or f32");
  if (code_dtype != U8 && code_dtype != E4M3) return fail(TFO_ERR_DTYPE, std::string(fn) + ": codes must be U8 or E4M3");
  if (activation < TFO_ACT_SILU || activation > TFO_ACT_GELU_TANH)
    return fail(TFO_ERR_INVALID, std::string(fn) + ": unknown activation");
  if (M < 0 || N < 0 || K <= 0) return fail(TFO_ERR_INVALID, std::string(fn) + ": bad dimension (K must be positive)");
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
    return fail(TFO_ERR_INVALID, std::string(fn) + ": dimensions must fit in int32");
  if (scale == nullptr && scale_out == nullptr)
    return fail(TFO_ERR_INVALID, std::string(fn) + ": a dynamic scale needs scale_out");
  auto st = static_cast<cudaStream_t>(stream);
  if (M == 0 || N == 0) {
    if (scale != nullptr) return TFO_OK;
    if (!workspace || workspace_bytes < sizeof(uint32_t))
      return fail(TFO_ERR_INVALID, std::string(fn) + ": workspace too small");
    uint32_t* parts = static_cast<uint32_t*>(workspace);
    cudaError_t e = amax_partials_launch(x, 0, x_dtype, parts, 1, st);
    if (e == cudaSuccess) e = finalize_scale_launch(parts, 1, scale_out, st);
    return e == cudaSuccess ? TFO_OK : cuda_fail(e, fn);
  }
  if (!x || !w_gate || !w_up || !codes) return fail(TFO_ERR_INVALID, std::string(fn) + ": NULL pointer");
  const MlpQuantLayout l = mlp_quant_layout(x, w_gate, w_up, M, N, K, x_dtype, w_dtype, scale != nullptr);
  if (!workspace || workspace_bytes < l.total)
    return fail(TFO_ERR_INVALID, std::string(fn) + ": workspace smaller than tfo_gated_mlp_quantize_workspace_bytes()");
  char* ws = static_cast<char*>(workspace);
  void* rows = ws + l.mlp;
  void* tail = ws + l.mlp + l.rows;
  const int64_t n = M * N;
  GatedMlpArgs g{x, w_gate, w_up, nullptr, M, N, K, x_dtype, w_dtype, activation, ws, l.mlp};
  cudaError_t e;
  if (l.one_pass) {
    // codes straight from the MLP epilogue
    g.codes = static_cast<uint8_t*>(codes);
    g.scale = scale;
    g.e4m3 = code_dtype == E4M3 ? 1 : 0;
    e = gated_mlp_launch(g, st);
  } else if (l.tensor) {
    // rows + one max per epilogue warp, then the encode reduces the maxima to the scale
    int ctas = 0;
    g.out = rows;
    g.amax_parts = static_cast<uint32_t*>(tail);
    g.ctas_out = &ctas;
    e = gated_mlp_launch(g, st);
    if (e == cudaSuccess)
      e = encode_launch(rows, n, x_dtype, nullptr, static_cast<uint32_t*>(tail), 4 * ctas, scale_out, codes,
                        code_dtype, st);
  } else {
    // CUDA-core MLP: the rows, then the ordinary quantize
    g.out = rows;
    e = gated_mlp_launch(g, st);
    if (e == cudaSuccess)
      e = scale != nullptr ? encode_launch(rows, n, x_dtype, scale, nullptr, 0, nullptr, codes, code_dtype, st)
                           : quantize_dynamic_launch(rows, n, x_dtype, scale_out, codes, code_dtype, tail, l.tail, st);
  }
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return TFO_OK;
}

int tfo_selftest_bounded_wait(int64_t budget_cycles, void* stream) {
  if (budget_cycles <= 0 || budget_cycles > (1ll << 32))
    return fail(TFO_ERR_INVALID, "tfo_selftest_bounded_wait: budget must be in (0, 2^32] cycles");
  selftest_bounded_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(budget_cycles, error_word_ptr());
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "tfo_selftest_bounded_wait");
  return TFO_OK;
}

}  // extern "C"
