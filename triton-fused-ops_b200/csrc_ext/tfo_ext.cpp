// PyTorch extension over the C ABI for the calls whose kernels take a few
// microseconds (decode-size activations), where the host work of the Python
// wrappers (argument checks, two or three allocations, several ctypes calls)
// took longer than the kernels. One Python -> C++ call here checks the common
// case, allocates through torch's caching allocator, reuses a scratch buffer
// per (device, stream) and calls the library; anything outside the common
// case returns None and the Python wrapper takes its full path (which raises
// the package's exceptions). The arithmetic is the library's: these functions
// produce exactly what the Python path produces.
//
// Mirrors: triton_ops/kernels/fp8_quantize.py:128-173 (quantize_fp8, dynamic
// scale) and triton_ops/kernels/fp8_gemm.py:272-310 (FP8Linear.forward).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "tfo_b200.h"

namespace py = pybind11;

namespace {

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kHalf: return TFO_DTYPE_F16;
    case at::kBFloat16: return TFO_DTYPE_BF16;
    case at::kFloat: return TFO_DTYPE_F32;
    case at::kByte: return TFO_DTYPE_U8;
    case at::kFloat8_e4m3fn: return TFO_DTYPE_E4M3;
    default: return -1;
  }
}

bool is_float(at::ScalarType t) { return t == at::kHalf || t == at::kBFloat16 || t == at::kFloat; }

// Non-zero status -> Python RuntimeError "tfo status <n>: <message>"; the
// wrapper maps it to the package's exception for that status.
void check(int status, const char* what) {
  if (status != TFO_OK) {
    const char* msg = tfo_last_error();
    throw std::runtime_error(std::string("tfo status ") + std::to_string(status) + ": " + what + ": " +
                             (msg ? msg : ""));
  }
}

// One grow-only scratch buffer per (device, stream), at most kMaxEntries kept
// (least recently used dropped), as the Python wrappers do; a fresh tensor
// while the stream is being captured into a CUDA graph.
constexpr size_t kMaxEntries = 8;
struct WsEntry {
  int device;
  cudaStream_t stream;
  at::Tensor buf;
};
std::mutex g_ws_mu;
std::vector<WsEntry> g_ws;  // most recently used last

// `st` is torch's current stream on `dev` (the device guard is set).
at::Tensor workspace(size_t bytes, const at::Device& dev, cudaStream_t st) {
  bytes = std::max<size_t>(bytes, 16);
  const auto opts = at::TensorOptions().dtype(at::kByte).device(dev);
  if (at::cuda::currentStreamCaptureStatusMayInitCtx() != at::cuda::CaptureStatus::None)
    return at::empty({static_cast<int64_t>(bytes)}, opts);
  std::lock_guard<std::mutex> lock(g_ws_mu);
  for (size_t i = 0; i < g_ws.size(); ++i) {
    if (g_ws[i].device == dev.index() && g_ws[i].stream == st) {
      WsEntry e = g_ws[i];
      g_ws.erase(g_ws.begin() + static_cast<long>(i));
      if (static_cast<size_t>(e.buf.numel()) < bytes)
        e.buf = at::empty({static_cast<int64_t>(std::max(bytes, 2 * static_cast<size_t>(e.buf.numel())))}, opts);
      g_ws.push_back(e);
      return e.buf;
    }
  }
  g_ws.push_back(WsEntry{dev.index(), st, at::empty({static_cast<int64_t>(bytes)}, opts)});
  if (g_ws.size() > kMaxEntries) g_ws.erase(g_ws.begin());
  return g_ws.back().buf;
}

void clear_workspaces() {
  std::lock_guard<std::mutex> lock(g_ws_mu);
  g_ws.clear();
}

bool common_ok(const at::Tensor& x) { return x.is_cuda() && x.is_contiguous() && is_float(x.scalar_type()); }

// quantize_fp8(x) with a dynamic scale: (codes shaped like x, 0-dim fp32 scale),
// or None outside the common case (CUDA, contiguous, f16/bf16/f32 input,
// uint8 or float8_e4m3fn codes).
py::object quantize_dynamic(const at::Tensor& x, int64_t out_code) {
  if (!common_ok(x) || (out_code != TFO_DTYPE_U8 && out_code != TFO_DTYPE_E4M3)) return py::none();
  const c10::cuda::CUDAGuard guard(x.device());
  const auto st = at::cuda::getCurrentCUDAStream(x.device().index()).stream();
  const auto code_type = out_code == TFO_DTYPE_U8 ? at::kByte : at::kFloat8_e4m3fn;
  at::Tensor out = at::empty(x.sizes(), x.options().dtype(code_type));
  at::Tensor scale = at::empty({}, x.options().dtype(at::kFloat));
  const int64_t n = x.numel();
  at::Tensor ws = workspace(tfo_fp8_scale_workspace_bytes(n), x.device(), st);
  check(tfo_fp8_quantize(x.data_ptr(), n, dtype_code(x.scalar_type()), nullptr, scale.data_ptr<float>(),
                         out.data_ptr(), static_cast<int>(out_code), ws.data_ptr(), static_cast<size_t>(ws.numel()),
                         st),
        "tfo_fp8_quantize");
  return py::make_tuple(out, scale);
}

// FP8Linear.forward with the weight prepared once (w_s8 = codes ^ 0x80, w_sums
// its row sums): x [..., K] -> dynamic quantize -> GEMM with the bias in the
// epilogue -> [..., N] in x's dtype (torch's promotion with the bias dtype).
// None outside the common case.
py::object linear_prepared(const at::Tensor& x, const at::Tensor& w_s8, const at::Tensor& w_sums,
                           const at::Tensor& w_scale, const c10::optional<at::Tensor>& bias) {
  if (!common_ok(x) || x.dim() < 1) return py::none();
  const int64_t K = x.size(-1);
  const int64_t N = w_s8.size(0);
  if (K % 16 != 0 || w_s8.dim() != 2 || w_s8.size(1) != K || w_s8.scalar_type() != at::kChar ||
      !w_s8.is_contiguous() || w_s8.device() != x.device() || w_sums.device() != x.device() ||
      w_sums.scalar_type() != at::kInt || w_scale.device() != x.device() || w_scale.scalar_type() != at::kFloat ||
      !w_scale.is_contiguous() || w_scale.numel() != 1)
    return py::none();
  const at::Tensor* b = nullptr;
  if (bias.has_value()) {
    b = &bias.value();
    if (b->device() != x.device() || !b->is_contiguous() || !is_float(b->scalar_type()) || b->numel() != N)
      return py::none();
  }
  const c10::cuda::CUDAGuard guard(x.device());
  const auto st = at::cuda::getCurrentCUDAStream(x.device().index()).stream();
  const int64_t M = x.numel() / K;
  const auto gemm_type = x.scalar_type();
  const auto res_type = b ? at::promote_types(gemm_type, b->scalar_type()) : gemm_type;
  std::vector<int64_t> out_shape(x.sizes().begin(), x.sizes().end());
  out_shape.back() = N;
  at::Tensor out = at::empty(out_shape, x.options().dtype(res_type));
  if (out.numel() == 0) return py::cast(out);
  at::Tensor codes = at::empty({M, K}, x.options().dtype(at::kByte));
  at::Tensor x_scale = at::empty({}, x.options().dtype(at::kFloat));
  const size_t ws_bytes = std::max(tfo_fp8_scale_workspace_bytes(M * K),
                                   tfo_fp8_gemm_workspace_bytes(M, N, K, TFO_DTYPE_U8, TFO_B_NK));
  at::Tensor ws = workspace(ws_bytes, x.device(), st);  // the two calls run in stream order
  check(tfo_fp8_quantize(x.data_ptr(), M * K, dtype_code(gemm_type), nullptr, x_scale.data_ptr<float>(),
                         codes.data_ptr(), TFO_DTYPE_U8, ws.data_ptr(), static_cast<size_t>(ws.numel()), st),
        "tfo_fp8_quantize");
  check(tfo_fp8_linear_prepared(codes.data_ptr(), w_s8.data_ptr(), w_sums.data_ptr<int32_t>(),
                                x_scale.data_ptr<float>(), w_scale.data_ptr<float>(), b ? b->data_ptr() : nullptr,
                                b ? dtype_code(b->scalar_type()) : -1, out.data_ptr(), M, N, K, dtype_code(gemm_type),
                                dtype_code(res_type), ws.data_ptr(), static_cast<size_t>(ws.numel()), st),
        "tfo_fp8_linear_prepared");
  return py::cast(out);
}

}  // namespace

PYBIND11_MODULE(_tfo_ext, m) {
  m.doc() = "PyTorch entry points over the tfo_b200 C ABI for launch-latency-bound calls";
  m.def("quantize_dynamic", &quantize_dynamic, "dynamic-scale quantize (codes, scale) or None");
  m.def("linear_prepared", &linear_prepared, "FP8Linear forward with a prepared weight, or None");
  m.def("clear_workspaces", &clear_workspaces, "releases the cached scratch buffers");
}
