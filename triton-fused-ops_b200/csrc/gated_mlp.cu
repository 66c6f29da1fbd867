// Fused gated MLP: out[m, n] = g * act(u), g = x[m,:] . Wg[n,:], u = x[m,:] . Wu[n,:].
//
// Reference semantics (triton_ops/kernels/gated_mlp.py:31-146, oracle
// :221-251): both projections accumulate in fp32, the activation (SiLU or
// erf-GELU; tanh-GELU as an extension) is applied to the UP projection, and
// the product is rounded to x's dtype.
//
// Main path: one tcgen05 kernel (gemm_sm100.cuh) with NUM_B = 2: every
// 128-row tile of x is loaded once per K-block and multiplied against the
// 128-row gate and up weight tiles into two TMEM accumulators
// (2 x 128 fp32 columns, double-buffered = all 512 TMEM columns); the
// epilogue reads both, applies the activation in fp32 and stores x's dtype.
//  * x and weights both fp16 (or both bf16): kind::f16
//  * any fp32 operand (e.g. the fp32 module parameters with fp16 x): fp32
//    copies of the narrower operands are made in the workspace and the GEMM
//    runs as kind::tf32, matching the reference's fp32-cast TF32 dot.
// Shapes TMA cannot address (row pitch not a multiple of 16 bytes) use a
// CUDA-core tiled kernel.
#include "capi_internal.h"
#include "codec.cuh"
#include "common.cuh"
#include "epilogue.cuh"
#include "gemm_sm100.cuh"
#include "tma_host.h"

namespace tfo {

__device__ __forceinline__ float tanh_approx(float v) {
  float r;
  asm("tanh.approx.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}

// Activations on the fp32 up-projection. SiLU and tanh-GELU use the
// hardware's approximate exp2 / reciprocal / tanh (relative errors ~2^-21 to
// 2^-11, far below the fp16/bf16 output rounding); erf-GELU keeps erff.
template <int ACT>
__device__ __forceinline__ float act_fn(float u) {
  if constexpr (ACT == 0) {
    return __fdividef(u, 1.0f + __expf(-u));
  } else if constexpr (ACT == 1) {
    return 0.5f * u * (1.0f + erff(u * 0.7071067811865476f));
  } else {
    const float inner = 0.7978845608028654f * fmaf(0.044715f * u, u * u, u);
    return 0.5f * u * (1.0f + tanh_approx(inner));
  }
}

template <typename TO, int ACT>
struct GatedEpi {
  struct Params {
    TO* out;
    int64_t ldc;
    bool vec_ok;
    uint8_t* codes;         // optional 8-bit output
    const float* scale;     // its multiplier
    int e4m3;               // codes are e4m3 (else the reference codec)
    uint32_t* amax_parts;   // optional: one max |output| per epilogue warp
    bool stream_out;        // evict-first output stores (an output far larger than L2, not read back)
  };
  struct State {
    float s;        // code multiplier
    uint32_t amax;  // running max of |output| (fp32 bits of the TO-rounded values)
  };
  static __device__ __forceinline__ State init(const Params& p) {
    return {p.codes != nullptr ? *p.scale : 0.f, 0u};
  }
  static __device__ __forceinline__ void finish(const Params& p, State& st) {
    if (p.amax_parts == nullptr) return;
    const uint32_t m = warp_max_u32(st.amax);
    if ((threadIdx.x & 31) == 0) p.amax_parts[blockIdx.x * 4 + ((threadIdx.x >> 5) & 3)] = m;
  }
  __device__ __forceinline__ void operator()(const Params& p, State& st, const uint32_t (&r)[2][16], int row,
                                             int col0, int M, int N, int /*split*/) const {
    if (row >= M || col0 >= N) return;
    const int valid = min(16, N - col0);
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[0][i]) * act_fn<ACT>(__uint_as_float(r[1][i]));
    if (p.out != nullptr)
      store_row16<TO>(p.out + static_cast<int64_t>(row) * p.ldc + col0, v, valid, p.vec_ok, p.stream_out);
    if (p.codes == nullptr && p.amax_parts == nullptr) return;
    // the values the TO output holds
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = Ty<TO>::to_f(Ty<TO>::from_f(v[i]));
    if (p.amax_parts != nullptr) {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (i < valid) st.amax = max(st.amax, __float_as_uint(fabsf(v[i])));
    }
    if (p.codes != nullptr) {
      uint32_t w[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t word = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float c = __fmul_rn(v[4 * q + j], st.s);
          const uint32_t b = p.e4m3 ? static_cast<uint32_t>(__nv_cvt_float_to_fp8(c, __NV_SATFINITE, __NV_E4M3))
                                    : ref_encode(c);
          word |= b << (8 * j);
        }
        w[q] = word;
      }
      uint8_t* dst = p.codes + static_cast<int64_t>(row) * p.ldc + col0;
      if (valid == 16 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
        *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (i < valid) dst[i] = static_cast<uint8_t>(w[i >> 2] >> (8 * (i & 3)));
      }
    }
  }
};

// CUDA-core fallback for layouts TMA cannot address: 16 x 16 outputs per CTA.
template <typename TO, int ACT>
__global__ void __launch_bounds__(256) gated_simt_kernel(const void* __restrict__ x, const void* __restrict__ wg,
                                                         const void* __restrict__ wu, TO* __restrict__ out, int64_t M,
                                                         int64_t N, int64_t K, int x_dt, int w_dt) {
  __shared__ float xs[16][33], gs[16][33], us[16][33];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t m = static_cast<int64_t>(blockIdx.y) * 16 + ty;
  const int64_t n = static_cast<int64_t>(blockIdx.x) * 16 + tx;
  float g = 0.f, u = 0.f;
  for (int64_t k0 = 0; k0 < K; k0 += 32) {
    for (int i = threadIdx.x; i < 16 * 32; i += 256) {
      const int r = i / 32, c = i % 32;
      const int64_t k = k0 + c;
      const int64_t mr = static_cast<int64_t>(blockIdx.y) * 16 + r;
      const int64_t nr = static_cast<int64_t>(blockIdx.x) * 16 + r;
      xs[r][c] = (mr < M && k < K) ? load_as_float(x, mr * K + k, x_dt) : 0.f;
      gs[r][c] = (nr < N && k < K) ? load_as_float(wg, nr * K + k, w_dt) : 0.f;
      us[r][c] = (nr < N && k < K) ? load_as_float(wu, nr * K + k, w_dt) : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < 32; ++c) {
      g = fmaf(xs[ty][c], gs[tx][c], g);
      u = fmaf(xs[ty][c], us[tx][c], u);
    }
    __syncthreads();
  }
  if (m < M && n < N) out[m * N + n] = Ty<TO>::from_f(g * act_fn<ACT>(u));
}

__global__ void to_f32_kernel(const void* __restrict__ src, int64_t n, int dt, float* __restrict__ dst) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = load_as_float(src, i, dt);
}

namespace {

constexpr int kStages = 4;      // 48 KB stages (one CTA per MMA)
constexpr int kStagesPair = 6;  // 32 KB stages (two CTAs per MMA)
constexpr int kBlockN = 128;
constexpr int64_t kStreamOutBytes = 64ll << 20;  // half the 126 MB L2
constexpr int kGroupM = 16;

inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

enum class Path { F16, TF32, SIMT };

struct MlpPlan {
  Path path;
  bool cvt_x, cvt_w;
  size_t off_x, off_wg, off_wu, bytes;
};

MlpPlan plan_mlp(const GatedMlpArgs& g) {
  MlpPlan p{};
  const bool same16 = (g.x_dtype == g.w_dtype) && (g.x_dtype == F16 || g.x_dtype == BF16);
  if (same16) {
    p.path = (g.K % 8 == 0 && al16(g.x) && al16(g.wg) && al16(g.wu)) ? Path::F16 : Path::SIMT;
  } else {
    p.cvt_x = g.x_dtype != F32;
    p.cvt_w = g.w_dtype != F32;
    const bool ok = g.K % 4 == 0 && (p.cvt_x || al16(g.x)) && (p.cvt_w || (al16(g.wg) && al16(g.wu)));
    p.path = ok ? Path::TF32 : Path::SIMT;
  }
  size_t off = 0;
  if (p.path == Path::TF32) {
    p.off_x = off;
    if (p.cvt_x) off += round_up(g.M * g.K * 4, 256);
    p.off_wg = off;
    if (p.cvt_w) off += round_up(g.N * g.K * 4, 256);
    p.off_wu = off;
    if (p.cvt_w) off += round_up(g.N * g.K * 4, 256);
  }
  p.bytes = off;
  return p;
}

template <MmaKind KIND, typename TO, int ACT, int CG>
cudaError_t launch_umma_cg(const CUtensorMap& tx, const CUtensorMap& tg, const CUtensorMap& tu, const GatedMlpArgs& g,
                           uint32_t idesc, cudaStream_t st) {
  constexpr int STAGES = (CG == 2) ? kStagesPair : kStages;
  using L = GemmLayout<kBlockN, 2, STAGES, CG>;
  using Epi = GatedEpi<TO, ACT>;
  auto kern = umma_gemm_kernel<KIND, kBlockN, 2, STAGES, Epi, false, CG>;
  const int resident = gemm_resident_units(reinterpret_cast<const void*>(kern), gemm_threads(4), L::SMEM_BYTES, CG);
  if (resident <= 0) return cudaErrorInvalidConfiguration;
  // An output of more than half the L2 is written evict-first: its lines then
  // drain to HBM while the tensor-bound MLP runs instead of after it (the
  // prefill step [65536, 11264] fp16: MLP 1360-1369 -> 1391-1403 TFLOP/s, the
  // RMSNorm+RoPE that follows it 235 -> 232 us, alternating runs on one box).
  // Smaller outputs (decode sizes) stay in L2 for the projection that reads
  // them; the rows of a dynamic-scale quantize are re-read by its encode.
  const bool stream_out = g.amax_parts == nullptr &&
                          g.M * g.N * static_cast<int64_t>(sizeof(TO)) > kStreamOutBytes;
  typename Epi::Params ep{static_cast<TO*>(g.out), g.N, al16(g.out) && (g.N * sizeof(TO)) % 16 == 0, g.codes,
                          g.scale, g.e4m3, g.amax_parts, stream_out};
  const int64_t tiles = ((g.M + L::PAIR_M - 1) / L::PAIR_M) * ((g.N + kBlockN - 1) / kBlockN);
  const int units = static_cast<int>(std::min<int64_t>(tiles, resident));
  if (g.ctas_out != nullptr) *g.ctas_out = units * CG;
  cudaError_t e = launch_gemm_units(kern, gemm_threads(4), CG, units, L::SMEM_BYTES, st, tx, tg, tu, static_cast<int>(g.M),
                                    static_cast<int>(g.N), static_cast<int>(g.K), kGroupM, idesc, ep,
                                    error_word_ptr(), 1);
  note_launch();
  return e;
}

// Two-CTA tiles (M = 256 per MMA, half the shared-memory operand traffic per
// SM) once there are at least two 128-row blocks.
template <MmaKind KIND, typename TO, int ACT>
cudaError_t launch_umma(const CUtensorMap& tx, const CUtensorMap& tg, const CUtensorMap& tu, const GatedMlpArgs& g,
                        uint32_t fmt_bits, cudaStream_t st) {
  if (g.M > 128 && pair_mma_enabled())
    return launch_umma_cg<KIND, TO, ACT, 2>(tx, tg, tu, g, fmt_bits | make_idesc(0, 0, 0, false, false, 256, 2 * kBlockN), st);
  return launch_umma_cg<KIND, TO, ACT, 1>(tx, tg, tu, g, fmt_bits | make_idesc(0, 0, 0, false, false, 128, 2 * kBlockN), st);
}

template <MmaKind KIND, typename TO>
cudaError_t launch_act(const CUtensorMap& tx, const CUtensorMap& tg, const CUtensorMap& tu, const GatedMlpArgs& g,
                       uint32_t idesc, cudaStream_t st) {
  switch (g.act) {
    case 0: return launch_umma<KIND, TO, 0>(tx, tg, tu, g, idesc, st);
    case 1: return launch_umma<KIND, TO, 1>(tx, tg, tu, g, idesc, st);
    default: return launch_umma<KIND, TO, 2>(tx, tg, tu, g, idesc, st);
  }
}

template <MmaKind KIND>
cudaError_t launch_out(const CUtensorMap& tx, const CUtensorMap& tg, const CUtensorMap& tu, const GatedMlpArgs& g,
                       uint32_t idesc, cudaStream_t st) {
  switch (g.x_dtype) {
    case F16: return launch_act<KIND, __half>(tx, tg, tu, g, idesc, st);
    case BF16: return launch_act<KIND, __nv_bfloat16>(tx, tg, tu, g, idesc, st);
    default: return launch_act<KIND, float>(tx, tg, tu, g, idesc, st);
  }
}

template <typename TO>
cudaError_t launch_simt_t(const GatedMlpArgs& g, cudaStream_t st) {
  dim3 grid(static_cast<unsigned>((g.N + 15) / 16), static_cast<unsigned>((g.M + 15) / 16));
  switch (g.act) {
    case 0: gated_simt_kernel<TO, 0><<<grid, 256, 0, st>>>(g.x, g.wg, g.wu, static_cast<TO*>(g.out), g.M, g.N, g.K, g.x_dtype, g.w_dtype); break;
    case 1: gated_simt_kernel<TO, 1><<<grid, 256, 0, st>>>(g.x, g.wg, g.wu, static_cast<TO*>(g.out), g.M, g.N, g.K, g.x_dtype, g.w_dtype); break;
    default: gated_simt_kernel<TO, 2><<<grid, 256, 0, st>>>(g.x, g.wg, g.wu, static_cast<TO*>(g.out), g.M, g.N, g.K, g.x_dtype, g.w_dtype); break;
  }
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_simt(const GatedMlpArgs& g, cudaStream_t st) {
  switch (g.x_dtype) {
    case F16: return launch_simt_t<__half>(g, st);
    case BF16: return launch_simt_t<__nv_bfloat16>(g, st);
    default: return launch_simt_t<float>(g, st);
  }
}

cudaError_t convert(const void* src, int64_t n, int dt, float* dst, cudaStream_t st) {
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, num_sms() * 8)));
  to_f32_kernel<<<grid, 256, 0, st>>>(src, n, dt, dst);
  note_launch();
  return cudaGetLastError();
}

}  // namespace

size_t gated_mlp_workspace_bytes(const GatedMlpArgs& g) { return plan_mlp(g).bytes; }

void gated_mlp_tile(int64_t M, int64_t N, int64_t K, int32_t out[6]) {
  (void)N;
  (void)K;
  const int cg = (M > 128 && pair_mma_enabled()) ? 2 : 1;
  out[0] = 128 * cg;
  out[1] = kBlockN;
  out[2] = cg;
  out[3] = cg == 2 ? kStagesPair : kStages;
  out[4] = 1;
  out[5] = kGroupM;
}

bool gated_mlp_tensor_path(const GatedMlpArgs& g) { return plan_mlp(g).path != Path::SIMT; }

int gated_mlp_max_ctas() { return 2 * num_sms(); }

cudaError_t gated_mlp_launch(const GatedMlpArgs& g, cudaStream_t st) {
  const MlpPlan p = plan_mlp(g);
  if (p.path == Path::SIMT) return launch_simt(g, st);
  if (g.ws_bytes < p.bytes || (p.bytes > 0 && g.ws == nullptr)) return cudaErrorInvalidValue;

  CUtensorMap tx, tg, tu;
  if (p.path == Path::F16) {
    const CUtensorMapDataType dt = (g.x_dtype == F16) ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    if (!make_tmap_kmajor(&tx, g.x, dt, 2, g.M, g.K, g.K, 128) ||
        !make_tmap_kmajor(&tg, g.wg, dt, 2, g.N, g.K, g.K, kBlockN) ||
        !make_tmap_kmajor(&tu, g.wu, dt, 2, g.N, g.K, g.K, kBlockN))
      return cudaErrorInvalidValue;
    const uint32_t fmt = (g.x_dtype == F16) ? 0u : 1u;
    return launch_out<MmaKind::F16>(tx, tg, tu, g, make_idesc(1, fmt, fmt, false, false, 0, 0), st);
  }

  uint8_t* ws = static_cast<uint8_t*>(g.ws);
  const void* x = g.x;
  const void* wg = g.wg;
  const void* wu = g.wu;
  cudaError_t e = cudaSuccess;
  if (p.cvt_x) {
    e = convert(g.x, g.M * g.K, g.x_dtype, reinterpret_cast<float*>(ws + p.off_x), st);
    x = ws + p.off_x;
  }
  if (e == cudaSuccess && p.cvt_w) {
    e = convert(g.wg, g.N * g.K, g.w_dtype, reinterpret_cast<float*>(ws + p.off_wg), st);
    if (e == cudaSuccess) e = convert(g.wu, g.N * g.K, g.w_dtype, reinterpret_cast<float*>(ws + p.off_wu), st);
    wg = ws + p.off_wg;
    wu = ws + p.off_wu;
  }
  if (e != cudaSuccess) return e;
  const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  if (!make_tmap_kmajor(&tx, x, dt, 4, g.M, g.K, g.K, 128) || !make_tmap_kmajor(&tg, wg, dt, 4, g.N, g.K, g.K, kBlockN) ||
      !make_tmap_kmajor(&tu, wu, dt, 4, g.N, g.K, g.K, kBlockN))
    return cudaErrorInvalidValue;
  return launch_out<MmaKind::TF32>(tx, tg, tu, g, make_idesc(1, 2, 2, false, false, 0, 0), st);
}

}  // namespace tfo
