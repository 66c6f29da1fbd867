// FP8 GEMM: C[M, N] = dec(A)[M, K] . dec(B)[K, N] / (sa * sb) on tcgen05.
//
// Reference semantics (triton_ops/kernels/fp8_gemm.py:123-225): operands are
// per-tensor scaled 8-bit codes; dec() of the reference codec is
// (u - 128) / 127 * 448, so for that codec the product is an integer GEMM:
//   C = (sum_k ia * ib) * (448/127)^2 / (sa * sb),   ia = u_a - 128 in [-127, 127]
// which runs on tcgen05.mma.kind::i8 with exact int32 accumulation
// (|sum| <= 127^2 * K, exact for K < 133,000). e4m3 operands run on
// kind::f8f6f4 with fp32 accumulation: C = sum(qa * qb) / (sa * sb).
//
// Operand staging: the UMMA path wants both operands K-major with 16-byte
// aligned rows. A prep kernel writes sign-flipped (u ^ 0x80 == u - 128 as
// int8) and/or transposed copies into the caller's workspace when the layout
// needs it (B given as [K, N], reference codec, or K not a multiple of 16).
// Padded K columns are zero in both operands, so they add nothing.
#include "capi_internal.h"
#include "common.cuh"
#include "epilogue.cuh"
#include "gemm_sm100.cuh"
#include "tma_host.h"

namespace tfo {

// ---------------------------------------------------------------------------
// operand preparation
// ---------------------------------------------------------------------------
// dst[r, k] = k < K ? src[r * lds + k] ^ flip : 0, for k < Kp (Kp % 16 == 0).
__global__ void prep_rows_kernel(const uint8_t* __restrict__ src, int64_t R, int64_t K, int64_t lds,
                                 uint8_t* __restrict__ dst, int64_t Kp, uint32_t flip, bool vec_src) {
  const int64_t chunks_per_row = Kp / 16;
  const int64_t total = R * chunks_per_row;
  const uint32_t f4 = flip * 0x01010101u;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / chunks_per_row;
    const int64_t k0 = (i - r * chunks_per_row) * 16;
    uint4 o;
    if (vec_src && k0 + 16 <= K) {
      uint4 u = __ldcs(reinterpret_cast<const uint4*>(src + r * lds + k0));
      o = make_uint4(u.x ^ f4, u.y ^ f4, u.z ^ f4, u.w ^ f4);
    } else {
      uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint32_t b = (k0 + j < K) ? (static_cast<uint32_t>(src[r * lds + k0 + j]) ^ flip) : 0u;
        w[j >> 2] |= b << (8 * (j & 3));
      }
      o = make_uint4(w[0], w[1], w[2], w[3]);
    }
    reinterpret_cast<uint4*>(dst + r * Kp)[k0 / 16] = o;
  }
}

// dst[n, k] = k < K ? src[k * N + n] ^ flip : 0 (dst is [N, Kp]); 64 x 64 tiles.
__global__ void __launch_bounds__(256) prep_transpose_kernel(const uint8_t* __restrict__ src, int64_t K, int64_t N,
                                                             uint8_t* __restrict__ dst, int64_t Kp, uint32_t flip) {
  __shared__ uint8_t tile[64][68];
  const int64_t k0 = static_cast<int64_t>(blockIdx.y) * 64;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * 64;
  const int t = threadIdx.x;
  {
    const int kr = t >> 2, nc = (t & 3) * 16;
    const int64_t k = k0 + kr;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int64_t n = n0 + nc + j;
      tile[kr][nc + j] = (k < K && n < N) ? static_cast<uint8_t>(src[k * N + n] ^ flip) : 0;
    }
  }
  __syncthreads();
  const int nr = t >> 2, kc = (t & 3) * 16;
  const int64_t n = n0 + nr;
  if (n < N && k0 + kc < Kp) {
    uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) w[j >> 2] |= static_cast<uint32_t>(tile[kc + j][nr]) << (8 * (j & 3));
    reinterpret_cast<uint4*>(dst + n * Kp + k0 + kc)[0] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// ---------------------------------------------------------------------------
// epilogue: scale and round
// ---------------------------------------------------------------------------
template <typename TO, bool INT_ACC>
struct Fp8Epi {
  struct Params {
    TO* out;
    const float* sa;
    const float* sb;
    double codec_k;  // (448/127)^2 for the reference codec, 1 for e4m3
    int64_t ldc;
    bool vec_ok;
  };
  __device__ __forceinline__ void operator()(const Params& p, const uint32_t (&r)[1][16], int row, int col0, int M,
                                             int N) const {
    if (row >= M || col0 >= N) return;
    const float alpha = static_cast<float>(p.codec_k / (static_cast<double>(__ldg(p.sa)) * __ldg(p.sb)));
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float a = INT_ACC ? static_cast<float>(static_cast<int32_t>(r[0][i])) : __uint_as_float(r[0][i]);
      v[i] = a * alpha;
    }
    store_row16<TO>(p.out + static_cast<int64_t>(row) * p.ldc + col0, v, min(16, N - col0), p.vec_ok);
  }
};

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
namespace {

constexpr int kStages = 4;
constexpr int kGroupM = 16;

inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

struct Fp8Plan {
  int64_t Kp;
  bool prep_a, prep_b;
  size_t off_a, off_b, bytes;
};

Fp8Plan plan_fp8(const Fp8GemmArgs& g) {
  Fp8Plan p{};
  p.Kp = round_up(std::max<int64_t>(g.K, 1), 16);
  const bool codec = (g.ab_dtype == U8);
  const bool a_aligned = (reinterpret_cast<uintptr_t>(g.a) & 15u) == 0 && g.K % 16 == 0;
  const bool b_aligned = (reinterpret_cast<uintptr_t>(g.b) & 15u) == 0 && g.K % 16 == 0;
  p.prep_a = codec || !a_aligned;
  p.prep_b = codec || !b_aligned || g.b_layout == 0;
  size_t off = 0;
  p.off_a = off;
  if (p.prep_a) off += round_up(g.M * p.Kp, 256);
  p.off_b = off;
  if (p.prep_b) off += round_up(g.N * p.Kp, 256);
  p.bytes = off;
  return p;
}

template <MmaKind KIND, int BN, typename TO>
cudaError_t launch_fp8_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const Fp8GemmArgs& g, int64_t Kp,
                            cudaStream_t st) {
  using L = GemmLayout<BN, 1, kStages>;
  constexpr bool INT_ACC = (KIND == MmaKind::I8);
  using Epi = Fp8Epi<TO, INT_ACC>;
  auto kern = umma_gemm_kernel<KIND, BN, 1, kStages, Epi>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(L::SMEM_BYTES));
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  typename Epi::Params ep{static_cast<TO*>(g.c), g.sa, g.sb,
                          INT_ACC ? (448.0 / 127.0) * (448.0 / 127.0) : 1.0, g.N,
                          (reinterpret_cast<uintptr_t>(g.c) & 15u) == 0 && (g.N * sizeof(TO)) % 16 == 0};
  // kind::i8: D = s32, A = B = s8; kind::f8f6f4: D = f32, A = B = e4m3.
  const uint32_t idesc = INT_ACC ? make_idesc(2, 1, 1, false, false, 128, BN) : make_idesc(1, 0, 0, false, false, 128, BN);
  const int64_t tiles = ((g.M + 127) / 128) * ((g.N + BN - 1) / BN);
  const int grid = static_cast<int>(std::min<int64_t>(tiles, num_sms()));
  kern<<<grid, 192, L::SMEM_BYTES, st>>>(ta, tb, tb, static_cast<int>(g.M), static_cast<int>(g.N),
                                          static_cast<int>(Kp), kGroupM, idesc, ep, error_word_ptr());
  note_launch();
  return cudaGetLastError();
}

template <MmaKind KIND, int BN>
cudaError_t launch_fp8_out(const CUtensorMap& ta, const CUtensorMap& tb, const Fp8GemmArgs& g, int64_t Kp,
                           cudaStream_t st) {
  switch (g.out_dtype) {
    case F16: return launch_fp8_gemm<KIND, BN, __half>(ta, tb, g, Kp, st);
    case BF16: return launch_fp8_gemm<KIND, BN, __nv_bfloat16>(ta, tb, g, Kp, st);
    default: return launch_fp8_gemm<KIND, BN, float>(ta, tb, g, Kp, st);
  }
}

}  // namespace

// Upper bound over operand alignments: room for both prepared operands.
size_t fp8_gemm_workspace_bytes(const Fp8GemmArgs& g) {
  const int64_t Kp = round_up(std::max<int64_t>(g.K, 1), 16);
  return static_cast<size_t>(round_up(g.M * Kp, 256) + round_up(g.N * Kp, 256));
}

// Static tile table: BLOCK_N = 256 once there are enough row blocks to fill the
// GPU, 128 for short-M problems (more column tiles in flight).
int fp8_gemm_block_n(int64_t M, int64_t N) {
  const int64_t mb = (M + 127) / 128;
  return (mb * ((N + 255) / 256) >= num_sms() || N <= 128) ? (N <= 128 ? 128 : 256) : 128;
}

cudaError_t fp8_gemm_launch(const Fp8GemmArgs& g, cudaStream_t st) {
  const Fp8Plan p = plan_fp8(g);
  if (g.ws_bytes < p.bytes || (p.bytes > 0 && g.ws == nullptr)) return cudaErrorInvalidValue;
  uint8_t* ws = static_cast<uint8_t*>(g.ws);
  const uint32_t flip = (g.ab_dtype == U8) ? 0x80u : 0u;
  const uint8_t* a = static_cast<const uint8_t*>(g.a);
  const uint8_t* b = static_cast<const uint8_t*>(g.b);
  const int prep_threads = 256;
  if (p.prep_a) {
    uint8_t* da = ws + p.off_a;
    const int64_t total = g.M * (p.Kp / 16);
    const int grid = static_cast<int>(std::min<int64_t>((total + prep_threads - 1) / prep_threads, num_sms() * 16));
    prep_rows_kernel<<<grid, prep_threads, 0, st>>>(a, g.M, g.K, g.K, da, p.Kp, flip,
                                                    (reinterpret_cast<uintptr_t>(a) & 15u) == 0 && g.K % 16 == 0);
    note_launch();
    a = da;
  }
  if (p.prep_b) {
    uint8_t* db = ws + p.off_b;
    if (g.b_layout == 0) {
      dim3 grid(static_cast<unsigned>((g.N + 63) / 64), static_cast<unsigned>((p.Kp + 63) / 64));
      prep_transpose_kernel<<<grid, 256, 0, st>>>(b, g.K, g.N, db, p.Kp, flip);
      note_launch();
    } else {
      const int64_t total = g.N * (p.Kp / 16);
      const int grid = static_cast<int>(std::min<int64_t>((total + prep_threads - 1) / prep_threads, num_sms() * 16));
      prep_rows_kernel<<<grid, prep_threads, 0, st>>>(b, g.N, g.K, g.K, db, p.Kp, flip,
                                                      (reinterpret_cast<uintptr_t>(b) & 15u) == 0 && g.K % 16 == 0);
      note_launch();
    }
    b = db;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  const int bn = fp8_gemm_block_n(g.M, g.N);
  CUtensorMap ta, tb;
  const int64_t lda = p.prep_a ? p.Kp : g.K;
  const int64_t ldb = p.prep_b ? p.Kp : g.K;
  if (!make_tmap_kmajor(&ta, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.M, p.prep_a ? p.Kp : g.K, lda, 128) ||
      !make_tmap_kmajor(&tb, b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.N, p.prep_b ? p.Kp : g.K, ldb, bn))
    return cudaErrorInvalidValue;
  const int64_t Kp = p.Kp;
  if (g.ab_dtype == U8) {
    return bn == 256 ? launch_fp8_out<MmaKind::I8, 256>(ta, tb, g, Kp, st) : launch_fp8_out<MmaKind::I8, 128>(ta, tb, g, Kp, st);
  }
  return bn == 256 ? launch_fp8_out<MmaKind::F8F6F4, 256>(ta, tb, g, Kp, st)
                   : launch_fp8_out<MmaKind::F8F6F4, 128>(ta, tb, g, Kp, st);
}

}  // namespace tfo
