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
  griddep_launch_dependents();  // the GEMM that follows may set up meanwhile
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
  griddep_launch_dependents();  // the GEMM that follows may set up meanwhile
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

// Sign flip + sums for the single-operand staging of the reference codec.
// Rows: dst[r, :] = src[r, :] ^ 0x80 (as int8) and sums[r] = sum of the
// row's int8 values; one warp per row, K % 16 == 0, 16-byte aligned rows.
constexpr int kRowUnroll = 8;
__global__ void __launch_bounds__(256) prep_rows_s8_sum_kernel(const uint8_t* __restrict__ src, int64_t R, int64_t K,
                                                               int8_t* __restrict__ dst, int32_t* __restrict__ sums) {
  griddep_launch_dependents();  // the GEMM that follows may set up meanwhile
  griddep_wait();  // launched as a programmatic dependent: inputs are read after this
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < R; r += warps) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src + r * K);
    uint4* d4 = reinterpret_cast<uint4*>(dst + r * K);
    int acc = 0;
    // kRowUnroll 16-byte loads per lane are issued before the first is used:
    // a 4 KB row is one DRAM round trip, not eight in sequence
    const int64_t nv = K / 16;
    for (int64_t c0 = lane; c0 < nv; c0 += 32 * kRowUnroll) {
      uint4 u[kRowUnroll];
#pragma unroll
      for (int i = 0; i < kRowUnroll; ++i)
        if (c0 + 32 * i < nv) u[i] = __ldcs(s4 + c0 + 32 * i);
#pragma unroll
      for (int i = 0; i < kRowUnroll; ++i) {
        if (c0 + 32 * i < nv) {
          uint4 v = u[i];
          v.x ^= 0x80808080u; v.y ^= 0x80808080u; v.z ^= 0x80808080u; v.w ^= 0x80808080u;
          acc = __dp4a(static_cast<int>(v.x), 0x01010101, acc);
          acc = __dp4a(static_cast<int>(v.y), 0x01010101, acc);
          acc = __dp4a(static_cast<int>(v.z), 0x01010101, acc);
          acc = __dp4a(static_cast<int>(v.w), 0x01010101, acc);
          d4[c0 + 32 * i] = v;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) sums[r] = acc;
  }
}

// Columns: dst[k, n] = src[k, n] ^ 0x80 for a [K, N] matrix (N % 16 == 0) and
// sums[n] += the column's int8 values over this CTA's K range (sums zeroed
// first; integer atomics keep the result exact and order-independent).
// A CTA covers kColChunks 16-byte column chunks (1024 columns) and
// kColGroups * kColRows rows; thread (group g, chunk c) reads rows g, g + G, ...
// so a warp reads 512 contiguous bytes of one row, with kColUnroll loads in
// flight. Raw codes are summed two bytes per 32-bit word in 16-bit lanes (at
// most kColRows * 255 per lane), the groups are combined in shared memory,
// and each column receives one atomic per CTA.
constexpr int kColChunks = 64, kColGroups = 8, kColRows = 16, kColUnroll = 8;
constexpr int kColThreads = kColChunks * kColGroups;
static_assert(kColRows * 255 < 65536 && kColRows % kColUnroll == 0, "16-bit lane sums");

__global__ void __launch_bounds__(kColThreads) prep_cols_s8_sum_kernel(const uint8_t* __restrict__ src, int64_t K,
                                                                        int64_t N, int8_t* __restrict__ dst,
                                                                        int32_t* __restrict__ sums) {
  griddep_launch_dependents();  // the GEMM that follows may set up meanwhile
  __shared__ int32_t part[kColGroups][kColChunks * 17];  // 17-word stride: no bank conflicts
  const int cx = threadIdx.x % kColChunks, g = threadIdx.x / kColChunks;
  const int64_t chunks = N / 16;
  const int64_t c = static_cast<int64_t>(blockIdx.x) * kColChunks + cx;
  const int64_t k0 = static_cast<int64_t>(blockIdx.y) * (kColGroups * kColRows) + g;
  uint32_t even[4] = {0u, 0u, 0u, 0u}, odd[4] = {0u, 0u, 0u, 0u};
  int rows = 0;
  if (c < chunks) {
#pragma unroll 1
    for (int i0 = 0; i0 < kColRows; i0 += kColUnroll) {
      uint4 u[kColUnroll];
#pragma unroll
      for (int i = 0; i < kColUnroll; ++i) {
        const int64_t k = k0 + static_cast<int64_t>(i0 + i) * kColGroups;
        if (k < K) u[i] = __ldcs(reinterpret_cast<const uint4*>(src + k * N) + c);
      }
#pragma unroll
      for (int i = 0; i < kColUnroll; ++i) {
        const int64_t k = k0 + static_cast<int64_t>(i0 + i) * kColGroups;
        if (k < K) {
          const uint32_t w[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            even[q] += w[q] & 0x00FF00FFu;
            odd[q] += (w[q] >> 8) & 0x00FF00FFu;
          }
          reinterpret_cast<uint4*>(dst + k * N)[c] =
              make_uint4(w[0] ^ 0x80808080u, w[1] ^ 0x80808080u, w[2] ^ 0x80808080u, w[3] ^ 0x80808080u);
          ++rows;
        }
      }
    }
  }
  // word q holds columns 4q .. 4q+3 in bytes 0..3: bytes 0, 2 in `even`, 1, 3 in `odd`
  int32_t* mine = &part[g][cx * 17];
  const int32_t bias = 128 * rows;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    mine[4 * q + 0] = static_cast<int32_t>(even[q] & 0xFFFFu) - bias;
    mine[4 * q + 1] = static_cast<int32_t>(odd[q] & 0xFFFFu) - bias;
    mine[4 * q + 2] = static_cast<int32_t>(even[q] >> 16) - bias;
    mine[4 * q + 3] = static_cast<int32_t>(odd[q] >> 16) - bias;
  }
  __syncthreads();
  for (int j = threadIdx.x; j < kColChunks * 16; j += kColThreads) {
    const int64_t col = static_cast<int64_t>(blockIdx.x) * kColChunks * 16 + j;
    if (col < N) {
      int32_t t = 0;
#pragma unroll
      for (int gg = 0; gg < kColGroups; ++gg) t += part[gg][(j >> 4) * 17 + (j & 15)];
      atomicAdd(sums + col, t);
    }
  }
}

// ---------------------------------------------------------------------------
// epilogue: correction, scale and round (or raw partials for split-K)
// ---------------------------------------------------------------------------
// With the reference codec, one operand may reach the tensor cores unflipped
// (raw u8 = int8 value + 128); then acc = exact + 128 * (sum of the other
// operand's int8 values along K), which corr_row (per output row, the A sums)
// or corr_col (per output column, the B sums) removes.
// FP8Linear's `fp8_gemm(...) + bias`: the product rounded to the GEMM's
// output dtype, then the bias added in fp32 (torch's arithmetic for the sum).
__device__ __forceinline__ float round_to_dtype(float v, int dt) {
  if (dt == F16) return __half2float(__float2half_rn(v));
  if (dt == BF16) return __bfloat162float(__float2bfloat16_rn(v));
  return v;
}
// The 16 bias values of columns col0.. as fp32: 16-byte loads when all 16
// exist and are 16-byte aligned (col0 is a multiple of 16), else one by one.
__device__ __forceinline__ void load_bias16(float (&b)[16], const void* bias, int bias_dt, int col0, int valid) {
  const int esz = bias_dt == F32 ? 4 : 2;
  const uint8_t* p = static_cast<const uint8_t*>(bias) + static_cast<int64_t>(col0) * esz;
  if (valid == 16 && (reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
    if (bias_dt == F32) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(p) + q);
        b[4 * q] = t.x; b[4 * q + 1] = t.y; b[4 * q + 2] = t.z; b[4 * q + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const uint4 t = __ldg(reinterpret_cast<const uint4*>(p) + q);
        const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = bias_dt == F16 ? __half22float2(*reinterpret_cast<const __half2*>(&w[j]))
                                          : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
          b[8 * q + 2 * j] = f.x;
          b[8 * q + 2 * j + 1] = f.y;
        }
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) b[i] = i < valid ? load_as_float(bias, col0 + i, bias_dt) : 0.f;
  }
}
__device__ __forceinline__ void linear_bias16(float (&v)[16], const void* bias, int bias_dt, int round_dt, int col0,
                                              int valid) {
  float b[16];
  load_bias16(b, bias, bias_dt, col0, valid);
  // the product rounded to the GEMM's output dtype (one branch per call), then the bias in fp32
  if (round_dt == F16) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __half2float(__float2half_rn(v[i]));
  } else if (round_dt == BF16) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __bfloat162float(__float2bfloat16_rn(v[i]));
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __fadd_rn(v[i], b[i]);
}

template <typename TO, bool INT_ACC>
struct Fp8Epi {
  struct Params {
    TO* out;
    const float* sa;
    const float* sb;
    double codec_k;  // (448/127)^2 for the reference codec, 1 for e4m3
    int64_t ldc;
    bool vec_ok;
    const int32_t* corr_row;
    const int32_t* corr_col;
    uint32_t* partial;  // split-K: [splits][M][N] raw accumulators
    const void* bias;   // FP8Linear: bias[N] of dtype bias_dt, added after rounding to round_dt
    int bias_dt, round_dt;
    const float* ra;    // per-row factors codec_k / sa[m] (replace alpha when set, with rb)
    const float* rb;    // per-column factors 1 / sb[n]
  };
  // alpha = fp32(codec_k / (sa * sb)), computed once per thread
  struct State {
    float alpha;
  };
  static __device__ __forceinline__ State init(const Params& p) {
    return {static_cast<float>(p.codec_k / (static_cast<double>(__ldg(p.sa)) * __ldg(p.sb)))};
  }
  // cluster K split: sum of two slices' raw accumulators (int32 wraps exactly;
  // fp32 in slice order) and the parameters of the final epilogue call
  static __device__ __forceinline__ uint32_t add_partial(uint32_t a, uint32_t b) {
    if constexpr (INT_ACC) return a + b;
    else return __float_as_uint(__uint_as_float(a) + __uint_as_float(b));
  }
  static __device__ __forceinline__ Params final_params(const Params& p) {
    Params q = p;
    q.partial = nullptr;
    return q;
  }
  static __device__ __forceinline__ void finish(const Params&, State&) {}
  __device__ __forceinline__ void operator()(const Params& p, State& st, const uint32_t (&r)[1][16], int row,
                                             int col0, int M, int N, int split) const {
    if (row >= M || col0 >= N) return;
    const int valid = min(16, N - col0);
    if (p.partial != nullptr) {
      uint32_t* dst = p.partial + (static_cast<int64_t>(split) * M + row) * N + col0;
      if (valid == 16 && (N & 3) == 0) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          reinterpret_cast<uint4*>(dst)[q] = make_uint4(r[0][4 * q], r[0][4 * q + 1], r[0][4 * q + 2], r[0][4 * q + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (i < valid) dst[i] = r[0][i];
      }
      return;
    }
    const float alpha = st.alpha;
    float v[16];
    float colf[16];  // per-element factor: alpha, or ra[row] * rb[col]
    if (p.ra != nullptr) {
      const float rr = __ldg(p.ra + row);
#pragma unroll
      for (int i = 0; i < 16; ++i) colf[i] = rr * __ldg(p.rb + min(col0 + i, N - 1));
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) colf[i] = alpha;
    }
    if constexpr (INT_ACC) {
      int32_t cc[16];
      const int32_t cr = p.corr_row ? 128 * __ldg(p.corr_row + row) : 0;
      if (p.corr_col && valid == 16) {
        // the sums array is 256-byte aligned and col0 is a multiple of 16
        const int4* q = reinterpret_cast<const int4*>(p.corr_col + col0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int4 t = __ldg(q + j);
          cc[4 * j] = t.x; cc[4 * j + 1] = t.y; cc[4 * j + 2] = t.z; cc[4 * j + 3] = t.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) cc[i] = p.corr_col ? __ldg(p.corr_col + min(col0 + i, N - 1)) : 0;
      }
#pragma unroll
      for (int i = 0; i < 16; ++i)
        v[i] = static_cast<float>(static_cast<int32_t>(r[0][i]) - cr - 128 * cc[i]) * colf[i];
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[0][i]) * colf[i];
    }
    if (p.bias != nullptr) linear_bias16(v, p.bias, p.bias_dt, p.round_dt, col0, valid);
    store_row16<TO>(p.out + static_cast<int64_t>(row) * p.ldc + col0, v, valid, p.vec_ok);
  }
};

// Per-token / per-channel factors: ra[m] = codec_k / sa[m] (or / sa), rb[n] = 1 / sb[n] (or 1 / sb).
__global__ void fp8_scale_vectors_kernel(const float* __restrict__ sa, const float* __restrict__ sa_rows,
                                         const float* __restrict__ sb, const float* __restrict__ sb_cols, int64_t M,
                                         int64_t N, double codec_k, float* __restrict__ ra, float* __restrict__ rb) {
  griddep_launch_dependents();  // the GEMM that follows may set up meanwhile
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < M + N;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (i < M) ra[i] = static_cast<float>(codec_k / static_cast<double>(sa_rows != nullptr ? sa_rows[i] : *sa));
    else rb[i - M] = static_cast<float>(1.0 / static_cast<double>(sb_cols != nullptr ? sb_cols[i - M] : *sb));
  }
}

// Sums the split-K partials of each output, applies the correction and scale,
// rounds to the output dtype.
template <typename TO, bool INT_ACC>
__global__ void __launch_bounds__(256) fp8_splitk_finalize_kernel(const uint32_t* __restrict__ partial, int splits,
                                                                  int64_t M, int64_t N, const float* __restrict__ sa,
                                                                  const float* __restrict__ sb, double codec_k,
                                                                  const int32_t* __restrict__ corr_row,
                                                                  const int32_t* __restrict__ corr_col,
                                                                  const void* __restrict__ bias, int bias_dt,
                                                                  int round_dt, const float* __restrict__ ra,
                                                                  const float* __restrict__ rb, TO* __restrict__ out) {
  const float alpha = static_cast<float>(codec_k / (static_cast<double>(__ldg(sa)) * __ldg(sb)));
  const int64_t total = M * N;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v;
    if constexpr (INT_ACC) {
      int32_t acc = 0;
      for (int s = 0; s < splits; ++s) acc += static_cast<int32_t>(partial[s * total + i]);
      if (corr_row) acc -= 128 * corr_row[i / N];
      if (corr_col) acc -= 128 * corr_col[i % N];
      v = static_cast<float>(acc);
    } else {
      float acc = 0.f;
      for (int s = 0; s < splits; ++s) acc += __uint_as_float(partial[s * total + i]);
      v = acc;
    }
    float r = v * (ra != nullptr ? ra[i / N] * rb[i % N] : alpha);
    if (bias != nullptr) r = __fadd_rn(round_to_dtype(r, round_dt), load_as_float(bias, i % N, bias_dt));
    out[i] = Ty<TO>::from_f(r);
  }
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
namespace {

constexpr int kStages = 4;      // 48 KB stages (one CTA per MMA, 256-column tiles)
constexpr int kStages128 = 7;   // 32 KB stages (one CTA per MMA, 128-column tiles)
constexpr int kStagesPair = 6;  // 32 KB stages (two CTAs per MMA)
constexpr int kStagesSmallA = 11;  // 20 KB stages (128-column tiles, 32-row A stages for M <= 32)
constexpr int stages_for(int bn, int cg, int a_rows = 128) {
  return cg == 2 ? kStagesPair : (bn == 256 ? kStages : (a_rows == 32 ? kStagesSmallA : kStages128));
}
constexpr int kGroupM = 16;
constexpr int kEpiWarps = 8;  // two epilogue warps per TMEM sub-partition
constexpr int kThreads = gemm_threads(kEpiWarps);

inline int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }
inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Operand staging plan.
//  * legacy: some operand is not TMA-addressable (unaligned base, K % 16 or,
//    for a [K, N] B, N % 16): both operands are rewritten K-major, zero-padded
//    and (reference codec) sign-flipped; B tiles K-major.
//  * direct: both operands are read in place by TMA (B [K, N] as an MN-major
//    operand). With the reference codec only the smaller operand is
//    sign-flipped (with its sums for the epilogue correction); e4m3 needs none.
struct Fp8Plan {
  bool legacy;
  int64_t Kp;
  bool prep_a, prep_b;  // legacy: both; direct + codec: exactly one
  bool b_mn;            // B read MN-major from [K, N]
  size_t off_a, off_b, off_sum, off_part, off_vec, bytes;
  int bn, cg, splits;
  int a_rows;           // rows of an A stage: 32 for M <= 32 with 128-column single-CTA tiles, else 128
  bool ksplit_cluster;  // K slices of a tile reduced inside one cluster (no partials, no finalize)
};

// Tile shape: 256-column tiles, as two-CTA 256 x 256 tiles when M has more
// than one 128-row block (half the operand bytes per SM of 128 x 256 tiles);
// for M <= 128, 128-column tiles unless the 256-column ones already cover the
// GPU. K is split when the tiles alone cannot occupy half the GPU.
void pick_tiles(int64_t M, int64_t N, int64_t Kp, Fp8Plan& p) {
  const int sms = num_sms();
  p.bn = 256;
  if (N <= 128 || (M <= 128 && ((N + 255) / 256) < sms)) p.bn = 128;
  p.cg = (p.bn == 256 && M > 128 && pair_mma_enabled()) ? 2 : 1;
  const int64_t tiles = ((M + 128 * p.cg - 1) / (128 * p.cg)) * ((N + p.bn - 1) / p.bn);
  const int64_t units = sms / p.cg;
  const int64_t num_k = (Kp + 127) / 128;
  p.splits = 1;
  if (tiles < units / 2) p.splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(num_k / 4, units / tiles)));
  p.ksplit_cluster = (p.splits > 1 && p.splits <= 8 && p.cg == 1 && p.bn == 128);
  // few rows: 32-row A stages (4 KB instead of 16 KB of mostly zero-filled
  // rows), so 11 stages fit and a K slice's blocks are all requested at once
  p.a_rows = (p.cg == 1 && p.bn == 128 && M <= 32) ? 32 : 128;
}

Fp8Plan plan_fp8(const Fp8GemmArgs& g, bool assume_aligned) {
  Fp8Plan p{};
  const bool codec = (g.ab_dtype == U8);
  const bool a_ok = (assume_aligned || al16(g.a)) && g.K % 16 == 0;
  const bool b_ok = (assume_aligned || al16(g.b)) && (g.b_layout == 1 ? g.K % 16 == 0 : g.N % 16 == 0);
  p.legacy = !(a_ok && b_ok);
  size_t off = 0;
  if (p.legacy) {
    p.Kp = round_up(std::max<int64_t>(g.K, 1), 16);
    p.prep_a = p.prep_b = true;
    p.b_mn = false;
    p.off_a = off;
    off += round_up(g.M * p.Kp, 256);
    p.off_b = off;
    off += round_up(g.N * p.Kp, 256);
    p.off_sum = off;
  } else {
    p.Kp = g.K;
    p.b_mn = (g.b_layout == 0);
    if (codec) {
      p.prep_a = (g.M <= g.N);
      p.prep_b = !p.prep_a;
    }
    p.off_a = off;
    if (p.prep_a) off += round_up(g.M * g.K, 256);
    p.off_b = off;
    if (p.prep_b) off += round_up(g.N * g.K, 256);
    p.off_sum = off;
    if (codec) off += round_up(4 * (p.prep_a ? g.M : g.N), 256);
  }
  pick_tiles(g.M, g.N, p.Kp, p);
  p.off_part = off;
  if (p.splits > 1 && !p.ksplit_cluster) off += round_up(static_cast<int64_t>(p.splits) * g.M * g.N * 4, 256);
  p.off_vec = off;
  if (g.sa_rows != nullptr || g.sb_cols != nullptr) off += round_up(4 * (g.M + g.N), 256);
  p.bytes = off;
  return p;
}

template <MmaKind KIND, int BN, typename TO, bool B_MN, int CG, int A_ROWS>
cudaError_t launch_fp8_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const Fp8GemmArgs& g, const Fp8Plan& p,
                            uint32_t idesc, const int32_t* corr_row, const int32_t* corr_col, uint32_t* partial,
                            cudaStream_t st) {
  const float* ra = nullptr;
  const float* rb = nullptr;
  if (g.sa_rows != nullptr || g.sb_cols != nullptr) {
    ra = reinterpret_cast<const float*>(static_cast<uint8_t*>(g.ws) + p.off_vec);
    rb = ra + g.M;
  }
  constexpr int STAGES = stages_for(BN, CG, A_ROWS);
  using L = GemmLayout<BN, 1, STAGES, CG, false, A_ROWS>;
  constexpr bool INT_ACC = (KIND == MmaKind::I8);
  using Epi = Fp8Epi<TO, INT_ACC>;
  auto kern = umma_gemm_kernel<KIND, BN, 1, STAGES, Epi, B_MN, CG, false, kEpiWarps, A_ROWS>;
  const int resident = gemm_resident_units(reinterpret_cast<const void*>(kern), kThreads, L::SMEM_BYTES, CG);
  if (resident <= 0) return cudaErrorInvalidConfiguration;
  const double codec_k = INT_ACC ? (448.0 / 127.0) * (448.0 / 127.0) : 1.0;
  typename Epi::Params ep{static_cast<TO*>(g.c), g.sa, g.sb, codec_k, g.N,
                          al16(g.c) && (g.N * sizeof(TO)) % 16 == 0, corr_row, corr_col,
                          p.splits > 1 ? partial : nullptr, g.bias, g.bias_dtype, g.round_dtype, ra, rb};
  const int64_t work = ((g.M + L::PAIR_M - 1) / L::PAIR_M) * ((g.N + BN - 1) / BN) * p.splits;
  if constexpr (CG == 1 && BN == 128) {
    if (p.ksplit_cluster) {
      // one CTA per (tile, K slice); the slices of a tile form one cluster and
      // sum their raw tiles through distributed shared memory
      using LK = GemmLayout<BN, 1, STAGES, 1, true, A_ROWS>;
      auto kk = umma_gemm_kernel<KIND, BN, 1, STAGES, Epi, B_MN, 1, true, kEpiWarps, A_ROWS>;
      if (gemm_resident_units(reinterpret_cast<const void*>(kk), kThreads, LK::SMEM_BYTES, 1) <= 0)
        return cudaErrorInvalidConfiguration;
      typename Epi::Params epk = ep;
      epk.partial = nullptr;
      cudaError_t ek = launch_gemm_grid(kk, kThreads, static_cast<int>(work), p.splits, LK::SMEM_BYTES, st, ta, tb, tb,
                                        static_cast<int>(g.M), static_cast<int>(g.N), static_cast<int>(p.Kp),
                                        kGroupM, idesc, epk, error_word_ptr(), p.splits);
      note_launch();
      return ek;
    }
  }
  const int units = static_cast<int>(std::min<int64_t>(work, resident));
  cudaError_t e = launch_gemm_units(kern, kThreads, CG, units, L::SMEM_BYTES, st, ta, tb, tb, static_cast<int>(g.M),
                                    static_cast<int>(g.N), static_cast<int>(p.Kp), kGroupM, idesc, ep,
                                    error_word_ptr(), p.splits);
  note_launch();
  if (e != cudaSuccess || p.splits == 1) return e;
  const int64_t total = g.M * g.N;
  const int fgrid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, num_sms() * 8)));
  fp8_splitk_finalize_kernel<TO, INT_ACC><<<fgrid, 256, 0, st>>>(partial, p.splits, g.M, g.N, g.sa, g.sb, codec_k,
                                                                 corr_row, corr_col, g.bias, g.bias_dtype,
                                                                 g.round_dtype, ra, rb, static_cast<TO*>(g.c));
  note_launch();
  return cudaGetLastError();
}

template <MmaKind KIND, int BN, bool B_MN, int CG, int A_ROWS = 128>
cudaError_t launch_fp8_out(const CUtensorMap& ta, const CUtensorMap& tb, const Fp8GemmArgs& g, const Fp8Plan& p,
                           uint32_t idesc, const int32_t* cr, const int32_t* cc, uint32_t* part, cudaStream_t st) {
  switch (g.out_dtype) {
    case F16: return launch_fp8_gemm<KIND, BN, __half, B_MN, CG, A_ROWS>(ta, tb, g, p, idesc, cr, cc, part, st);
    case BF16:
      return launch_fp8_gemm<KIND, BN, __nv_bfloat16, B_MN, CG, A_ROWS>(ta, tb, g, p, idesc, cr, cc, part, st);
    default: return launch_fp8_gemm<KIND, BN, float, B_MN, CG, A_ROWS>(ta, tb, g, p, idesc, cr, cc, part, st);
  }
}

template <MmaKind KIND, bool B_MN>
cudaError_t launch_fp8_bn(const CUtensorMap& ta, const CUtensorMap& tb, const Fp8GemmArgs& g, const Fp8Plan& p,
                          uint32_t idesc, const int32_t* cr, const int32_t* cc, uint32_t* part, cudaStream_t st) {
  if (p.bn == 256) {
    return p.cg == 2 ? launch_fp8_out<KIND, 256, B_MN, 2>(ta, tb, g, p, idesc, cr, cc, part, st)
                     : launch_fp8_out<KIND, 256, B_MN, 1>(ta, tb, g, p, idesc, cr, cc, part, st);
  }
  return p.a_rows == 32 ? launch_fp8_out<KIND, 128, B_MN, 1, 32>(ta, tb, g, p, idesc, cr, cc, part, st)
                        : launch_fp8_out<KIND, 128, B_MN, 1>(ta, tb, g, p, idesc, cr, cc, part, st);
}

}  // namespace

cudaError_t fp8_prepare_rows_launch(const void* codes, int64_t rows, int64_t K, void* dst, int32_t* sums,
                                    cudaStream_t st) {
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((rows + 7) / 8, num_sms() * 8)));
  prep_rows_s8_sum_kernel<<<grid, 256, 0, st>>>(static_cast<const uint8_t*>(codes), rows, K, static_cast<int8_t*>(dst),
                                                 sums);
  note_launch();
  return cudaGetLastError();
}

// Upper bound over operand alignments.
size_t fp8_gemm_workspace_bytes(const Fp8GemmArgs& g) {
  Fp8GemmArgs u = g;
  const Fp8Plan a = plan_fp8(u, true);
  u.K = round_up(std::max<int64_t>(g.K, 1), 16) + 1;  // forces the legacy plan's sizes
  Fp8Plan b = plan_fp8(u, false);
  b.bytes = round_up(g.M * round_up(std::max<int64_t>(g.K, 1), 16), 256) +
            round_up(g.N * round_up(std::max<int64_t>(g.K, 1), 16), 256) + (b.bytes - b.off_part);
  return std::max(a.bytes, b.bytes);
}

void fp8_gemm_tile(int64_t M, int64_t N, int64_t K, int ab_dtype, int b_layout, int32_t out[6]) {
  Fp8GemmArgs g{};
  g.M = M;
  g.N = N;
  g.K = K;
  g.ab_dtype = ab_dtype;
  g.b_layout = b_layout;
  const Fp8Plan p = plan_fp8(g, true);
  out[0] = 128 * p.cg;
  out[1] = p.bn;
  out[2] = p.cg;
  out[3] = stages_for(p.bn, p.cg, p.a_rows);
  out[4] = p.splits;
  out[5] = kGroupM;
}

cudaError_t fp8_gemm_launch(const Fp8GemmArgs& g, cudaStream_t st) {
  const Fp8Plan p = plan_fp8(g, false);
  if (g.ws_bytes < p.bytes || (p.bytes > 0 && g.ws == nullptr)) return cudaErrorInvalidValue;
  uint8_t* ws = static_cast<uint8_t*>(g.ws);
  const bool codec = (g.ab_dtype == U8);
  const uint8_t* a = static_cast<const uint8_t*>(g.a);
  const uint8_t* b = static_cast<const uint8_t*>(g.b);
  const int32_t* corr_row = nullptr;
  const int32_t* corr_col = nullptr;
  uint32_t* partial = reinterpret_cast<uint32_t*>(ws + p.off_part);
  const int prep_threads = 256;
  cudaError_t e = cudaSuccess;
  // A and B tensor-core formats: kind::i8 {0 u8, 1 s8}, kind::f8f6f4 {0 e4m3}
  uint32_t a_fmt = codec ? 1u : 0u, b_fmt = codec ? 1u : 0u;

  if (p.legacy) {
    const uint32_t flip = codec ? 0x80u : 0u;
    uint8_t* da = ws + p.off_a;
    const int64_t total_a = g.M * (p.Kp / 16);
    const int grid_a = static_cast<int>(std::min<int64_t>((total_a + prep_threads - 1) / prep_threads, num_sms() * 16));
    prep_rows_kernel<<<grid_a, prep_threads, 0, st>>>(a, g.M, g.K, g.K, da, p.Kp, flip, al16(a) && g.K % 16 == 0);
    note_launch();
    a = da;
    uint8_t* db = ws + p.off_b;
    if (g.b_layout == 0) {
      dim3 grid(static_cast<unsigned>((g.N + 63) / 64), static_cast<unsigned>((p.Kp + 63) / 64));
      prep_transpose_kernel<<<grid, 256, 0, st>>>(b, g.K, g.N, db, p.Kp, flip);
      note_launch();
    } else {
      const int64_t total_b = g.N * (p.Kp / 16);
      const int grid_b = static_cast<int>(std::min<int64_t>((total_b + prep_threads - 1) / prep_threads, num_sms() * 16));
      prep_rows_kernel<<<grid_b, prep_threads, 0, st>>>(b, g.N, g.K, g.K, db, p.Kp, flip, al16(b) && g.K % 16 == 0);
      note_launch();
    }
    b = db;
  } else if (codec && p.prep_a && g.b_s8_sums == nullptr) {
    int32_t* sums = reinterpret_cast<int32_t*>(ws + p.off_sum);
    int8_t* da = reinterpret_cast<int8_t*>(ws + p.off_a);
    const int grid = static_cast<int>(std::min<int64_t>((g.M + 7) / 8, num_sms() * 8));
    e = launch_dependent(prep_rows_s8_sum_kernel, grid, 256, st, a, g.M, g.K, da, sums);
    note_launch();
    if (e != cudaSuccess) return e;
    a = reinterpret_cast<const uint8_t*>(da);
    corr_row = sums;
    b_fmt = 0;  // B stays raw u8
  } else if (codec && g.b_s8_sums != nullptr) {
    // B prepared once by the caller: A raw u8 x B int8, corrected per column
    corr_col = g.b_s8_sums;
    a_fmt = 0;
  } else if (codec && p.prep_b) {
    int32_t* sums = reinterpret_cast<int32_t*>(ws + p.off_sum);
    int8_t* db = reinterpret_cast<int8_t*>(ws + p.off_b);
    if (g.b_layout == 0) {
      e = cudaMemsetAsync(sums, 0, static_cast<size_t>(g.N) * 4, st);
      note_launch();
      if (e != cudaSuccess) return e;
      const int64_t chunks = g.N / 16;
      const int64_t rows_per_cta = kColGroups * kColRows;
      dim3 grid(static_cast<unsigned>((chunks + kColChunks - 1) / kColChunks),
                static_cast<unsigned>((g.K + rows_per_cta - 1) / rows_per_cta));
      prep_cols_s8_sum_kernel<<<grid, kColThreads, 0, st>>>(b, g.K, g.N, db, sums);
      note_launch();
    } else {
      const int grid = static_cast<int>(std::min<int64_t>((g.N + 7) / 8, num_sms() * 8));
      e = launch_dependent(prep_rows_s8_sum_kernel, grid, 256, st, b, g.N, g.K, db, sums);
      note_launch();
      if (e != cudaSuccess) return e;
    }
    b = reinterpret_cast<const uint8_t*>(db);
    corr_col = sums;
    a_fmt = 0;  // A stays raw u8
  }
  if (g.sa_rows != nullptr || g.sb_cols != nullptr) {
    float* ra = reinterpret_cast<float*>(ws + p.off_vec);
    const double codec_k = codec ? (448.0 / 127.0) * (448.0 / 127.0) : 1.0;
    const int grid = static_cast<int>(std::min<int64_t>((g.M + g.N + 255) / 256, num_sms() * 4));
    fp8_scale_vectors_kernel<<<grid, 256, 0, st>>>(g.sa, g.sa_rows, g.sb, g.sb_cols, g.M, g.N, codec_k, ra, ra + g.M);
    note_launch();
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  CUtensorMap ta, tb;
  const int64_t lda = p.legacy ? p.Kp : g.K;
  if (!make_tmap_kmajor(&ta, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.M, lda, lda, static_cast<uint32_t>(p.a_rows)))
    return cudaErrorInvalidValue;
  if (p.b_mn) {
    // [K, N] with N contiguous: boxes of 128 bytes of N x 128 K rows
    if (!make_tmap_kmajor(&tb, b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.K, g.N, g.N, 128)) return cudaErrorInvalidValue;
  } else {
    const int64_t ldb = p.legacy ? p.Kp : g.K;
    if (!make_tmap_kmajor(&tb, b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, g.N, ldb, ldb, p.bn / p.cg))
      return cudaErrorInvalidValue;
  }
  const uint32_t c_fmt = codec ? 2u : 1u;  // s32 / f32 accumulators
  const uint32_t idesc = make_idesc(c_fmt, a_fmt, b_fmt, false, p.b_mn, 128 * p.cg, p.bn);
  if (codec) {
    return p.b_mn ? launch_fp8_bn<MmaKind::I8, true>(ta, tb, g, p, idesc, corr_row, corr_col, partial, st)
                  : launch_fp8_bn<MmaKind::I8, false>(ta, tb, g, p, idesc, corr_row, corr_col, partial, st);
  }
  return p.b_mn ? launch_fp8_bn<MmaKind::F8F6F4, true>(ta, tb, g, p, idesc, nullptr, nullptr, partial, st)
                : launch_fp8_bn<MmaKind::F8F6F4, false>(ta, tb, g, p, idesc, nullptr, nullptr, partial, st);
}

}  // namespace tfo
