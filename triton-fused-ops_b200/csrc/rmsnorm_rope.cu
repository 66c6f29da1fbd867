// Fused RMSNorm + rotate-half RoPE, one pass over each token row.
//
// Semantics follow the reference's oracle, op for op
// (triton_ops/kernels/rmsnorm_rope.py:305-383, kernel :138-235):
//   ms   = sum(x^2) / H                      (fp32)
//   rms  = sqrt(ms + eps)                    (fp32, eps rounded to fp32)
//   y    = RN_x( (x / rms) * w )             (fp32 math, rounded to x's dtype)
//   per head h, i < D/2, pos = row % S, c = cos[pos, i], s = sin[pos, i]:
//   out[h*D + i]       = RN_x( y1*c - y2*s )   (each product rounded, no FMA)
//   out[h*D + D/2 + i] = RN_x( y1*s + y2*c )
// Columns at or past num_heads*D are written as y (normalised, not rotated).
//
// Fast path: persistent CTAs stream whole rows through a shared-memory ring
// filled by bulk copies (several rows in flight per CTA at no register cost);
// the sum of squares is a warp-shuffle + one-barrier block reduction and the
// rotate-half partner is fetched with one __shfl_xor per 32-bit word.
#include "capi_internal.h"
#include "common.cuh"

namespace tfo {

// ---- packed 16-byte vector helpers ---------------------------------------
template <typename T> struct Pack;
template <> struct Pack<__half> {
  static constexpr int E = 8;
  __device__ static void unpack(const uint4& u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 p = __half22float2(h);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
  __device__ static uint32_t pack2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct Pack<__nv_bfloat16> {
  static constexpr int E = 8;
  __device__ static void unpack(const uint4& u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
      float2 p = __bfloat1622float2(h);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
  }
  __device__ static uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct Pack<float> {
  static constexpr int E = 4;
  __device__ static void unpack(const uint4& u, float (&f)[4]) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  }
};

// Round 2*W floats to T and return them packed in W 32-bit words.
template <typename T, int E>
__device__ __forceinline__ void pack_vec(const float (&f)[E], uint32_t (&w)[4]) {
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = __float_as_uint(f[i]);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = Pack<T>::pack2(f[2 * i], f[2 * i + 1]);
  }
}
template <typename T, int E>
__device__ __forceinline__ void unpack_words(const uint32_t (&w)[4], float (&f)[E]) {
  uint4 u = make_uint4(w[0], w[1], w[2], w[3]);
  Pack<T>::unpack(u, f);
}

// Load E consecutive cos/sin entries starting at p as fp32.
template <typename TCS, int E, bool CS_VEC>
__device__ __forceinline__ void load_cs(const TCS* __restrict__ p, int64_t sd, float (&f)[E]) {
  if constexpr (CS_VEC && sizeof(TCS) * E == 16) {
    uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    Pack<TCS>::unpack(u, f);
  } else if constexpr (CS_VEC && sizeof(TCS) * E == 32) {  // fp32 tables, 8 entries
    const float4* q = reinterpret_cast<const float4*>(p);
    float4 a = __ldg(q), b = __ldg(q + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
#pragma unroll
    for (int j = 0; j < E; ++j) f[j] = Ty<TCS>::to_f(p[j * sd]);
  }
}

// Correctly rounded a / b for finite a and finite b > 0, given rb = RN(1/b):
// Markstein's FMA-corrected quotient (q0 = RN(a*rb), r = a - q0*b exactly,
// q = RN(q0 + r*rb)). Three instructions instead of a full IEEE division.
__device__ __forceinline__ float div_markstein(float a, float b, float rb) {
  const float q0 = __fmul_rn(a, rb);
  const float r = __fmaf_rn(-q0, b, a);
  return __fmaf_rn(r, rb, q0);
}

// Vector path. Each CTA owns rows blockIdx.x, blockIdx.x + gridDim.x, ...;
// one thread streams them into a ring of `stages` row buffers in shared
// memory with bulk copies (mbarrier completion), so the rows in flight cost
// shared memory, not registers. Thread t handles the 16-byte vectors
// g = v*T + t (v < NV) of each row; the weight row lives in shared memory as
// fp32. The sum of squares is a warp-shuffle + one-barrier block reduction;
// right after that barrier every thread has read its vectors of the slot, so
// the slot is refilled with the row `stages` ahead.
template <typename TX, typename TCS, int NV, bool CS_VEC>
__global__ void __launch_bounds__(256) rmsnorm_rope_vec_kernel(
    const TX* __restrict__ x, const void* __restrict__ w, const TCS* __restrict__ cosp, const TCS* __restrict__ sinp,
    TX* __restrict__ out, int64_t rows, int seq_len, int hidden, int head_dim, int rot_cols, int64_t cs_ss,
    int64_t cs_sd, float eps, int w_dtype, int stages, uint32_t* err) {
  constexpr int E = Pack<TX>::E;
  const int T = blockDim.x;
  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5, nwarps = T >> 5;
  const int nvec = hidden / E;
  const int dv = head_dim / E;     // vectors per head (power of two, <= 32)
  const int hv = dv >> 1;          // rotate-half partner distance, in vectors / lanes
  const int rot_vecs = rot_cols / E;
  const uint32_t row_bytes = static_cast<uint32_t>(hidden) * sizeof(TX);

  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);                 // [stages]
  float* red = reinterpret_cast<float*>(smem + 8 * 8);                // [2][32]
  float* wsm = reinterpret_cast<float*>(smem + 8 * 8 + 2 * 32 * 4);   // [hidden]
  uint8_t* ring = smem + ((8 * 8 + 2 * 32 * 4 + hidden * 4 + 127) / 128) * 128;  // [stages][row_bytes]

  const int64_t my_rows = (rows > blockIdx.x) ? (rows - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  if (t == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  for (int i = t; i < hidden; i += T) wsm[i] = load_as_float(w, i, w_dtype);
  __syncthreads();
  if (t == 0) {
    for (int s = 0; s < stages && s < my_rows; ++s) {
      const int64_t r = blockIdx.x + static_cast<int64_t>(s) * gridDim.x;
      mbar_arrive_expect_tx(&full[s], row_bytes);
      bulk_load(ring + static_cast<size_t>(s) * row_bytes, x + r * hidden, row_bytes, &full[s]);
    }
  }

  uint4* ov = reinterpret_cast<uint4*>(out);
  int buf = 0;
  for (int64_t i = 0; i < my_rows; ++i) {
    const int64_t row = blockIdx.x + i * gridDim.x;
    const int s = static_cast<int>(i % stages);
    const uint32_t par = static_cast<uint32_t>((i / stages) & 1);
    if (!mbar_wait(&full[s], par, err, ERR_WAIT_TIMEOUT_OTHER)) break;

    const uint4* rv = reinterpret_cast<const uint4*>(ring + static_cast<size_t>(s) * row_bytes);
    uint4 cur[NV];
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int g = v * T + t;
      cur[v] = (g < nvec) ? rv[g] : make_uint4(0, 0, 0, 0);
      float f[E];
      Pack<TX>::unpack(cur[v], f);
#pragma unroll
      for (int j = 0; j < E; ++j) ss = __fmaf_rn(f[j], f[j], ss);
    }
    ss = warp_sum(ss);
    if (lane == 0) red[buf * 32 + warp] = ss;
    __syncthreads();
    // every thread has consumed slot s: refill it with the row `stages` ahead
    if (t == 0 && i + stages < my_rows) {
      fence_proxy_async_smem();
      const int64_t r = row + static_cast<int64_t>(stages) * gridDim.x;
      mbar_arrive_expect_tx(&full[s], row_bytes);
      bulk_load(ring + static_cast<size_t>(s) * row_bytes, x + r * hidden, row_bytes, &full[s]);
    }
    float tot = 0.f;
    for (int k = 0; k < nwarps; ++k) tot += red[buf * 32 + k];
    buf ^= 1;

    const float ms = __fdiv_rn(tot, static_cast<float>(hidden));
    const float rms = __fsqrt_rn(__fadd_rn(ms, eps));
    const bool fast_div = (rms > 0.f) && (rms <= 3.0e38f);  // finite, positive
    const float rb = __frcp_rn(rms);
    const int pos = static_cast<int>(row % seq_len);

#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int g = v * T + t;
      float xf[E];
      Pack<TX>::unpack(cur[v], xf);
      const float4* wv = reinterpret_cast<const float4*>(wsm + static_cast<int64_t>(min(g, nvec - 1)) * E);
      float wr[E];
#pragma unroll
      for (int q = 0; q < E / 4; ++q) {
        const float4 w4 = wv[q];
        wr[4 * q] = w4.x; wr[4 * q + 1] = w4.y; wr[4 * q + 2] = w4.z; wr[4 * q + 3] = w4.w;
      }
      // y = RN_x((x / rms) * w), kept both packed (to exchange) and as fp32
      float y[E];
#pragma unroll
      for (int j = 0; j < E; ++j) {
        const float q = fast_div ? div_markstein(xf[j], rms, rb) : __fdiv_rn(xf[j], rms);
        y[j] = __fmul_rn(q, wr[j]);
      }
      uint32_t yw[4];
      pack_vec<TX, E>(y, yw);
      unpack_words<TX, E>(yw, y);
      uint32_t pw[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) pw[k] = __shfl_xor_sync(0xffffffffu, yw[k], hv);
      if (g >= nvec) continue;

      float o[E];
      if (g < rot_vecs) {
        float p[E];
        unpack_words<TX, E>(pw, p);
        const int hi = g & (dv - 1);
        const bool first = hi < hv;
        const int i0 = (first ? hi : hi - hv) * E;
        float c[E], sn[E];
        load_cs<TCS, E, CS_VEC>(cosp + pos * cs_ss + i0 * cs_sd, cs_sd, c);
        load_cs<TCS, E, CS_VEC>(sinp + pos * cs_ss + i0 * cs_sd, cs_sd, sn);
        if (first) {
#pragma unroll
          for (int j = 0; j < E; ++j) o[j] = __fsub_rn(__fmul_rn(y[j], c[j]), __fmul_rn(p[j], sn[j]));
        } else {
#pragma unroll
          for (int j = 0; j < E; ++j) o[j] = __fadd_rn(__fmul_rn(p[j], sn[j]), __fmul_rn(y[j], c[j]));
        }
      } else {
#pragma unroll
        for (int j = 0; j < E; ++j) o[j] = y[j];
      }
      uint32_t ow[4];
      pack_vec<TX, E>(o, ow);
      __stcs(ov + row * nvec + g, make_uint4(ow[0], ow[1], ow[2], ow[3]));
    }
  }
}

// Shared memory of the vector path: barriers + reduction slots + fp32 weight
// row (128-byte aligned) + `stages` row buffers.
inline size_t vec_smem_bytes(int hidden, int row_bytes, int stages) {
  return ((8 * 8 + 2 * 32 * 4 + static_cast<size_t>(hidden) * 4 + 127) / 128) * 128 +
         static_cast<size_t>(stages) * row_bytes;
}

// Generic path: any hidden size / head_dim / alignment. One CTA per row
// (grid-stride); the row is staged in shared memory as fp32.
template <typename TX>
__global__ void __launch_bounds__(256) rmsnorm_rope_generic_kernel(
    const TX* __restrict__ x, const void* __restrict__ w, const void* __restrict__ cosp, const void* __restrict__ sinp,
    TX* __restrict__ out, int64_t rows, int seq_len, int hidden, int head_dim, int rot_cols, int64_t cs_ss,
    int64_t cs_sd, float eps, int w_dtype, int cos_dtype, int sin_dtype) {
  extern __shared__ float rowbuf[];
  __shared__ float red[32];
  const int t = threadIdx.x, T = blockDim.x;
  const int half = head_dim / 2;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const TX* xr = x + row * hidden;
    float ss = 0.f;
    for (int i = t; i < hidden; i += T) {
      const float f = Ty<TX>::to_f(xr[i]);
      rowbuf[i] = f;
      ss = __fmaf_rn(f, f, ss);
    }
    ss = warp_sum(ss);
    if ((t & 31) == 0) red[t >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int i = 0; i < (T >> 5); ++i) tot += red[i];
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(hidden)), eps));
    for (int i = t; i < hidden; i += T) {
      const float yv = __fmul_rn(__fdiv_rn(rowbuf[i], rms), load_as_float(w, i, w_dtype));
      rowbuf[i] = Ty<TX>::to_f(Ty<TX>::from_f(yv));
    }
    __syncthreads();
    const int64_t pos = row % seq_len;
    TX* orow = out + row * hidden;
    for (int i = t; i < hidden; i += T) {
      float o;
      if (i < rot_cols) {
        const int p = i % head_dim;
        const int ii = (p < half) ? p : p - half;
        const float c = load_as_float(cosp, pos * cs_ss + ii * cs_sd, cos_dtype);
        const float s = load_as_float(sinp, pos * cs_ss + ii * cs_sd, sin_dtype);
        if (p < half) {
          o = __fsub_rn(__fmul_rn(rowbuf[i], c), __fmul_rn(rowbuf[i + half], s));
        } else {
          o = __fadd_rn(__fmul_rn(rowbuf[i - half], s), __fmul_rn(rowbuf[i], c));
        }
      } else {
        o = rowbuf[i];
      }
      orow[i] = Ty<TX>::from_f(o);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// host dispatch
// ---------------------------------------------------------------------------
namespace {

template <typename TX, typename TCS, int NV, bool CS_VEC>
cudaError_t launch_vec(const RmsNormRopeArgs& a, int threads, cudaStream_t st) {
  auto kern = rmsnorm_rope_vec_kernel<TX, TCS, NV, CS_VEC>;
  const int row_bytes = static_cast<int>(a.hidden * sizeof(TX));
  // ring of up to 8 rows, about 48 KB, at least 2
  const int stages = std::max(2, std::min(8, (48 * 1024) / row_bytes));
  const size_t smem = vec_smem_bytes(static_cast<int>(a.hidden), row_bytes, stages);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const int occ = cached_occupancy(reinterpret_cast<const void*>(kern), threads, smem);
  const int64_t rows = a.batch * a.seq_len;
  const int64_t grid = std::min<int64_t>(rows, static_cast<int64_t>(num_sms()) * std::max(occ, 1));
  kern<<<static_cast<unsigned>(grid), threads, smem, st>>>(
      static_cast<const TX*>(a.x), a.weight, static_cast<const TCS*>(a.cos), static_cast<const TCS*>(a.sin),
      static_cast<TX*>(a.out), rows, static_cast<int>(a.seq_len), static_cast<int>(a.hidden),
      static_cast<int>(a.head_dim), static_cast<int>(a.num_heads * a.head_dim), a.cs_stride_seq, a.cs_stride_dim,
      a.eps, a.w_dtype, stages, error_word_ptr());
  note_launch();
  return cudaGetLastError();
}

template <typename TX, typename TCS, bool CS_VEC>
cudaError_t pick_nv(const RmsNormRopeArgs& a, int nvec, cudaStream_t st) {
  for (int nv : {1, 2, 4, 8}) {
    const int threads = ((nvec + nv - 1) / nv + 31) / 32 * 32;
    if (threads <= 256) {
      switch (nv) {
        case 1: return launch_vec<TX, TCS, 1, CS_VEC>(a, threads, st);
        case 2: return launch_vec<TX, TCS, 2, CS_VEC>(a, threads, st);
        case 4: return launch_vec<TX, TCS, 4, CS_VEC>(a, threads, st);
        default: return launch_vec<TX, TCS, 8, CS_VEC>(a, threads, st);
      }
    }
  }
  return cudaErrorInvalidConfiguration;
}

template <typename TX>
cudaError_t dispatch_cs(const RmsNormRopeArgs& a, int nvec, bool cs_vec, cudaStream_t st) {
  switch (a.cos_dtype) {
    case F16: return cs_vec ? pick_nv<TX, __half, true>(a, nvec, st) : pick_nv<TX, __half, false>(a, nvec, st);
    case BF16:
      return cs_vec ? pick_nv<TX, __nv_bfloat16, true>(a, nvec, st) : pick_nv<TX, __nv_bfloat16, false>(a, nvec, st);
    default: return cs_vec ? pick_nv<TX, float, true>(a, nvec, st) : pick_nv<TX, float, false>(a, nvec, st);
  }
}

template <typename TX>
cudaError_t launch_generic(const RmsNormRopeArgs& a, cudaStream_t st) {
  const int64_t rows = a.batch * a.seq_len;
  const size_t smem = static_cast<size_t>(a.hidden) * sizeof(float);
  auto kern = rmsnorm_rope_generic_kernel<TX>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(reinterpret_cast<const void*>(kern),
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const int occ = cached_occupancy(reinterpret_cast<const void*>(kern), 256, smem);
  const int64_t grid = std::min<int64_t>(rows, static_cast<int64_t>(num_sms()) * std::max(occ, 1));
  kern<<<static_cast<unsigned>(grid), 256, smem, st>>>(
      static_cast<const TX*>(a.x), a.weight, a.cos, a.sin, static_cast<TX*>(a.out), rows,
      static_cast<int>(a.seq_len), static_cast<int>(a.hidden), static_cast<int>(a.head_dim),
      static_cast<int>(a.num_heads * a.head_dim), a.cs_stride_seq, a.cs_stride_dim, a.eps, a.w_dtype, a.cos_dtype,
      a.sin_dtype);
  note_launch();
  return cudaGetLastError();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// Chooses the vectorised path when the row, head and table layout allow it.
cudaError_t rmsnorm_rope_launch(const RmsNormRopeArgs& a, cudaStream_t st) {
  const int esz = (a.x_dtype == F32) ? 4 : 2;
  const int E = 16 / esz;
  const int64_t D = a.head_dim;
  const int64_t dv = D / E;
  bool vec = aligned16(a.x) && aligned16(a.out) && (a.hidden % E == 0) && (D % (2 * E) == 0) && dv >= 2 &&
             dv <= 32 && (dv & (dv - 1)) == 0 && (a.hidden / E) <= 8 * 256 && a.cos_dtype == a.sin_dtype;
  if (vec) {
    const int csz = (a.cos_dtype == F32) ? 4 : 2;
    const bool cs_vec = a.cs_stride_dim == 1 && aligned16(a.cos) && aligned16(a.sin) &&
                        ((a.cs_stride_seq * csz) % 16 == 0) && ((E * csz) % 16 == 0);
    const int nvec = static_cast<int>(a.hidden / E);
    switch (a.x_dtype) {
      case F16: return dispatch_cs<__half>(a, nvec, cs_vec, st);
      case BF16: return dispatch_cs<__nv_bfloat16>(a, nvec, cs_vec, st);
      default: return dispatch_cs<float>(a, nvec, cs_vec, st);
    }
  }
  switch (a.x_dtype) {
    case F16: return launch_generic<__half>(a, st);
    case BF16: return launch_generic<__nv_bfloat16>(a, st);
    default: return launch_generic<float>(a, st);
  }
}

}  // namespace tfo
