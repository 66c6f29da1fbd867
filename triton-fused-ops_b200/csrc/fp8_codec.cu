// FP8 codec kernels: per-tensor amax -> scale, encode, decode.
//
// Two 8-bit encodings are produced from the same scaled value c = fp32(x)*s:
//  * the reference codec ("uint8"), bit-exact with
//    triton_ops/kernels/fp8_quantize.py:258-287:
//        u = uint8( int8( rint( RN(RN(clamp(c, +-448) / 448) * 127) ) ) + 128 )
//  * true e4m3fn bytes: RN_e4m3( clamp(c, +-448) ), saturating, NaN kept.
// The dynamic scale follows triton_ops/models.py:282-299: amax = max|x| (in
// x's dtype), scale = fp32(448.0 / double(amax)), or 1.0 when amax == 0.
//
// Pipeline for a dynamic scale (no host sync, no zero-initialised memory):
//   amax_partial_kernel : grid-stride max|x|, one partial per CTA
//   encode kernel       : every CTA reduces the partials (a few KB from L2),
//                         derives the scale in double, CTA 0 publishes it,
//                         then encodes its share of the tensor.
// The second read of x is served by L2 for tensors that fit in it.
#include <cuda.h>

#include <mutex>
#include <string>

#include "capi_internal.h"
#include "codec.cuh"
#include "common.cuh"
#include "tfo_b200.h"

namespace tfo {

// ---- 16 elements at a time -------------------------------------------------
// A chunk is 16 consecutive elements: two 16-byte vectors for 16-bit types,
// four for fp32. Loads are issued for several chunks before any of them is
// used, so each thread keeps that many vectors in flight.
template <typename T> struct Chunk {
  static constexpr int VECS = 16 * static_cast<int>(sizeof(T)) / 16;
  uint4 v[VECS];
  template <bool STREAM>
  __device__ __forceinline__ void load(const T* p) {
    const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int i = 0; i < VECS; ++i) v[i] = STREAM ? __ldcs(q + i) : __ldg(q + i);
  }
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < VECS; ++i) v[i] = make_uint4(0u, 0u, 0u, 0u);
  }
  __device__ __forceinline__ void to_f(float (&f)[16]) const {
#pragma unroll
    for (int i = 0; i < VECS; ++i) {
      const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if constexpr (std::is_same<T, float>::value) {
          f[4 * i + j] = __uint_as_float(w[j]);
        } else if constexpr (std::is_same<T, __half>::value) {
          const float2 p2 = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
          f[8 * i + 2 * j] = p2.x;
          f[8 * i + 2 * j + 1] = p2.y;
        } else {
          const float2 p2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
          f[8 * i + 2 * j] = p2.x;
          f[8 * i + 2 * j + 1] = p2.y;
        }
      }
    }
  }
};

// max |x| over this thread's share of x, as the fp32 bit pattern (|x| >= 0
// orders like its bits; NaN bits exceed every finite value, as in torch's max).
// Chunk i belongs to thread i mod stride; U chunks are loaded per iteration.
// The vector part compares the sign-cleared bit patterns directly (per 16-bit
// lane for 16-bit types, vmax.u16x2), which orders them like |x| without
// converting any element; the larger lane is converted once at the end.
template <typename T, int U>
__device__ __forceinline__ uint32_t amax_share(const T* __restrict__ x, int64_t n, bool vec, int64_t tid,
                                               int64_t stride) {
  uint32_t mv = 0;  // absmax_vec lanes
  int64_t done = 0;
  if (vec) {
    const int64_t n16 = n / 16;
    for (int64_t i = tid; i < n16; i += U * stride) {
      Chunk<T> c[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (i + u * stride < n16) c[u].template load<false>(x + (i + u * stride) * 16);
        else c[u].zero();
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
#pragma unroll
        for (int q = 0; q < Chunk<T>::VECS; ++q) mv = absmax_vec<T>(mv, c[u].v[q]);
      }
    }
    done = n16 * 16;
  }
  uint32_t m = absmax_to_f32_bits<T>(mv);
  for (int64_t i = done + tid; i < n; i += stride) m = max(m, __float_as_uint(fabsf(Ty<T>::to_f(x[i]))));
  return m;
}

// Encodes this thread's share of x with scale s (chunk i -> thread i mod stride).
// IN_RANGE: every |x * s| <= 448 + 1 ulp (a finite, non-zero dynamic scale).
// For e4m3 the clamp to +-448 is the satfinite conversion itself (NaN stays
// NaN, +-inf -> +-448), so both variants convert pairs directly.
template <typename T, bool E4M3, int U, bool IN_RANGE>
__device__ __forceinline__ void encode_share(const T* __restrict__ x, int64_t n, bool vec, float s,
                                             uint8_t* __restrict__ out, int64_t tid, int64_t stride) {
  auto enc1 = [s](float xf) -> uint32_t {
    const float c = __fmul_rn(xf, s);
    if constexpr (E4M3) {
      return static_cast<uint32_t>(__nv_cvt_float_to_fp8(c, __NV_SATFINITE, __NV_E4M3));
    } else {
      return ref_encode(c);
    }
  };
  auto enc4 = [s, &enc1](const float* f) -> uint32_t {
    if constexpr (E4M3) {
      const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(__fmul_rn(f[0], s), __fmul_rn(f[1], s)),
                                                   __NV_SATFINITE, __NV_E4M3);
      const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(__fmul_rn(f[2], s), __fmul_rn(f[3], s)),
                                                   __NV_SATFINITE, __NV_E4M3);
      return lo | (hi << 16);
    } else if constexpr (IN_RANGE) {
      return ref_encode4_in_range_scaled(f, s);
    } else {
      return enc1(f[0]) | (enc1(f[1]) << 8) | (enc1(f[2]) << 16) | (enc1(f[3]) << 24);
    }
  };
  int64_t done = 0;
  if (vec) {
    const int64_t n16 = n / 16;
    for (int64_t i = tid; i < n16; i += U * stride) {
      Chunk<T> c[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (i + u * stride < n16) c[u].template load<true>(x + (i + u * stride) * 16);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (i + u * stride < n16) {
          float f[16];
          c[u].to_f(f);
          uint32_t w[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) w[q] = enc4(f + 4 * q);
          __stcs(reinterpret_cast<uint4*>(out) + i + u * stride, make_uint4(w[0], w[1], w[2], w[3]));
        }
      }
    }
    done = n16 * 16;
  }
  for (int64_t i = done + tid; i < n; i += stride) out[i] = static_cast<uint8_t>(enc1(Ty<T>::to_f(x[i])));
}

// ---- amax (scale-only calls and the no-allocation quantize) ----------------
constexpr int kAmaxThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kAmaxThreads) amax_partial_kernel(const T* __restrict__ x, int64_t n, bool vec,
                                                                     uint32_t* __restrict__ partials) {
  griddep_launch_dependents();  // the encode that follows may be scheduled early
  __shared__ uint32_t red[32];
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const uint32_t b = block_max_u32(amax_share<T, 4>(x, n, vec, tid, stride), red);
  if (threadIdx.x == 0) partials[blockIdx.x] = b;
}

__global__ void finalize_scale_kernel(const uint32_t* __restrict__ partials, int nparts, float* __restrict__ scale_out) {
  __shared__ uint32_t red[32];
  const float s = reduce_partials_to_scale(partials, nparts, red);
  if (threadIdx.x == 0) *scale_out = s;
}

// ---- encode with a given scale, or from amax partials ----------------------
constexpr int kEncThreads = 256;

template <typename T, bool E4M3>
__global__ void __launch_bounds__(kEncThreads) encode_kernel(const T* __restrict__ x, int64_t n, bool vec,
                                                             const float* __restrict__ scale_in,
                                                             const uint32_t* __restrict__ partials, int nparts,
                                                             float* __restrict__ scale_out, uint8_t* __restrict__ out) {
  griddep_launch_dependents();  // a programmatic-dependent GEMM that follows may be scheduled early
  griddep_wait();               // launched as a programmatic dependent: inputs are read after this
  __shared__ float s_sh;
  __shared__ uint32_t red[32];
  if (partials != nullptr) {
    const float s = reduce_partials_to_scale(partials, nparts, red);
    if (threadIdx.x == 0) {
      s_sh = s;
      if (blockIdx.x == 0 && scale_out != nullptr) *scale_out = s;
    }
  } else if (threadIdx.x == 0) {
    s_sh = *scale_in;
  }
  __syncthreads();
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const float s = s_sh;
  if (partials != nullptr && s > 0.f && s < INFINITY) encode_share<T, E4M3, 2, true>(x, n, vec, s, out, tid, stride);
  else encode_share<T, E4M3, 2, false>(x, n, vec, s, out, tid, stride);
}

// ---- dynamic-scale quantize in one kernel ----------------------------------
// Cooperative launch (all CTAs resident). Pass 1: each CTA folds its max |x|
// into one global word and arrives on a counter (both in the workspace,
// zeroed by the host before the launch); after the grid barrier every CTA
// reads the max, derives the scale (CTA 0 publishes it) and, in pass 2,
// encodes the same elements it read in pass 1, which for tensors up to the L2
// size come back from L2 rather than HBM. The barrier wait is bounded: on
// expiry the CTA sets ERR_GRID_BARRIER and returns without writing its share
// of the output.
constexpr int kQuantThreads = 512;

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide max and scale with a single global word: every CTA folds its max
// into barrier[1] (atomicMax on the bits of a non-negative float orders like
// the value, NaN above inf), then arrives on the counter barrier[0]; both
// words are zeroed by the host before the launch. After the (bounded) wait one
// load gives the max. Returns false if the wait ran out of budget
// (ERR_GRID_BARRIER set; the caller must not write its output).
__device__ __forceinline__ bool grid_max_scale(uint32_t b, uint32_t* __restrict__ barrier, uint32_t* __restrict__ err,
                                               float* s_sh, int* ok_sh) {
  if (threadIdx.x == 0) {
    atomicMax(barrier + 1, b);
    __threadfence();
    atomicAdd(barrier, 1u);
    int ok = 1;
    if (ld_acquire_gpu(barrier) < gridDim.x) {
      const long long t0 = clock64();
      while (ld_acquire_gpu(barrier) < gridDim.x) {
        if (clock64() - t0 > kWaitBudgetCycles) {
          set_error(err, ERR_GRID_BARRIER);
          ok = 0;
          break;
        }
        __nanosleep(32);
      }
    }
    *ok_sh = ok;
    *s_sh = scale_from_amax(ld_acquire_gpu(barrier + 1));
  }
  __syncthreads();
  return *ok_sh != 0;
}

template <typename T, bool E4M3>
__global__ void __launch_bounds__(kQuantThreads, 2)
    quantize_dynamic_kernel(const T* __restrict__ x, int64_t n, bool vec, uint32_t* __restrict__ barrier,
                            float* __restrict__ scale_out,
                            uint8_t* __restrict__ out, uint32_t* __restrict__ err) {
  griddep_launch_dependents();  // a programmatic-dependent GEMM that follows may be scheduled early
  __shared__ uint32_t red[32];
  __shared__ float s_sh;
  __shared__ int ok_sh;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const uint32_t b = block_max_u32(amax_share<T, 4>(x, n, vec, tid, stride), red);
  if (!grid_max_scale(b, barrier, err, &s_sh, &ok_sh)) return;
  const float sc = s_sh;
  if (threadIdx.x == 0 && blockIdx.x == 0) *scale_out = sc;
  if (sc > 0.f && sc < INFINITY) encode_share<T, E4M3, 2, true>(x, n, vec, sc, out, tid, stride);
  else encode_share<T, E4M3, 2, false>(x, n, vec, sc, out, tid, stride);
}

// Codes of the EV = 16 / sizeof(T) elements of one 16-byte vector q at scale
// s (in_range: s finite and non-zero, so every |x * s| <= 448 + 1 ulp and the
// clamp can be skipped); w[0] (and w[1] for 16-bit T) receive the bytes in
// element order.
template <typename T, bool E4M3>
__device__ __forceinline__ void encode_vec16(const uint4& q, float s, bool in_range, uint32_t (&w)[2]) {
  constexpr int EV = 16 / sizeof(T);
  Chunk<T> c;  // reuse the 16-element converter on half a chunk for 16-bit types
#pragma unroll
  for (int i = 0; i < Chunk<T>::VECS; ++i) c.v[i] = q;
  float f[16];
  c.to_f(f);
  if constexpr (E4M3) {
#pragma unroll
    for (int h = 0; h < EV / 4; ++h) {
      const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(__fmul_rn(f[4 * h], s), __fmul_rn(f[4 * h + 1], s)),
                                                   __NV_SATFINITE, __NV_E4M3);
      const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(__fmul_rn(f[4 * h + 2], s), __fmul_rn(f[4 * h + 3], s)),
                                                   __NV_SATFINITE, __NV_E4M3);
      w[h] = lo | (hi << 16);
    }
  } else if (in_range) {
#pragma unroll
    for (int h = 0; h < EV / 4; ++h) w[h] = ref_encode4_in_range_scaled(f + 4 * h, s);
  } else {
#pragma unroll
    for (int h = 0; h < EV / 4; ++h)
      w[h] = ref_encode(__fmul_rn(f[4 * h], s)) | (ref_encode(__fmul_rn(f[4 * h + 1], s)) << 8) |
             (ref_encode(__fmul_rn(f[4 * h + 2], s)) << 16) | (ref_encode(__fmul_rn(f[4 * h + 3], s)) << 24);
  }
}

template <typename T>
__device__ __forceinline__ void store_codes16(uint8_t* out, int64_t v, const uint32_t (&w)[2]) {
  if constexpr (sizeof(T) == 2) reinterpret_cast<uint2*>(out)[v] = make_uint2(w[0], w[1]);
  else reinterpret_cast<uint32_t*>(out)[v] = w[0];
}

// ---- dynamic-scale quantize of small tensors: one cluster, no grid barrier --
// For 16-byte-aligned tensors of whole vectors, up to kSmallMaxCtas x
// kSmallThreads x kSmallVecs vectors (1 MB of fp16), the size of decode-step
// activations: one cluster of C <= kSmallMaxCtas CTAs (enough for
// kSmallMinVecs vectors per thread). Each thread loads its (at most
// kSmallVecs) vectors into registers, all loads in flight at once;
// the CTA maxima meet through distributed shared memory between two cluster
// barriers; every CTA then encodes its vectors from registers. No memset, no
// global atomics, no cooperative launch: through the grid-barrier forms one
// 4096-element row took 6.2 us. Same amax, scale and encode as the other
// forms, so the bytes are identical.
constexpr int kSmallThreads = 512;
constexpr int kSmallVecs = 16;     // vectors per thread at most (held in registers)
constexpr int kSmallMinVecs = 2;   // vectors per thread below which fewer CTAs are used
constexpr int kSmallMaxCtas = 8;

__device__ __forceinline__ uint32_t ld_cluster_u32(uint32_t cluster_addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(cluster_addr) : "memory");
  return v;
}

template <typename T, bool E4M3>
__global__ void __launch_bounds__(kSmallThreads, 1)
    quantize_small_kernel(const T* __restrict__ x, int64_t nvec, float* __restrict__ scale_out,
                          uint8_t* __restrict__ out) {
  griddep_launch_dependents();  // a programmatic-dependent GEMM that follows may be scheduled early
  griddep_wait();               // launched as a programmatic dependent: x is read after this
  __shared__ uint32_t red[32];
  __shared__ uint32_t cta_max;
  // vector i of this thread: base + i * stride (the cluster's threads in turn)
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kSmallThreads + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kSmallThreads;
  uint4 q[kSmallVecs];
#pragma unroll
  for (int i = 0; i < kSmallVecs; ++i)
    if (base + i * stride < nvec) q[i] = __ldcs(reinterpret_cast<const uint4*>(x) + base + i * stride);
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < kSmallVecs; ++i)
    if (base + i * stride < nvec) m = absmax_vec<T>(m, q[i]);
  const uint32_t bmax = block_max_u32(absmax_to_f32_bits<T>(m), red);
  if (threadIdx.x == 0) cta_max = bmax;
  cluster_sync();  // every CTA's maximum is in its shared memory
  uint32_t g = 0;
  for (int r = 0; r < static_cast<int>(gridDim.x); ++r)
    g = max(g, ld_cluster_u32(mapa_shared(smem_u32(&cta_max), static_cast<uint32_t>(r))));
  cluster_sync();  // no CTA leaves while another may still read its maximum
  const float s = scale_from_amax(g);
  if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = s;
  const bool in_range = (s > 0.f && s < INFINITY);
#pragma unroll
  for (int i = 0; i < kSmallVecs; ++i) {
    if (base + i * stride < nvec) {
      uint32_t w[2];
      encode_vec16<T, E4M3>(q[i], s, in_range, w);
      store_codes16<T>(out, base + i * stride, w);
    }
  }
}

// Bit pattern of v rounded to TO (16 bits for fp16/bf16, 32 for fp32).
template <typename TO> struct Raw { using type = uint16_t; };
template <> struct Raw<float> { using type = uint32_t; };

template <typename TO>
__device__ __forceinline__ typename Raw<TO>::type to_raw(float v) {
  if constexpr (sizeof(TO) == 4) {
    return __float_as_uint(v);
  } else {
    TO h = Ty<TO>::from_f(v);
    return *reinterpret_cast<uint16_t*>(&h);
  }
}

// ---- per-row (per-token / per-channel) scales ------------------------------
// One warp per row of a [rows, cols] matrix (row-major, contiguous).
constexpr int kRowThreads = 256;

// scales[r] = 448 / max|x[r, :]| as FP8Format.compute_scale_per_channel
// (triton_ops/models.py:301-314) evaluates it in torch: a zero max counts as
// 1, and `448.0 / t` is `t.reciprocal() * 448`, each step rounded to x's dtype
// (computed in fp32 first). The value is stored as fp32.
template <typename T>
__global__ void __launch_bounds__(kRowThreads) row_scales_kernel(const T* __restrict__ x, int64_t rows, int64_t cols,
                                                                 bool vec, float* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * kRowThreads + threadIdx.x) >> 5; r < rows;
       r += (static_cast<int64_t>(gridDim.x) * kRowThreads) >> 5) {
    uint32_t m = 0;
    const T* xr = x + r * cols;
    if (vec) {  // rows of whole 16-element chunks, 16-byte aligned: two chunks in flight per lane
      const int64_t cpr = cols / 16;
      for (int64_t c = lane; c < cpr; c += 64) {
        Chunk<T> a, b;
        a.template load<false>(xr + c * 16);
        if (c + 32 < cpr) b.template load<false>(xr + (c + 32) * 16);
        else b.zero();
        float f[16];
        a.to_f(f);
#pragma unroll
        for (int j = 0; j < 16; ++j) m = max(m, __float_as_uint(fabsf(f[j])));
        b.to_f(f);
#pragma unroll
        for (int j = 0; j < 16; ++j) m = max(m, __float_as_uint(fabsf(f[j])));
      }
    } else {
      for (int64_t c = lane; c < cols; c += 32) m = max(m, __float_as_uint(fabsf(Ty<T>::to_f(xr[c]))));
    }
    m = warp_max_u32(m);
    if (lane == 0) {
      const float amax = __uint_as_float(m);
      const float rcp = Ty<T>::to_f(Ty<T>::from_f(__frcp_rn(amax == 0.f ? 1.0f : amax)));
      scales[r] = Ty<T>::to_f(Ty<T>::from_f(__fmul_rn(rcp, 448.0f)));
    }
  }
}

// Codes of x[r, c] * scales[r] (reference codec: clamp, NaN kept; or e4m3).
// VEC: x and out 16-byte aligned and cols a multiple of 16, so each thread
// takes one 16-element chunk (one row, one scale) and stores 16 codes at once.
template <typename T, bool E4M3>
__global__ void __launch_bounds__(kRowThreads) encode_rows_kernel(const T* __restrict__ x, int64_t rows, int64_t cols,
                                                                  bool vec, const float* __restrict__ scales,
                                                                  uint8_t* __restrict__ out) {
  griddep_launch_dependents();  // a programmatic-dependent GEMM that follows may be scheduled early
  auto enc1 = [](float c) -> uint32_t {
    return E4M3 ? static_cast<uint32_t>(__nv_cvt_float_to_fp8(c, __NV_SATFINITE, __NV_E4M3)) : ref_encode(c);
  };
  const int64_t n = rows * cols;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * kRowThreads + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kRowThreads;
  if (vec) {
    const int64_t cpr = cols / 16;
    for (int64_t i = tid; i < n / 16; i += stride) {
      Chunk<T> c;
      c.template load<true>(x + i * 16);
      const float s = __ldg(scales + i / cpr);
      float f[16];
      c.to_f(f);
      uint32_t w[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if constexpr (E4M3) {
          const uint32_t lo = __nv_cvt_float2_to_fp8x2(
              make_float2(__fmul_rn(f[4 * q], s), __fmul_rn(f[4 * q + 1], s)), __NV_SATFINITE, __NV_E4M3);
          const uint32_t hi = __nv_cvt_float2_to_fp8x2(
              make_float2(__fmul_rn(f[4 * q + 2], s), __fmul_rn(f[4 * q + 3], s)), __NV_SATFINITE, __NV_E4M3);
          w[q] = lo | (hi << 16);
        } else {
          w[q] = enc1(__fmul_rn(f[4 * q], s)) | (enc1(__fmul_rn(f[4 * q + 1], s)) << 8) |
                 (enc1(__fmul_rn(f[4 * q + 2], s)) << 16) | (enc1(__fmul_rn(f[4 * q + 3], s)) << 24);
        }
      }
      __stcs(reinterpret_cast<uint4*>(out) + i, make_uint4(w[0], w[1], w[2], w[3]));
    }
    return;
  }
  for (int64_t i = tid; i < n; i += stride)
    out[i] = static_cast<uint8_t>(enc1(__fmul_rn(Ty<T>::to_f(x[i]), __ldg(scales + i / cols))));
}

// ---- per-token dynamic quantize: row scales and codes in one launch --------
// One warp per row: max |x| over the row (the element-wise fp32 maxima of
// row_scales_kernel), the row's scale with row_scales_kernel's rounding,
// written in x's dtype (the value compute_scale_per_channel returns), then
// the row encoded with that scale exactly as encode_rows_kernel does. Rows of
// up to 32 x kTokRegChunks chunks are loaded into registers at once and
// encoded from there; longer rows are read again (an L2 hit: this warp has
// just read them). One HBM read of x instead of two, and one launch instead
// of three (row scales, the cast of the scales to x's dtype, the encode).
template <typename T, bool E4M3>
__device__ __forceinline__ uint4 encode_chunk_scaled(const Chunk<T>& c, float s) {
  float f[16];
  c.to_f(f);
  uint32_t w[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if constexpr (E4M3) {
      const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(__fmul_rn(f[4 * q], s), __fmul_rn(f[4 * q + 1], s)),
                                                   __NV_SATFINITE, __NV_E4M3);
      const uint32_t hi = __nv_cvt_float2_to_fp8x2(
          make_float2(__fmul_rn(f[4 * q + 2], s), __fmul_rn(f[4 * q + 3], s)), __NV_SATFINITE, __NV_E4M3);
      w[q] = lo | (hi << 16);
    } else {
      w[q] = ref_encode(__fmul_rn(f[4 * q], s)) | (ref_encode(__fmul_rn(f[4 * q + 1], s)) << 8) |
             (ref_encode(__fmul_rn(f[4 * q + 2], s)) << 16) | (ref_encode(__fmul_rn(f[4 * q + 3], s)) << 24);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Reference-codec bytes of a chunk whose every |x * s| stays below 449.76
// (see quantize_rows_dynamic_kernel): the in-range encode, no clamp.
template <typename T>
__device__ __forceinline__ uint4 encode_chunk_in_range(const Chunk<T>& c, float s) {
  float f[16];
  c.to_f(f);
  return make_uint4(ref_encode4_in_range_scaled(f, s), ref_encode4_in_range_scaled(f + 4, s),
                    ref_encode4_in_range_scaled(f + 8, s), ref_encode4_in_range_scaled(f + 12, s));
}

// 16-element chunks per lane that the per-token kernel holds in registers
// (a 4096-column 16-bit row, a 2048-column fp32 row: 64 registers of data)
template <typename T>
constexpr int kTokRegChunks = sizeof(T) == 4 ? 4 : 8;

template <typename T, bool E4M3>
__global__ void __launch_bounds__(kRowThreads) quantize_rows_dynamic_kernel(const T* __restrict__ x, int64_t rows,
                                                                            int64_t cols, bool vec,
                                                                            T* __restrict__ scales_out,
                                                                            uint8_t* __restrict__ out) {
  griddep_launch_dependents();  // a programmatic-dependent GEMM that follows may be scheduled early
  const int lane = threadIdx.x & 31;
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * kRowThreads + threadIdx.x) >> 5; r < rows;
       r += (static_cast<int64_t>(gridDim.x) * kRowThreads) >> 5) {
    const T* xr = x + r * cols;
    uint8_t* orow = out + r * cols;
    uint32_t m = 0;
    const int64_t cpr = cols / 16;
    // bf16 rows keep the loop below: held in registers they measured slower
    // ([4096, 4096]: 15.0 against 13.6 us), fp16 faster (13.6 -> 12.2 us)
    if (vec && cpr <= 32 * kTokRegChunks<T> && !std::is_same<T, __nv_bfloat16>::value) {
      // the whole row in registers: every load in flight at once, one read of x
      Chunk<T> ch[kTokRegChunks<T>];
#pragma unroll
      for (int k = 0; k < kTokRegChunks<T>; ++k)
        if (lane + 32 * k < cpr) ch[k].template load<false>(xr + (lane + 32 * k) * 16);
#pragma unroll
      for (int k = 0; k < kTokRegChunks<T>; ++k) {
        if (lane + 32 * k < cpr) {
          float f[16];
          ch[k].to_f(f);
#pragma unroll
          for (int j = 0; j < 16; ++j) m = max(m, __float_as_uint(fabsf(f[j])));
        }
      }
      m = warp_max_u32(m);
      const float amax = __uint_as_float(m);
      const float rcp = Ty<T>::to_f(Ty<T>::from_f(__frcp_rn(amax == 0.f ? 1.0f : amax)));
      const float s = Ty<T>::to_f(Ty<T>::from_f(__fmul_rn(rcp, 448.0f)));
      if (lane == 0) scales_out[r] = Ty<T>::from_f(s);
      const bool in_range = !E4M3 && amax < INFINITY && s > 0.f && s < INFINITY && __fmul_rn(amax, s) <= 449.0f;
      // one branch per row (warp-uniform), each side with its own unrolled loop
      if (in_range) {
#pragma unroll
        for (int k = 0; k < kTokRegChunks<T>; ++k)
          if (lane + 32 * k < cpr) __stcs(reinterpret_cast<uint4*>(orow) + lane + 32 * k, encode_chunk_in_range<T>(ch[k], s));
      } else {
#pragma unroll
        for (int k = 0; k < kTokRegChunks<T>; ++k)
          if (lane + 32 * k < cpr)
            __stcs(reinterpret_cast<uint4*>(orow) + lane + 32 * k, encode_chunk_scaled<T, E4M3>(ch[k], s));
      }
      continue;
    }
    if (vec) {  // rows of whole 16-element chunks, 16-byte aligned: two chunks in flight per lane
      for (int64_t c = lane; c < cpr; c += 64) {
        Chunk<T> a, b;
        a.template load<false>(xr + c * 16);
        if (c + 32 < cpr) b.template load<false>(xr + (c + 32) * 16);
        else b.zero();
        float f[16];
        a.to_f(f);
#pragma unroll
        for (int j = 0; j < 16; ++j) m = max(m, __float_as_uint(fabsf(f[j])));
        b.to_f(f);
#pragma unroll
        for (int j = 0; j < 16; ++j) m = max(m, __float_as_uint(fabsf(f[j])));
      }
    } else {
      for (int64_t c = lane; c < cols; c += 32) m = max(m, __float_as_uint(fabsf(Ty<T>::to_f(xr[c]))));
    }
    m = warp_max_u32(m);
    const float amax = __uint_as_float(m);
    const float rcp = Ty<T>::to_f(Ty<T>::from_f(__frcp_rn(amax == 0.f ? 1.0f : amax)));
    const float s = Ty<T>::to_f(Ty<T>::from_f(__fmul_rn(rcp, 448.0f)));
    if (lane == 0) scales_out[r] = Ty<T>::from_f(s);
    // Reference codec: s is 448 / amax within a few roundings in x's dtype,
    // so RN(amax * s) is close to 448. When it is at most 449, every
    // |RN(x * s)| <= RN(amax * s) <= 449 < 448 * 127.5 / 127 (RN is monotonic),
    // so rint(RN(RN(c / 448) * 127)) equals the clamped value's code and the
    // unclamped in-range encode gives the same bytes. fp16 and fp32 rows always
    // pass (at most 0.25 % high); bf16 rows whose two roundings push the
    // product past 449, and non-finite amax or scales, keep the clamped encode.
    const bool in_range = !E4M3 && amax < INFINITY && s > 0.f && s < INFINITY && __fmul_rn(amax, s) <= 449.0f;
    if (vec) {
      for (int64_t c = lane; c < cpr; c += 64) {
        Chunk<T> a, b;
        const bool has_b = c + 32 < cpr;
        a.template load<false>(xr + c * 16);
        if (has_b) b.template load<false>(xr + (c + 32) * 16);
        if (in_range) {
          __stcs(reinterpret_cast<uint4*>(orow) + c, encode_chunk_in_range<T>(a, s));
          if (has_b) __stcs(reinterpret_cast<uint4*>(orow) + c + 32, encode_chunk_in_range<T>(b, s));
        } else {
          __stcs(reinterpret_cast<uint4*>(orow) + c, encode_chunk_scaled<T, E4M3>(a, s));
          if (has_b) __stcs(reinterpret_cast<uint4*>(orow) + c + 32, encode_chunk_scaled<T, E4M3>(b, s));
        }
      }
    } else {
      for (int64_t c = lane; c < cols; c += 32) {
        const float v = __fmul_rn(Ty<T>::to_f(xr[c]), s);
        orow[c] = static_cast<uint8_t>(
            E4M3 ? static_cast<uint32_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3)) : ref_encode(v));
      }
    }
  }
}

// out[r, c] = dec(q[r, c]) / scales[r], dec as in the per-tensor decode.
// VEC: q and out 16-byte aligned and cols a multiple of 16, so each thread
// takes one 16-code vector (one row, one scale) and stores its outputs as
// 16-byte vectors.
template <typename TO, bool E4M3>
__global__ void __launch_bounds__(kRowThreads) decode_rows_kernel(const uint8_t* __restrict__ q, int64_t rows,
                                                                  int64_t cols, bool vec,
                                                                  const float* __restrict__ scales,
                                                                  TO* __restrict__ out) {
  using R = typename Raw<TO>::type;
  __shared__ float dec[256];
  for (int u = threadIdx.x; u < 256; u += kRowThreads) {
    if constexpr (E4M3) {
      __half_raw hr = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(u), __NV_E4M3);
      dec[u] = __half2float(__half(hr));
    } else {
      dec[u] = __fmul_rn(__fdiv_rn(static_cast<float>(u - 128), 127.0f), 448.0f);
    }
  }
  __syncthreads();
  const int64_t n = rows * cols;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * kRowThreads + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kRowThreads;
  if (vec) {
    constexpr int OV = static_cast<int>(sizeof(R));  // 16-byte output vectors per 16 codes
    const int64_t cpr = cols / 16;
    for (int64_t i = tid; i < n / 16; i += stride) {
      const uint4 in = __ldcs(reinterpret_cast<const uint4*>(q) + i);
      const float s = __ldg(scales + i / cpr);
      const uint32_t w[4] = {in.x, in.y, in.z, in.w};
      uint32_t o[4 * OV];  // the 16 outputs as 32-bit words, element k in the low bits first
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const uint32_t r = to_raw<TO>(__fdiv_rn(dec[(w[k >> 2] >> (8 * (k & 3))) & 0xffu], s));
        if constexpr (sizeof(R) == 2) {
          if (k & 1) o[k >> 1] |= r << 16;
          else o[k >> 1] = r;
        } else {
          o[k] = r;
        }
      }
      uint4* dst = reinterpret_cast<uint4*>(out) + i * OV;
#pragma unroll
      for (int v = 0; v < OV; ++v) __stcs(dst + v, make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]));
    }
    return;
  }
  for (int64_t i = tid; i < n; i += stride) out[i] = Ty<TO>::from_f(__fdiv_rn(dec[q[i]], __ldg(scales + i / cols)));
}

// Rows of at least kLutRowCols codes (VEC conditions as above): one CTA per
// pair of rows at a time builds the two rows' 256 outputs each in shared
// memory (one division per code value instead of one per element; the same
// rounded values), then streams both rows, contiguous in memory, as table
// lookups with four 16-byte code vectors in flight per thread.
constexpr int64_t kLutRowCols = 4096;

template <typename TO, bool E4M3>
__global__ void __launch_bounds__(kRowThreads) decode_rows_lut_kernel(const uint8_t* __restrict__ q, int64_t rows,
                                                                      int64_t cols, const float* __restrict__ scales,
                                                                      TO* __restrict__ out) {
  static_assert(kRowThreads == 256, "one thread per code value");
  using R = typename Raw<TO>::type;
  constexpr int OV = static_cast<int>(sizeof(R));  // 16-byte output vectors per 16 codes
  constexpr int U = 4;                              // code vectors in flight per thread
  __shared__ R lut[2][256];
  float d;  // this thread's code value, decoded
  if constexpr (E4M3) {
    __half_raw hr = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(threadIdx.x), __NV_E4M3);
    d = __half2float(__half(hr));
  } else {
    d = __fmul_rn(__fdiv_rn(static_cast<float>(static_cast<int>(threadIdx.x) - 128), 127.0f), 448.0f);
  }
  const int64_t cpr = cols / 16;
  for (int64_t r0 = 2 * static_cast<int64_t>(blockIdx.x); r0 < rows; r0 += 2 * static_cast<int64_t>(gridDim.x)) {
    const bool two = r0 + 1 < rows;
    const float s0 = __ldg(scales + r0);
    const float s1 = two ? __ldg(scales + r0 + 1) : 1.0f;
    __syncthreads();  // the previous pair's lookups are done before the tables change
    lut[0][threadIdx.x] = static_cast<R>(to_raw<TO>(__fdiv_rn(d, s0)));
    lut[1][threadIdx.x] = static_cast<R>(to_raw<TO>(__fdiv_rn(d, s1)));
    __syncthreads();
    const int64_t nch = (two ? 2 : 1) * cpr;  // chunks of the pair; chunk k is in row r0 + (k >= cpr)
    const uint4* qr = reinterpret_cast<const uint4*>(q + r0 * cols);
    uint4* orow = reinterpret_cast<uint4*>(out + r0 * cols);
    for (int64_t c = threadIdx.x; c < nch; c += U * kRowThreads) {
      uint4 in[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (c + u * kRowThreads < nch) in[u] = __ldcs(qr + c + u * kRowThreads);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t cc = c + u * kRowThreads;
        if (cc < nch) {
          const R* tab = lut[cc >= cpr ? 1 : 0];
          const uint32_t w[4] = {in[u].x, in[u].y, in[u].z, in[u].w};
          uint32_t o[4 * OV];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const uint32_t v = tab[(w[k >> 2] >> (8 * (k & 3))) & 0xffu];
            if constexpr (sizeof(R) == 2) {
              if (k & 1) o[k >> 1] |= v << 16;
              else o[k >> 1] = v;
            } else {
              o[k] = v;
            }
          }
#pragma unroll
          for (int v = 0; v < OV; ++v)
            __stcs(orow + cc * OV + v, make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]));
        }
      }
    }
  }
}

// ---- decode ----------------------------------------------------------------
constexpr int kDecThreads = 512;

// out = RN_out( dec(u) / s ), dec(u) = RN(RN(float(u - 128) / 127) * 448) for
// the reference codec (triton_ops/kernels/fp8_quantize.py:305-312) or the
// e4m3 value of u. Only 256 outputs exist per call, so each CTA builds them
// in shared memory and the stream becomes a table lookup.
template <typename TO, bool E4M3>
__global__ void __launch_bounds__(kDecThreads) decode_kernel(const uint8_t* __restrict__ q, int64_t n, bool vec,
                                                             const float* __restrict__ scale, TO* __restrict__ out) {
  using R = typename Raw<TO>::type;
  constexpr int U = 8;  // 16-byte code vectors in flight per thread
  // One copy of the 256 outputs per lane (lut[u * 32 + lane]), so the
  // data-dependent lookups of a warp never collide on a shared-memory bank.
  __shared__ R base[256];
  __shared__ uint32_t lut[256 * 32];
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t n16 = vec ? n / 16 : 0;
  // this thread's first U code vectors are requested before the table is
  // built, so the table's construction overlaps their DRAM latency
  uint4 in[U];
#pragma unroll
  for (int u = 0; u < U; ++u)
    if (tid + u * stride < n16) in[u] = __ldcs(reinterpret_cast<const uint4*>(q) + tid + u * stride);
  const float s = *scale;
  for (int u = threadIdx.x; u < 256; u += blockDim.x) {
    float v;
    if constexpr (E4M3) {
      __half_raw hr = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(u), __NV_E4M3);
      v = __half2float(__half(hr));
    } else {
      v = __fmul_rn(__fdiv_rn(static_cast<float>(u - 128), 127.0f), 448.0f);
    }
    base[u] = to_raw<TO>(__fdiv_rn(v, s));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 256 * 32; i += blockDim.x) lut[i] = base[i >> 5];
  __syncthreads();
  const uint32_t* my_lut = lut + (threadIdx.x & 31);
  constexpr int OV = 16 * sizeof(R) / 16;  // 16-byte output vectors per code vector
  int64_t done = 0;
  if (vec) {
    for (int64_t i = tid; i < n16; i += U * stride) {
      if (i != tid) {
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (i + u * stride < n16) in[u] = __ldcs(reinterpret_cast<const uint4*>(q) + i + u * stride);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (i + u * stride < n16) {
          const uint32_t w[4] = {in[u].x, in[u].y, in[u].z, in[u].w};
          uint32_t o[4 * OV];
          if constexpr (sizeof(R) == 2) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint32_t b0 = (w[k >> 1] >> (16 * (k & 1))) & 0xffu;
              const uint32_t b1 = (w[k >> 1] >> (16 * (k & 1) + 8)) & 0xffu;
              o[k] = my_lut[b0 * 32] | (my_lut[b1 * 32] << 16);
            }
          } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) o[k] = my_lut[((w[k >> 2] >> (8 * (k & 3))) & 0xffu) * 32];
          }
          uint4* dst = reinterpret_cast<uint4*>(out) + (i + u * stride) * OV;
#pragma unroll
          for (int v = 0; v < OV; ++v) __stcs(dst + v, make_uint4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]));
        }
      }
    }
    done = n16 * 16;
  }
  R* orow = reinterpret_cast<R*>(out);
  for (int64_t i = done + tid; i < n; i += stride) orow[i] = static_cast<R>(my_lut[q[i] * 32]);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {
bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int grid_for(int64_t work_items, int threads, int per_sm) {
  const int64_t want = (work_items + threads - 1) / threads;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(num_sms()) * per_sm)));
}
}  // namespace

// Four amax CTAs per SM (each thread keeps four 16-element loads in flight):
// streaming 32 MiB with eight 16-byte loads in flight per thread took 10.3 us
// with 2 CTAs of 256 threads per SM and 8.2 us with 4 or 8. The encode
// kernel's CTAs each reduce at most 4 x SM-count partials.
int amax_partials_count(int64_t n) { return grid_for(std::max<int64_t>(n / 64, 1), kAmaxThreads, 4); }

cudaError_t amax_partials_launch(const void* x, int64_t n, int x_dtype, uint32_t* partials, int nparts,
                                 cudaStream_t st) {
  const bool vec = al16(x);
  switch (x_dtype) {
    case F16: amax_partial_kernel<__half><<<nparts, kAmaxThreads, 0, st>>>(static_cast<const __half*>(x), n, vec, partials); break;
    case BF16: amax_partial_kernel<__nv_bfloat16><<<nparts, kAmaxThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(x), n, vec, partials); break;
    default: amax_partial_kernel<float><<<nparts, kAmaxThreads, 0, st>>>(static_cast<const float*>(x), n, vec, partials); break;
  }
  note_launch();
  return cudaGetLastError();
}

cudaError_t finalize_scale_launch(const uint32_t* partials, int nparts, float* scale_out, cudaStream_t st) {
  finalize_scale_kernel<<<1, 256, 0, st>>>(partials, nparts, scale_out);
  note_launch();
  return cudaGetLastError();
}

template <typename T>
static cudaError_t enc_t(const void* x, int64_t n, const float* scale_in, const uint32_t* partials, int nparts,
                         float* scale_out, void* out, int out_dtype, cudaStream_t st) {
  const bool vec = al16(x) && al16(out);
  const void* kern = (out_dtype == E4M3) ? reinterpret_cast<const void*>(encode_kernel<T, true>)
                                         : reinterpret_cast<const void*>(encode_kernel<T, false>);
  const int grid = grid_for(std::max<int64_t>(n / 32, 1), kEncThreads, cached_occupancy(kern, kEncThreads, 0));
  // a programmatic dependent of the kernel before it (e.g. the amax partials)
  cudaError_t e = (out_dtype == E4M3)
                      ? launch_dependent(encode_kernel<T, true>, grid, kEncThreads, st, static_cast<const T*>(x), n,
                                         vec, scale_in, partials, nparts, scale_out, static_cast<uint8_t*>(out))
                      : launch_dependent(encode_kernel<T, false>, grid, kEncThreads, st, static_cast<const T*>(x), n,
                                         vec, scale_in, partials, nparts, scale_out, static_cast<uint8_t*>(out));
  note_launch();
  return e;
}

cudaError_t encode_launch(const void* x, int64_t n, int x_dtype, const float* scale_in, const uint32_t* partials,
                          int nparts, float* scale_out, void* out, int out_dtype, cudaStream_t st) {
  switch (x_dtype) {
    case F16: return enc_t<__half>(x, n, scale_in, partials, nparts, scale_out, out, out_dtype, st);
    case BF16: return enc_t<__nv_bfloat16>(x, n, scale_in, partials, nparts, scale_out, out, out_dtype, st);
    default: return enc_t<float>(x, n, scale_in, partials, nparts, scale_out, out, out_dtype, st);
  }
}

namespace {
constexpr size_t kQuantPartialsOffset = 256;

template <typename T, bool E4M3>
cudaError_t quant_dyn_t(const void* x, int64_t n, float* scale_out, void* out, void* ws, size_t ws_bytes,
                        cudaStream_t st) {
  auto kernel = quantize_dynamic_kernel<T, E4M3>;
  const int occ = cached_occupancy(reinterpret_cast<const void*>(kernel), kQuantThreads, 0);
  const int64_t want = std::max<int64_t>(1, (n / 16 + kQuantThreads - 1) / kQuantThreads);
  const int grid = static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(occ) * num_sms()));
  if (ws_bytes < kQuantPartialsOffset + sizeof(uint32_t) * static_cast<size_t>(grid)) return cudaErrorInvalidValue;
  auto* barrier = static_cast<uint32_t*>(ws);
  cudaError_t e = cudaMemsetAsync(barrier, 0, 2 * sizeof(uint32_t), st);  // counter + max
  note_launch();
  if (e != cudaSuccess) return e;
  const T* xp = static_cast<const T*>(x);
  const bool vec = al16(x) && al16(out);
  auto* op = static_cast<uint8_t*>(out);
  uint32_t* err = error_word_ptr();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kQuantThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kernel, xp, n, vec, barrier, scale_out, op, err);
  note_launch();
  return e;
}
// The one-cluster form for small aligned tensors of whole vectors; *used
// tells whether it was launched.
template <typename T, bool E4M3>
cudaError_t quant_small_t(const void* x, int64_t n, float* scale_out, void* out, cudaStream_t st, bool* used) {
  *used = false;
  constexpr int EV = 16 / sizeof(T);
  const int64_t nvec = n / EV;
  const int64_t per_cta = static_cast<int64_t>(kSmallThreads) * kSmallVecs;
  if (!al16(x) || !al16(out) || n % EV != 0 || nvec < 1 || nvec > kSmallMaxCtas * per_cta) return cudaSuccess;
  // spread over the cluster down to kSmallMinVecs vectors per thread, so that
  // the encode of even one CTA's worth runs on several SMs
  const int64_t per_cta_min = static_cast<int64_t>(kSmallThreads) * kSmallMinVecs;
  const int ctas = static_cast<int>(std::min<int64_t>(kSmallMaxCtas, (nvec + per_cta_min - 1) / per_cta_min));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(kSmallThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(ctas);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, quantize_small_kernel<T, E4M3>, static_cast<const T*>(x), nvec, scale_out,
                                     static_cast<uint8_t*>(out));
  note_launch();
  *used = true;
  return e;
}

// Mid-size tensors (above the one-cluster form, up to kMidMaxBytes): two
// ordinary launches, per-CTA amax partials then an encode that reduces them
// (re-reading x, which at these sizes is still in L2). No barrier memset, no
// cooperative launch. [4096, 4096] fp16 (32 MiB): 16.7 us (e4m3 14.5 us)
// against 18.7 / 17.4 us for a cooperative one-kernel form that kept x in
// shared memory over a grid barrier (one HBM read, but the slab load, the
// barrier and the encode ran back to back). Larger tensors no longer fit L2
// reliably and take the grid-barrier form below.
constexpr int64_t kMidMaxBytes = 48ll << 20;

template <typename T, bool E4M3>
cudaError_t quant_any_t(const void* x, int64_t n, float* scale_out, void* out, void* ws, size_t ws_bytes,
                        cudaStream_t st) {
  bool used = false;
  cudaError_t e = quant_small_t<T, E4M3>(x, n, scale_out, out, st, &used);
  if (e != cudaSuccess || used) return e;
  if (n * static_cast<int64_t>(sizeof(T)) <= kMidMaxBytes) {
    const int nparts = amax_partials_count(n);
    if (ws_bytes < static_cast<size_t>(nparts) * sizeof(uint32_t)) return cudaErrorInvalidValue;
    uint32_t* parts = static_cast<uint32_t*>(ws);
    const int x_dtype = std::is_same<T, float>::value ? F32 : (std::is_same<T, __half>::value ? F16 : BF16);
    e = amax_partials_launch(x, n, x_dtype, parts, nparts, st);
    if (e != cudaSuccess) return e;
    return encode_launch(x, n, x_dtype, nullptr, parts, nparts, scale_out, out,
                         E4M3 ? static_cast<int>(DType::E4M3) : static_cast<int>(DType::U8), st);
  }
  return quant_dyn_t<T, E4M3>(x, n, scale_out, out, ws, ws_bytes, st);
}
}  // namespace

size_t quantize_dynamic_workspace_bytes() {
  // at most 4 CTAs of kQuantThreads per SM (2048 threads)
  return kQuantPartialsOffset + sizeof(uint32_t) * 4 * static_cast<size_t>(num_sms());
}

cudaError_t quantize_dynamic_launch(const void* x, int64_t n, int x_dtype, float* scale_out, void* out, int out_dtype,
                                    void* ws, size_t ws_bytes, cudaStream_t st) {
  const bool e4 = (out_dtype == E4M3);
  switch (x_dtype) {
    case F16: return e4 ? quant_any_t<__half, true>(x, n, scale_out, out, ws, ws_bytes, st)
                        : quant_any_t<__half, false>(x, n, scale_out, out, ws, ws_bytes, st);
    case BF16: return e4 ? quant_any_t<__nv_bfloat16, true>(x, n, scale_out, out, ws, ws_bytes, st)
                         : quant_any_t<__nv_bfloat16, false>(x, n, scale_out, out, ws, ws_bytes, st);
    default: return e4 ? quant_any_t<float, true>(x, n, scale_out, out, ws, ws_bytes, st)
                       : quant_any_t<float, false>(x, n, scale_out, out, ws, ws_bytes, st);
  }
}

template <typename TO>
static cudaError_t dec_t(const void* q, int64_t n, bool e4m3, const float* scale, void* out, cudaStream_t st) {
  const bool vec = al16(q) && al16(out);
  // the per-lane tables take 33 KB of shared memory per CTA
  const void* kern = e4m3 ? reinterpret_cast<const void*>(decode_kernel<TO, true>)
                          : reinterpret_cast<const void*>(decode_kernel<TO, false>);
  const int per_sm = cached_occupancy(kern, kDecThreads, 0);
  const int grid = grid_for(std::max<int64_t>(n / 128, 1), kDecThreads, per_sm);
  if (e4m3) {
    decode_kernel<TO, true><<<grid, kDecThreads, 0, st>>>(static_cast<const uint8_t*>(q), n, vec, scale, static_cast<TO*>(out));
  } else {
    decode_kernel<TO, false><<<grid, kDecThreads, 0, st>>>(static_cast<const uint8_t*>(q), n, vec, scale, static_cast<TO*>(out));
  }
  note_launch();
  return cudaGetLastError();
}

cudaError_t dequantize_launch(const void* q, int64_t n, int q_dtype, const float* scale, void* out, int out_dtype,
                              cudaStream_t st) {
  const bool e4m3 = (q_dtype == E4M3);
  switch (out_dtype) {
    case F16: return dec_t<__half>(q, n, e4m3, scale, out, st);
    case BF16: return dec_t<__nv_bfloat16>(q, n, e4m3, scale, out, st);
    default: return dec_t<float>(q, n, e4m3, scale, out, st);
  }
}

namespace {
int rows_grid(int64_t work) { return grid_for(std::max<int64_t>(work, 1), kRowThreads, 8); }
}  // namespace

cudaError_t row_scales_launch(const void* x, int64_t rows, int64_t cols, int x_dtype, float* scales, cudaStream_t st) {
  const int grid = rows_grid(rows * 32);
  const bool vec = al16(x) && cols % 16 == 0;  // every row starts on a 16-byte boundary
  switch (x_dtype) {
    case F16: row_scales_kernel<__half><<<grid, kRowThreads, 0, st>>>(static_cast<const __half*>(x), rows, cols, vec, scales); break;
    case BF16: row_scales_kernel<__nv_bfloat16><<<grid, kRowThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(x), rows, cols, vec, scales); break;
    default: row_scales_kernel<float><<<grid, kRowThreads, 0, st>>>(static_cast<const float*>(x), rows, cols, vec, scales); break;
  }
  note_launch();
  return cudaGetLastError();
}

template <typename T>
static cudaError_t enc_rows_t(const void* x, int64_t rows, int64_t cols, const float* scales, void* out, bool e4m3,
                              cudaStream_t st) {
  const bool vec = al16(x) && al16(out) && cols % 16 == 0;
  const int grid = rows_grid(vec ? rows * cols / 16 : rows * cols);
  if (e4m3) encode_rows_kernel<T, true><<<grid, kRowThreads, 0, st>>>(static_cast<const T*>(x), rows, cols, vec, scales, static_cast<uint8_t*>(out));
  else encode_rows_kernel<T, false><<<grid, kRowThreads, 0, st>>>(static_cast<const T*>(x), rows, cols, vec, scales, static_cast<uint8_t*>(out));
  note_launch();
  return cudaGetLastError();
}

cudaError_t encode_rows_launch(const void* x, int64_t rows, int64_t cols, int x_dtype, const float* scales, void* out,
                               int out_dtype, cudaStream_t st) {
  const bool e4 = out_dtype == E4M3;
  switch (x_dtype) {
    case F16: return enc_rows_t<__half>(x, rows, cols, scales, out, e4, st);
    case BF16: return enc_rows_t<__nv_bfloat16>(x, rows, cols, scales, out, e4, st);
    default: return enc_rows_t<float>(x, rows, cols, scales, out, e4, st);
  }
}

template <typename T>
static cudaError_t quant_rows_dyn_t(const void* x, int64_t rows, int64_t cols, void* scales_out, void* out, bool e4m3,
                                    cudaStream_t st) {
  const bool vec = al16(x) && al16(out) && cols % 16 == 0;
  const int grid = rows_grid(rows * 32);
  auto* xs = static_cast<const T*>(x);
  auto* so = static_cast<T*>(scales_out);
  auto* o = static_cast<uint8_t*>(out);
  if (e4m3) quantize_rows_dynamic_kernel<T, true><<<grid, kRowThreads, 0, st>>>(xs, rows, cols, vec, so, o);
  else quantize_rows_dynamic_kernel<T, false><<<grid, kRowThreads, 0, st>>>(xs, rows, cols, vec, so, o);
  note_launch();
  return cudaGetLastError();
}

cudaError_t quantize_rows_dynamic_launch(const void* x, int64_t rows, int64_t cols, int x_dtype, void* scales_out,
                                         void* out, int out_dtype, cudaStream_t st) {
  const bool e4 = out_dtype == E4M3;
  switch (x_dtype) {
    case F16: return quant_rows_dyn_t<__half>(x, rows, cols, scales_out, out, e4, st);
    case BF16: return quant_rows_dyn_t<__nv_bfloat16>(x, rows, cols, scales_out, out, e4, st);
    default: return quant_rows_dyn_t<float>(x, rows, cols, scales_out, out, e4, st);
  }
}

template <typename TO>
static cudaError_t dec_rows_t(const void* q, int64_t rows, int64_t cols, bool e4m3, const float* scales, void* out,
                              cudaStream_t st) {
  const bool vec = al16(q) && al16(out) && cols % 16 == 0;
  if (vec && cols >= kLutRowCols) {
    const int grid = static_cast<int>(std::min<int64_t>((rows + 1) / 2, static_cast<int64_t>(num_sms()) * 8));
    if (e4m3) decode_rows_lut_kernel<TO, true><<<grid, kRowThreads, 0, st>>>(static_cast<const uint8_t*>(q), rows, cols, scales, static_cast<TO*>(out));
    else decode_rows_lut_kernel<TO, false><<<grid, kRowThreads, 0, st>>>(static_cast<const uint8_t*>(q), rows, cols, scales, static_cast<TO*>(out));
    note_launch();
    return cudaGetLastError();
  }
  const int grid = rows_grid(vec ? rows * cols / 16 : rows * cols);
  if (e4m3) decode_rows_kernel<TO, true><<<grid, kRowThreads, 0, st>>>(static_cast<const uint8_t*>(q), rows, cols, vec, scales, static_cast<TO*>(out));
  else decode_rows_kernel<TO, false><<<grid, kRowThreads, 0, st>>>(static_cast<const uint8_t*>(q), rows, cols, vec, scales, static_cast<TO*>(out));
  note_launch();
  return cudaGetLastError();
}

cudaError_t decode_rows_launch(const void* q, int64_t rows, int64_t cols, int q_dtype, const float* scales, void* out,
                               int out_dtype, cudaStream_t st) {
  const bool e4 = q_dtype == E4M3;
  switch (out_dtype) {
    case F16: return dec_rows_t<__half>(q, rows, cols, e4, scales, out, st);
    case BF16: return dec_rows_t<__nv_bfloat16>(q, rows, cols, e4, scales, out, st);
    default: return dec_rows_t<float>(q, rows, cols, e4, scales, out, st);
  }
}

// ---------------------------------------------------------------------------
// Dynamic-scale quantize that allocates no device memory
// ---------------------------------------------------------------------------
// Scratch for the per-block amax partials of tfo_fp8_quantize_noalloc: a
// file-scope device array, so every GPU that loads the library holds these
// 16 KiB until the process exits. All calls share it and it keeps the last
// call's contents; every slot a call reads is written by that same call's
// amax kernel first, so nothing needs clearing.
constexpr int kNoallocMaxPartials = 4096;
static __device__ __align__(256) uint32_t g_noalloc_partials[kNoallocMaxPartials];

namespace {
// Device address of g_noalloc_partials, looked up with cudaGetSymbolAddress
// (in host code the array's name is only a host-side stand-in) and cached per
// CUDA context. The key is the context's unique id (cuCtxGetId), never reused
// within a process: after cudaDeviceReset, or with another context made
// current through the driver API, the id changes and the address is looked up
// again instead of reusing one that belongs to a destroyed or other context.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

struct NoallocSlot {
  unsigned long long ctx_id;
  uint32_t* ptr;
};
constexpr int kNoallocSlots = 64;
NoallocSlot g_noalloc_slots[kNoallocSlots];
int g_noalloc_next = 0;
std::mutex g_noalloc_mu;

bool current_context_id(unsigned long long* id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  CUcontext ctx = nullptr;
  if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr)
    return false;
  return get_id(ctx, id) == CUDA_SUCCESS;
}

cudaError_t noalloc_scratch(uint32_t** out) {
  unsigned long long id = 0;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  const bool have_id = current_context_id(&id);
  if (have_id) {
    for (int i = 0; i < kNoallocSlots; ++i) {
      if (g_noalloc_slots[i].ptr != nullptr && g_noalloc_slots[i].ctx_id == id) {
        *out = g_noalloc_slots[i].ptr;
        return cudaSuccess;
      }
    }
  }
  // First call in this context (this also makes the runtime's context current
  // when none was): look the address up with the device current.
  void* addr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&addr, g_noalloc_partials);
  if (e != cudaSuccess) return e;
  if (have_id || current_context_id(&id)) {
    g_noalloc_slots[g_noalloc_next] = NoallocSlot{id, static_cast<uint32_t*>(addr)};
    g_noalloc_next = (g_noalloc_next + 1) % kNoallocSlots;
  }
  *out = static_cast<uint32_t*>(addr);
  return cudaSuccess;
}
}  // namespace

}  // namespace tfo

using tfo::report_error;

extern "C" int tfo_fp8_quantize_noalloc(const void* x, int64_t numel, int x_dtype, float* scale_out, void* out,
                                        int out_dtype, void* stream) {
  using namespace tfo;
  if (x_dtype != F16 && x_dtype != BF16 && x_dtype != F32)
    return report_error(TFO_ERR_DTYPE, "tfo_fp8_quantize_noalloc: x must be f16, bf16 or f32");
  if (out_dtype != U8 && out_dtype != E4M3)
    return report_error(TFO_ERR_DTYPE, "tfo_fp8_quantize_noalloc: out must be U8 or E4M3");
  if (numel < 0) return report_error(TFO_ERR_INVALID, "tfo_fp8_quantize_noalloc: negative numel");
  if (!scale_out || (numel > 0 && (!x || !out)))
    return report_error(TFO_ERR_INVALID, "tfo_fp8_quantize_noalloc: NULL pointer");
  const int nparts = amax_partials_count(numel);
  if (nparts > kNoallocMaxPartials)
    return report_error(TFO_ERR_INVALID,
                        "tfo_fp8_quantize_noalloc: this device needs more amax partial slots than the 4096 in the "
                        "library's static scratch; use tfo_fp8_quantize with a caller-provided workspace");
  uint32_t* parts = nullptr;
  cudaError_t e = noalloc_scratch(&parts);
  if (e != cudaSuccess) {
    return report_error(TFO_ERR_CUDA, (std::string("tfo_fp8_quantize_noalloc: scratch address lookup failed: ") +
                                       cudaGetErrorString(e)).c_str());
  }
  auto st = static_cast<cudaStream_t>(stream);
  e = amax_partials_launch(x, numel, x_dtype, parts, nparts, st);
  if (e == cudaSuccess) {
    e = (numel == 0) ? finalize_scale_launch(parts, nparts, scale_out, st)
                     : encode_launch(x, numel, x_dtype, nullptr, parts, nparts, scale_out, out, out_dtype, st);
  }
  if (e != cudaSuccess)
    return report_error(TFO_ERR_CUDA, (std::string("tfo_fp8_quantize_noalloc: ") + cudaGetErrorString(e)).c_str());
  return TFO_OK;
}
