// Reference 8-bit codec and amax helpers shared by the codec kernels
// (fp8_codec.cu) and the fused RMSNorm+RoPE -> quantize kernel
// (rmsnorm_rope.cu). The code follows triton_ops/kernels/fp8_quantize.py:258-287
// and the scale triton_ops/models.py:282-299.
#pragma once

#include "common.cuh"

namespace tfo {

__device__ __forceinline__ float min_nan(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Reference-codec byte for a scaled value c:
//   u = int8(rint(RN(RN(clamp(c, +-448) / 448) * 127))) + 128.
// Since 448 = 7 * 2^6, RN(c / 448) = RN(c / 7) * 2^-6 exactly (a power-of-two
// scaling commutes with rounding; where it would not, |c| is so small that
// the code is 0 anyway), and RN(RN(c / 7) * 2^-6 * 127) = RN(RN(c / 7) * 1.984375)
// because 127 / 64 = 1.984375 is exact. RN(c / 7) is Markstein's
// FMA-corrected quotient with y = RN(1/7): q0 = RN(c*y), r = c - 7*q0 (exact),
// q = RN(q0 + r*y). The clamp keeps NaN (it encodes as 0, like the
// reference's float -> int8 conversion); +-inf clamp to +-448.
__device__ __forceinline__ uint32_t ref_encode(float c) {
  const float cl = min_nan(max_nan(c, -448.0f), 448.0f);
  constexpr float kInv7 = 0.142857142857142857f;
  const float q0 = __fmul_rn(cl, kInv7);
  const float r = __fmaf_rn(-q0, 7.0f, cl);
  const float q = __fmaf_rn(r, kInv7, q0);
  const int k = __float2int_rn(__fmul_rn(q, 1.984375f));  // NaN -> 0, |k| <= 127
  return static_cast<uint32_t>(k + 128) & 0xffu;
}

// Reference-codec bytes of four scaled values with |c| <= 448 + 1 ulp (true
// for every element under a finite, non-zero dynamic scale s = 448 / amax):
// no clamp or NaN handling is needed, and rint(y) for |y| <= 128 is read
// from the low byte of y + 1.5 * 2^23 (one round-to-nearest-even addition,
// exact for |y| < 2^22). The low byte is rint(y) mod 256, so the code
// rint(y) + 128 is that byte XOR 0x80.
__device__ __forceinline__ uint32_t ref_encode4_in_range(float c0, float c1, float c2, float c3) {
  // RN(c / 7) on two packed lanes at a time. The last multiply and the
  // rounding addition stay scalar: __fmul_rn / __fadd_rn are never contracted
  // into an fma, while a packed mul followed by a packed add was seen to be
  // (which skips the rounding of q * 1.984375 and breaks exact ties).
  const F2 inv7 = f2(0.142857142857142857f, 0.142857142857142857f), m7 = f2(-7.0f, -7.0f);
  auto kbits2 = [&](F2 c) -> F2 {
    const F2 q0 = mul2(c, inv7);
    const F2 r = fma2(q0, m7, c);  // c - 7 q0, exact
    const F2 q = fma2(r, inv7, q0);
    return f2(__fadd_rn(__fmul_rn(q.x, 1.984375f), 12582912.0f), __fadd_rn(__fmul_rn(q.y, 1.984375f), 12582912.0f));
  };
  const F2 a = kbits2(f2(c0, c1)), b = kbits2(f2(c2, c3));
  const uint32_t lo = __byte_perm(__float_as_uint(a.x), __float_as_uint(a.y), 0x0040);
  const uint32_t hi = __byte_perm(__float_as_uint(b.x), __float_as_uint(b.y), 0x0040);
  return __byte_perm(lo, hi, 0x5410) ^ 0x80808080u;
}

// As above for x0..x3 * s (the scale product rounded first, also packed).
__device__ __forceinline__ uint32_t ref_encode4_in_range_scaled(const float* x, float s) {
  const F2 ss = f2(s, s);
  const F2 c01 = mul2(f2(x[0], x[1]), ss), c23 = mul2(f2(x[2], x[3]), ss);
  return ref_encode4_in_range(c01.x, c01.y, c23.x, c23.y);
}

// Block-wide max of one value per thread; every thread gets the result.
__device__ __forceinline__ uint32_t block_max_u32(uint32_t m, uint32_t* red /* smem, >= 32 */) {
  m = warp_max_u32(m);
  __syncthreads();  // red may still be read by an earlier call
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  uint32_t b = 0;
  for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) b = max(b, red[i]);
  return b;
}

// The reference's host-side scale from amax (bits of a non-negative float):
// fp32(448.0 / double(amax)), 1.0 for amax == 0.
// A NaN amax gives the quiet NaN 0x7FC00000, the bits the reference's
// Python float division produces.
__device__ __forceinline__ float scale_from_amax(uint32_t amax_bits) {
  const float amax = __uint_as_float(amax_bits);
  if (amax != amax) return __uint_as_float(0x7FC00000u);
  return (amax == 0.f) ? 1.0f : __double2float_rn(__ddiv_rn(448.0, static_cast<double>(amax)));
}

// Reduces the per-CTA partial maxima (read through L2: other SMs wrote them)
// and derives the scale exactly as the reference's host code does.
__device__ __forceinline__ float reduce_partials_to_scale(const uint32_t* __restrict__ partials, int nparts,
                                                          uint32_t* red /* smem, >= 32 */) {
  uint32_t m = 0;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) m = max(m, __ldcg(partials + i));
  return scale_from_amax(block_max_u32(m, red));
}

// max over the |x| bit patterns of one 16-byte vector, kept per 16-bit lane
// for 16-bit types (|x| orders like its bits; NaN above inf) and per word for fp32
template <typename T>
__device__ __forceinline__ uint32_t absmax_vec(uint32_t m, uint4 v) {
  if constexpr (sizeof(T) == 2) {
    m = __vmaxu2(m, v.x & 0x7FFF7FFFu);
    m = __vmaxu2(m, v.y & 0x7FFF7FFFu);
    m = __vmaxu2(m, v.z & 0x7FFF7FFFu);
    return __vmaxu2(m, v.w & 0x7FFF7FFFu);
  } else {
    m = max(m, v.x & 0x7FFFFFFFu);
    m = max(m, v.y & 0x7FFFFFFFu);
    m = max(m, v.z & 0x7FFFFFFFu);
    return max(m, v.w & 0x7FFFFFFFu);
  }
}
// the fp32 bit pattern of the larger lane
template <typename T>
__device__ __forceinline__ uint32_t absmax_to_f32_bits(uint32_t m) {
  if constexpr (std::is_same<T, float>::value) {
    return m;
  } else {
    const uint32_t h = max(m & 0xFFFFu, m >> 16);
    if constexpr (std::is_same<T, __half>::value) {
      return __float_as_uint(__half2float(__ushort_as_half(static_cast<unsigned short>(h))));
    } else {
      return h << 16;
    }
  }
}

}  // namespace tfo
