// Epilogue helpers shared by the tcgen05 GEMMs: rounding 16 fp32 values to the
// output dtype and storing them as 16-byte vectors (or element by element at
// ragged edges).
#pragma once

#include "common.cuh"

namespace tfo {

template <typename TO>
__device__ __forceinline__ uint32_t pack2_out(float a, float b) {
  if constexpr (std::is_same<TO, __half>::value) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// dst points at column col0 of one output row; `valid` columns (<= 16) exist.
// stream: the vector stores are evict-first (st.global.cs), for outputs far
// larger than L2 that nothing reads back soon.
template <typename TO>
__device__ __forceinline__ void store_row16(TO* dst, const float (&v)[16], int valid, bool vec_ok,
                                            bool stream = false) {
  if (vec_ok && valid == 16) {
    uint4* d = reinterpret_cast<uint4*>(dst);
    auto put = [stream](uint4* q, uint4 val) {
      if (stream) __stcs(q, val);
      else *q = val;
    };
    if constexpr (sizeof(TO) == 2) {
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] = pack2_out<TO>(v[2 * i], v[2 * i + 1]);
      put(d, make_uint4(w[0], w[1], w[2], w[3]));
      put(d + 1, make_uint4(w[4], w[5], w[6], w[7]));
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        put(d + i, make_uint4(__float_as_uint(v[4 * i]), __float_as_uint(v[4 * i + 1]), __float_as_uint(v[4 * i + 2]),
                              __float_as_uint(v[4 * i + 3])));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i < valid) dst[i] = Ty<TO>::from_f(v[i]);
  }
}

}  // namespace tfo
