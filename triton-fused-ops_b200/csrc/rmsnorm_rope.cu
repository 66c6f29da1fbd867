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
#include <type_traits>

#include "capi_internal.h"
#include "codec.cuh"
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
// fp32, and before each row's reduction barrier the row's cos/sin entries are
// converted to fp32 once into shared memory (double-buffered with the
// reduction slots). The sum of squares is a warp-shuffle + one-barrier block
// reduction; right after that barrier every thread has read its vectors of
// the slot, so the slot is refilled with the row `stages` ahead.
constexpr int kMaxHalfHead = 128;  // head_dim <= 256 on the vector path

struct VecSmem {
  static constexpr int kBar = 0;                           // uint64_t[8]
  static constexpr int kRed = 64;                          // float[2][32]
  static constexpr int kCs = kRed + 2 * 32 * 4;            // float[2][3 * kMaxHalfHead]: cos, sin, -sin
  static constexpr int kW = kCs + 2 * 3 * kMaxHalfHead * 4;  // float[hidden]
  __host__ __device__ static size_t ring_offset(int hidden) { return ((kW + static_cast<size_t>(hidden) * 4 + 127) / 128) * 128; }
};

// FULL: every thread owns exactly NV vectors of the row (NV * blockDim.x ==
// hidden / E) and every column is rotated (num_heads * head_dim == hidden),
// so no per-vector bounds or rotation checks are needed.
template <typename TX, typename TCS, int NV, bool FULL>
__global__ void __launch_bounds__(256, 4) rmsnorm_rope_vec_kernel(
    const TX* __restrict__ x, const void* __restrict__ w, const TCS* __restrict__ cosp, const TCS* __restrict__ sinp,
    TX* __restrict__ out, int64_t rows, int seq_len, int hidden, int head_dim, int rot_cols, int64_t cs_ss,
    int64_t cs_sd, float eps, int w_dtype, int stages, uint32_t* err) {
  griddep_launch_dependents();  // a programmatic-dependent GEMM that follows may be scheduled early
  constexpr int E = Pack<TX>::E;
  // With 16-bit x and tables, y*c and p*s are exact in fp32, so the
  // reference's RN(RN(y*c) -/+ RN(p*s)) equals one FMA on an exact product.
  constexpr bool kExactProducts = sizeof(TX) == 2 && sizeof(TCS) == 2;
  const int T = blockDim.x;
  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5, nwarps = T >> 5;
  const int nvec = hidden / E;
  const int dv = head_dim / E;     // vectors per head (power of two, <= 32)
  const int hv = dv >> 1;          // rotate-half partner distance, in vectors / lanes
  const int half = head_dim >> 1;
  const int rot_vecs = rot_cols / E;
  const uint32_t row_bytes = static_cast<uint32_t>(hidden) * sizeof(TX);

  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + VecSmem::kBar);
  float* red = reinterpret_cast<float*>(smem + VecSmem::kRed);
  float* csm = reinterpret_cast<float*>(smem + VecSmem::kCs);
  float* wsm = reinterpret_cast<float*>(smem + VecSmem::kW);
  uint8_t* ring = smem + VecSmem::ring_offset(hidden);

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

  // Row-invariant per-vector offsets (shared-memory float offsets of the
  // weight slice and of the cos / signed-sin entries within a cos-sin buffer).
  int w_off[NV], c_off[NV], s_off[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int g = v * T + t;
    w_off[v] = (FULL ? g : min(g, nvec - 1)) * E;
    const int hi = g & (dv - 1);
    const bool first = hi < hv;
    c_off[v] = (first ? hi : hi - hv) * E;
    s_off[v] = (first ? 2 * half : half) + c_off[v];
  }

  // ring slot, its phase parity and the RoPE position advance incrementally
  // (no per-row 64-bit division)
  int buf = 0, s = 0;
  uint32_t par = 0;
  int pos = static_cast<int>(blockIdx.x % static_cast<unsigned>(seq_len));
  const int pos_step = static_cast<int>(gridDim.x % static_cast<unsigned>(seq_len));
  int64_t row = blockIdx.x;
  for (int64_t i = 0; i < my_rows; ++i, row += gridDim.x) {
    // this row's cos, sin and -sin entries as fp32, published by the barrier below
    for (int q = t; q < 2 * half; q += T) {
      const int j = q < half ? q : q - half;
      const float v = Ty<TCS>::to_f((q < half ? cosp : sinp)[static_cast<int64_t>(pos) * cs_ss + j * cs_sd]);
      float* cs_buf = csm + buf * 3 * kMaxHalfHead;
      cs_buf[q] = v;
      if (q >= half) cs_buf[q + half] = -v;
    }
    if (!mbar_wait(&full[s], par, err, ERR_WAIT_TIMEOUT_OTHER)) break;

    const uint4* rv = reinterpret_cast<const uint4*>(ring + static_cast<size_t>(s) * row_bytes);
    float xf[NV][E];
    float ss0 = 0.f, ss1 = 0.f;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int g = v * T + t;
      const uint4 u = (FULL || g < nvec) ? rv[g] : make_uint4(0, 0, 0, 0);
      Pack<TX>::unpack(u, xf[v]);
#pragma unroll
      for (int j = 0; j < E; j += 2) {
        ss0 = __fmaf_rn(xf[v][j], xf[v][j], ss0);
        ss1 = __fmaf_rn(xf[v][j + 1], xf[v][j + 1], ss1);
      }
    }
    float ss = warp_sum(ss0 + ss1);
    if (lane == 0) red[buf * 32 + warp] = ss;
    __syncthreads();
    // every thread has consumed slot s: refill it with the row `stages` ahead
    if (t == 0 && i + stages < my_rows) {
      fence_proxy_async_smem();
      const int64_t r = row + static_cast<int64_t>(stages) * gridDim.x;
      mbar_arrive_expect_tx(&full[s], row_bytes);
      bulk_load(ring + static_cast<size_t>(s) * row_bytes, x + r * hidden, row_bytes, &full[s]);
    }
    // second stage of the reduction: each warp sums the per-warp partials
    const float tot = warp_sum(lane < nwarps ? red[buf * 32 + lane] : 0.f);
    const float* cs_row = csm + buf * 3 * kMaxHalfHead;
    buf ^= 1;

    const float ms = __fdiv_rn(tot, static_cast<float>(hidden));
    const float rms = __fsqrt_rn(__fadd_rn(ms, eps));
    const float rb = __frcp_rn(rms);
    uint4* orow = reinterpret_cast<uint4*>(out + row * hidden);

    // Row-uniform choice of division: Markstein for finite positive rms,
    // IEEE division otherwise (inf / NaN / zero rms, where x is not finite).
    auto process = [&](auto fast_tag) {
      constexpr bool FAST = decltype(fast_tag)::value;
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const int g = v * T + t;
        const float4* wv = reinterpret_cast<const float4*>(wsm + w_off[v]);
        float y[E];
#pragma unroll
        for (int q4 = 0; q4 < E / 4; ++q4) {
          const float4 w4 = wv[q4];
          const float wr[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float xv = xf[v][4 * q4 + j];
            const float q = FAST ? div_markstein(xv, rms, rb) : __fdiv_rn(xv, rms);
            y[4 * q4 + j] = __fmul_rn(q, wr[j]);
          }
        }
        // y rounded to x's dtype: packed (to exchange) and back in fp32
        uint32_t yw[4];
        pack_vec<TX, E>(y, yw);
        unpack_words<TX, E>(yw, y);
        uint32_t pw[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) pw[k] = __shfl_xor_sync(0xffffffffu, yw[k], hv);
        if (!FULL && g >= nvec) continue;

        if (FULL || g < rot_vecs) {
          float pv[E];
          unpack_words<TX, E>(pw, pv);
          // first half: a*c - b*s; second half: b*s + a*c. With s taken from
          // the negated copy for the first half, both are RN(RN(a*c) + RN(b*s')).
          const float4* c4 = reinterpret_cast<const float4*>(cs_row + c_off[v]);
          const float4* s4 = reinterpret_cast<const float4*>(cs_row + s_off[v]);
          float o[E];
#pragma unroll
          for (int q4 = 0; q4 < E / 4; ++q4) {
            const float4 cc = c4[q4], sv = s4[q4];
            const float c[4] = {cc.x, cc.y, cc.z, cc.w};
            const float sn[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float a = y[4 * q4 + j], b = pv[4 * q4 + j];
              if constexpr (kExactProducts) {
                o[4 * q4 + j] = __fmaf_rn(a, c[j], __fmul_rn(b, sn[j]));
              } else {
                o[4 * q4 + j] = __fadd_rn(__fmul_rn(a, c[j]), __fmul_rn(b, sn[j]));
              }
            }
          }
          uint32_t ow[4];
          pack_vec<TX, E>(o, ow);
          __stcs(orow + g, make_uint4(ow[0], ow[1], ow[2], ow[3]));
        } else {
          __stcs(orow + g, make_uint4(yw[0], yw[1], yw[2], yw[3]));
        }
      }
    };
    if (rms > 0.f && rms <= 3.0e38f) {
      process(std::integral_constant<bool, true>{});
    } else {
      process(std::integral_constant<bool, false>{});
    }
    if (++s == stages) {
      s = 0;
      par ^= 1u;
    }
    pos += pos_step;
    if (pos >= seq_len) pos -= seq_len;
  }
}

// Shared memory of the vector path: barriers, reduction and cos/sin slots,
// the fp32 weight row and `stages` row buffers.
inline size_t vec_smem_bytes(int hidden, int row_bytes, int stages) {
  return VecSmem::ring_offset(hidden) + static_cast<size_t>(stages) * row_bytes;
}

// Warp-per-row path (hidden = 32 * VPL vectors, VPL <= 16). Every warp owns
// the rows gw, gw + GW, ... (gw = global warp id, GW = warps in the grid) and
// one private row buffer in shared memory, filled by bulk copies, so no
// CTA-wide barrier is needed after setup. The first pass moves the row from
// shared memory into registers (VPL 16-byte vectors per lane) while summing
// squares; lane 0 then immediately refills the buffer with the warp's next
// row, whose load overlaps the second pass. The sum of squares is a pure
// warp-shuffle reduction. Vector g = j*32 + lane; a head spans dv <= 32
// vectors that divide 32, so a lane's position inside its head (and its
// cos/sin offsets) is the same for every j.
// At most 12 warps with 16 vectors per lane (row kept in 64 registers), 16 otherwise.
constexpr int warp_rows_max_warps(int vpl) { return vpl >= 16 ? 12 : 16; }
// Per-warp raw cos/sin slot of the warp-per-row kernel: two halves of up to
// kMaxHalfHead fp32 entries would be 1 KB; head_dim <= 64 tables use <= 256 B.
constexpr int kCsRawBytes = 256;
// Row buffers per warp: a warp's next row is in flight while it works on the
// current one and the one after that while it finishes (with one buffer the
// next load only started after the current row's first pass).
constexpr int kWarpSlots = 2;
constexpr int kWarpBarBytes = 32 * 8;  // up to 32 mbarriers (warps x slots)
static_assert(16 * kWarpSlots <= 32, "barrier area");

// MODE 0 stores the output rows; MODE 3 also writes one max |output value|
// per CTA to q.parts_out (the amax partials of a dynamic-scale quantize of the
// rows, so that no separate amax pass over the rows is needed).
template <typename TX, typename TCS, bool FULLROT, int VPL, int MODE>
__global__ void __launch_bounds__(32 * warp_rows_max_warps(VPL), 1) rmsnorm_rope_warp_kernel(
    const TX* __restrict__ x, const void* __restrict__ w, const TCS* __restrict__ cosp, const TCS* __restrict__ sinp,
    TX* __restrict__ out, int64_t rows, int seq_len, int hidden, int head_dim, int rot_cols, int64_t cs_ss,
    int64_t cs_sd, float eps, int w_dtype, int cs_stride, bool cs_bulk, uint32_t* err, const RowQuantArgs q) {
  griddep_launch_dependents();  // a programmatic-dependent GEMM that follows may be scheduled early
  constexpr int E = Pack<TX>::E;
  constexpr bool kExactProducts = sizeof(TX) == 2 && sizeof(TCS) == 2;
  const int W = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dv = head_dim / E;
  const int hv = dv >> 1;
  const int half = head_dim >> 1;
  const int rot_vecs = rot_cols / E;
  const uint32_t row_bytes = static_cast<uint32_t>(hidden) * sizeof(TX);

  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);                // [W][kWarpSlots]
  float* wsm = reinterpret_cast<float*>(smem + kWarpBarBytes);       // [hidden]
  float* csm = wsm + hidden;                                         // [W][cs_stride]
  uint8_t* ring = smem + ((kWarpBarBytes + (static_cast<size_t>(hidden) + W * cs_stride) * 4 + 127) / 128) * 128;

  float* cs_buf = csm + warp * cs_stride;   // cos[half], sin[half], -sin[half]
  // kWarpSlots row buffers per warp (row k of the warp in buffer k % kWarpSlots,
  // each with its own mbarrier): a buffer is refilled with row k + kWarpSlots
  // as soon as row k has moved into registers.
  // cs_bulk: the row's cos and sin halves (contiguous, 16-byte aligned) arrive
  // with the row by bulk copy into the buffer's raw table slot, so a row never
  // waits on global loads of its table entries
  const uint32_t cs_half_bytes = static_cast<uint32_t>(half) * sizeof(TCS);
  auto slot_of = [&](int b) { return ring + static_cast<size_t>(warp * kWarpSlots + b) * row_bytes; };
  auto cs_raw_of = [&](int b) {
    return reinterpret_cast<TCS*>(ring + static_cast<size_t>(W * kWarpSlots) * row_bytes +
                                  static_cast<size_t>(warp * kWarpSlots + b) * kCsRawBytes);
  };
  auto issue_row = [&](int b, int64_t r, int p) {
    uint64_t* bar = bars + warp * kWarpSlots + b;
    if (cs_bulk) {
      TCS* raw = cs_raw_of(b);
      mbar_arrive_expect_tx(bar, row_bytes + 2 * cs_half_bytes);
      bulk_load(raw, cosp + static_cast<int64_t>(p) * cs_ss, cs_half_bytes, bar);
      bulk_load(raw + half, sinp + static_cast<int64_t>(p) * cs_ss, cs_half_bytes, bar);
    } else {
      mbar_arrive_expect_tx(bar, row_bytes);
    }
    bulk_load(slot_of(b), x + r * hidden, row_bytes, bar);
  };

  const int64_t gw = static_cast<int64_t>(blockIdx.x) * W + warp;
  const int64_t GW = static_cast<int64_t>(gridDim.x) * W;
  const int64_t my_rows = rows > gw ? (rows - gw + GW - 1) / GW : 0;

  for (int i = threadIdx.x; i < hidden; i += blockDim.x) wsm[i] = load_as_float(w, i, w_dtype);
  if (lane == 0) {
    for (int b = 0; b < kWarpSlots; ++b) mbar_init(bars + warp * kWarpSlots + b, 1);
    fence_mbar_init();
  }
  __syncthreads();
  int pos = static_cast<int>(gw % seq_len);
  const int pos_step = static_cast<int>(GW % seq_len);
  auto advance = [&](int p) {
    p += pos_step;
    return p >= seq_len ? p - seq_len : p;
  };
  // position of the row kWarpSlots rows ahead of the current one
  int ahead_pos = pos;
  for (int b = 0; b < kWarpSlots; ++b) {
    if (lane == 0 && b < my_rows) issue_row(b, gw + b * GW, ahead_pos);
    ahead_pos = advance(ahead_pos);
  }

  // per-lane constants: position in head, cos / signed-sin offsets
  const int hi = lane & (dv - 1);
  const bool first = hi < hv;
  const int c_off = (first ? hi : hi - hv) * E;
  const int s_off = (first ? 2 * half : half) + c_off;

  __shared__ uint32_t qred[32];
  uint32_t amax_lanes = 0;  // MODE 3: max |output| bits (per 16-bit lane for 16-bit TX)

  // Stores output vector g of row `row` (16 bytes of packed TX words) and, in
  // MODE 3, folds it into the running max.
  auto emit = [&](int64_t row_, int g, const uint32_t (&wd)[4]) {
    __stcs(reinterpret_cast<uint4*>(out + row_ * hidden) + g, make_uint4(wd[0], wd[1], wd[2], wd[3]));
    if constexpr (MODE == 3) amax_lanes = absmax_vec<TX>(amax_lanes, make_uint4(wd[0], wd[1], wd[2], wd[3]));
  };

  int64_t row = gw;
  for (int64_t k = 0; k < my_rows; ++k, row += GW) {
    const int b = static_cast<int>(k % kWarpSlots);
    const uint32_t par = static_cast<uint32_t>(k / kWarpSlots) & 1u;
    const uint4* rv = reinterpret_cast<const uint4*>(slot_of(b));
    if (!cs_bulk) {
      for (int q = lane; q < 2 * half; q += 32) {
        const int j = q < half ? q : q - half;
        const float v = Ty<TCS>::to_f((q < half ? cosp : sinp)[static_cast<int64_t>(pos) * cs_ss + j * cs_sd]);
        cs_buf[q] = v;
        if (q >= half) cs_buf[q + half] = -v;
      }
    }

    if (!mbar_wait(bars + warp * kWarpSlots + b, par, err, ERR_WAIT_TIMEOUT_OTHER)) break;
    if (cs_bulk) {
      const TCS* raw = cs_raw_of(b);
      for (int q = lane; q < 2 * half; q += 32) {
        const float v = Ty<TCS>::to_f(raw[q]);
        cs_buf[q] = v;
        if (q >= half) cs_buf[q + half] = -v;
      }
    }

    uint4 xr[VPL];
    float ss0 = 0.f, ss1 = 0.f;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      xr[j] = rv[j * 32 + lane];
      float f[E];
      Pack<TX>::unpack(xr[j], f);
#pragma unroll
      for (int e = 0; e < E; e += 2) {
        ss0 = __fmaf_rn(f[e], f[e], ss0);
        ss1 = __fmaf_rn(f[e + 1], f[e + 1], ss1);
      }
    }
    __syncwarp();  // all lanes have read the buffers: refill them with this warp's next row
    if (lane == 0 && k + kWarpSlots < my_rows) {
      fence_proxy_async_smem();
      issue_row(b, row + kWarpSlots * GW, ahead_pos);
    }
    ahead_pos = advance(ahead_pos);
    const float tot = warp_sum(ss0 + ss1);  // also orders this warp's cs_buf writes before the reads below
    __syncwarp();
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, static_cast<float>(hidden)), eps));
    const float rb = __frcp_rn(rms);
    const float4* c4 = reinterpret_cast<const float4*>(cs_buf + c_off);
    const float4* s4 = reinterpret_cast<const float4*>(cs_buf + s_off);

    auto second_pass = [&](auto fast_tag) {
      constexpr bool FAST = decltype(fast_tag)::value;
#pragma unroll
      for (int j = 0; j < VPL; ++j) {
        const int g = j * 32 + lane;
        float xf[E];
        Pack<TX>::unpack(xr[j], xf);
        const float4* wv = reinterpret_cast<const float4*>(wsm + g * E);
        float y[E];
#pragma unroll
        for (int q4 = 0; q4 < E / 4; ++q4) {
          const float4 w4 = wv[q4];
          const float wr[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float xv = xf[4 * q4 + e];
            const float qv = FAST ? div_markstein(xv, rms, rb) : __fdiv_rn(xv, rms);
            y[4 * q4 + e] = __fmul_rn(qv, wr[e]);
          }
        }
        uint32_t yw[4];
        pack_vec<TX, E>(y, yw);
        unpack_words<TX, E>(yw, y);
        uint32_t pw[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) pw[q] = __shfl_xor_sync(0xffffffffu, yw[q], hv);
        if (FULLROT || g < rot_vecs) {
          float pv[E];
          unpack_words<TX, E>(pw, pv);
          float o[E];
#pragma unroll
          for (int q4 = 0; q4 < E / 4; ++q4) {
            const float4 cc = c4[q4], sv = s4[q4];
            const float c[4] = {cc.x, cc.y, cc.z, cc.w};
            const float sn[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float a = y[4 * q4 + e], b = pv[4 * q4 + e];
              if constexpr (kExactProducts) {
                o[4 * q4 + e] = __fmaf_rn(a, c[e], __fmul_rn(b, sn[e]));
              } else {
                o[4 * q4 + e] = __fadd_rn(__fmul_rn(a, c[e]), __fmul_rn(b, sn[e]));
              }
            }
          }
          uint32_t ow[4];
          pack_vec<TX, E>(o, ow);
          emit(row, g, ow);
        } else {
          emit(row, g, yw);
        }
      }
    };
    if (rms > 0.f && rms <= 3.0e38f) {
      second_pass(std::integral_constant<bool, true>{});
    } else {
      second_pass(std::integral_constant<bool, false>{});
    }
    __syncwarp();  // cs_buf is rewritten for the next row
    pos = advance(pos);
  }
  if constexpr (MODE == 3) {
    const uint32_t b = block_max_u32(absmax_to_f32_bits<TX>(amax_lanes), qred);
    if (threadIdx.x == 0) q.parts_out[blockIdx.x] = b;
  }
}

// Generic path: any hidden size / head_dim / alignment. One CTA per row
// (grid-stride); the row is staged in shared memory as fp32.
template <typename TX>
__global__ void __launch_bounds__(256) rmsnorm_rope_generic_kernel(
    const TX* __restrict__ x, const void* __restrict__ w, const void* __restrict__ cosp, const void* __restrict__ sinp,
    TX* __restrict__ out, int64_t rows, int seq_len, int hidden, int head_dim, int rot_cols, int64_t cs_ss,
    int64_t cs_sd, float eps, int w_dtype, int cos_dtype, int sin_dtype) {
  griddep_launch_dependents();  // a programmatic-dependent GEMM that follows may be scheduled early
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

template <typename TX, typename TCS, int NV, bool FULL>
cudaError_t launch_vec(const RmsNormRopeArgs& a, int threads, cudaStream_t st) {
  auto kern = rmsnorm_rope_vec_kernel<TX, TCS, NV, FULL>;
  const int row_bytes = static_cast<int>(a.hidden * sizeof(TX));
  // ring of up to 8 rows, about 32 KB, at least 2 (4 CTAs per SM at H = 4096 fp16)
  const int stages = std::max(2, std::min(8, (32 * 1024) / row_bytes));
  const size_t smem = vec_smem_bytes(static_cast<int>(a.hidden), row_bytes, stages);
  if (cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem); e != cudaSuccess) return e;
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

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// One CTA per SM at most, `warps` rows in flight per CTA.
inline int64_t warp_rows_grid(int64_t rows, int warps) {
  return std::max<int64_t>(1, std::min<int64_t>((rows + warps - 1) / warps, num_sms()));
}

template <typename TX, typename TCS, bool FULLROT, int VPL, int MODE>
cudaError_t launch_warp_rows_m(const RmsNormRopeArgs& a, int warps, int cs_stride, size_t smem, const RowQuantArgs& q,
                               cudaStream_t st) {
  auto kern = rmsnorm_rope_warp_kernel<TX, TCS, FULLROT, VPL, MODE>;
  if (cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem); e != cudaSuccess) return e;
  const int64_t rows = a.batch * a.seq_len;
  const int64_t grid = warp_rows_grid(rows, warps);
  // table rows by bulk copy: contiguous halves on 16-byte boundaries that fit the raw slot
  const int64_t half_bytes = (a.head_dim / 2) * static_cast<int64_t>(sizeof(TCS));
  const bool cs_bulk = a.cs_stride_dim == 1 && aligned16(a.cos) && aligned16(a.sin) && half_bytes % 16 == 0 &&
                       2 * half_bytes <= kCsRawBytes && (a.cs_stride_seq * static_cast<int64_t>(sizeof(TCS))) % 16 == 0;
  kern<<<static_cast<unsigned>(grid), warps * 32, smem, st>>>(
      static_cast<const TX*>(a.x), a.weight, static_cast<const TCS*>(a.cos), static_cast<const TCS*>(a.sin),
      static_cast<TX*>(a.out), rows, static_cast<int>(a.seq_len), static_cast<int>(a.hidden),
      static_cast<int>(a.head_dim), static_cast<int>(a.num_heads * a.head_dim), a.cs_stride_seq, a.cs_stride_dim,
      a.eps, a.w_dtype, cs_stride, cs_bulk, error_word_ptr(), q);
  note_launch();
  return cudaGetLastError();
}

template <typename TX, typename TCS, bool FULLROT, int VPL>
cudaError_t launch_warp_rows_t(const RmsNormRopeArgs& a, int warps, int cs_stride, size_t smem, int mode,
                               const RowQuantArgs& q, cudaStream_t st) {
  switch (mode) {
    case 3: return launch_warp_rows_m<TX, TCS, FULLROT, VPL, 3>(a, warps, cs_stride, smem, q, st);
    default: return launch_warp_rows_m<TX, TCS, FULLROT, VPL, 0>(a, warps, cs_stride, smem, q, st);
  }
}

// Warps per CTA (one CTA per SM, at most 16) so that the row buffers, the
// fp32 weight row and the per-warp cos/sin buffers fit in shared memory.
inline int warp_rows_config(int64_t hidden, int64_t head_dim, int elem, int max_warps, int* cs_stride, size_t* smem) {
  const size_t row_bytes = static_cast<size_t>(hidden) * elem;
  *cs_stride = static_cast<int>((3 * (head_dim / 2) + 3) / 4 * 4);
  const size_t fixed = kWarpBarBytes + static_cast<size_t>(hidden) * 4 + 128;
  const size_t per_warp = kWarpSlots * (row_bytes + kCsRawBytes) + static_cast<size_t>(*cs_stride) * 4;
  const size_t limit = 227 * 1024 - 256;  // room for the kernel's static shared memory
  if (fixed + 8 * per_warp > limit) return 0;
  const int warps = static_cast<int>(std::min<size_t>(max_warps, (limit - fixed) / per_warp));
  *smem = ((kWarpBarBytes + (static_cast<size_t>(hidden) + warps * *cs_stride) * 4 + 127) / 128) * 128 +
          warps * kWarpSlots * (row_bytes + kCsRawBytes);
  return warps;
}

template <typename TX, typename TCS, int VPL>
cudaError_t launch_warp_rows_v(const RmsNormRopeArgs& a, int warps, int cs_stride, size_t smem, int mode,
                               const RowQuantArgs& q, cudaStream_t st) {
  return (a.num_heads * a.head_dim == a.hidden)
             ? launch_warp_rows_t<TX, TCS, true, VPL>(a, warps, cs_stride, smem, mode, q, st)
             : launch_warp_rows_t<TX, TCS, false, VPL>(a, warps, cs_stride, smem, mode, q, st);
}

template <typename TX, typename TCS>
cudaError_t launch_warp_rows(const RmsNormRopeArgs& a, int vpl, int warps, int cs_stride, size_t smem, int mode,
                             const RowQuantArgs& q, cudaStream_t st) {
  switch (vpl) {
    case 4: return launch_warp_rows_v<TX, TCS, 4>(a, warps, cs_stride, smem, mode, q, st);
    case 8: return launch_warp_rows_v<TX, TCS, 8>(a, warps, cs_stride, smem, mode, q, st);
    default: return launch_warp_rows_v<TX, TCS, 16>(a, warps, cs_stride, smem, mode, q, st);
  }
}

template <typename TX, typename TCS>
cudaError_t launch_cta_vec(const RmsNormRopeArgs& a, const RmsPlan& p, cudaStream_t st) {
  switch (p.vec) {
    case 1: return p.full ? launch_vec<TX, TCS, 1, true>(a, p.threads, st) : launch_vec<TX, TCS, 1, false>(a, p.threads, st);
    case 2: return p.full ? launch_vec<TX, TCS, 2, true>(a, p.threads, st) : launch_vec<TX, TCS, 2, false>(a, p.threads, st);
    case 4: return p.full ? launch_vec<TX, TCS, 4, true>(a, p.threads, st) : launch_vec<TX, TCS, 4, false>(a, p.threads, st);
    default: return p.full ? launch_vec<TX, TCS, 8, true>(a, p.threads, st) : launch_vec<TX, TCS, 8, false>(a, p.threads, st);
  }
}

template <typename TX>
cudaError_t dispatch_warp_rows(const RmsNormRopeArgs& a, const RmsPlan& p, int mode, const RowQuantArgs& q,
                               cudaStream_t st) {
  switch (a.cos_dtype) {
    case F16: return launch_warp_rows<TX, __half>(a, p.vec, p.threads, p.cs_stride, p.smem, mode, q, st);
    case BF16: return launch_warp_rows<TX, __nv_bfloat16>(a, p.vec, p.threads, p.cs_stride, p.smem, mode, q, st);
    default: return launch_warp_rows<TX, float>(a, p.vec, p.threads, p.cs_stride, p.smem, mode, q, st);
  }
}

template <typename TX>
cudaError_t dispatch_plan(const RmsNormRopeArgs& a, const RmsPlan& p, cudaStream_t st) {
  if (p.kind == 2) return dispatch_warp_rows<TX>(a, p, 0, RowQuantArgs{}, st);
  switch (a.cos_dtype) {
    case F16: return launch_cta_vec<TX, __half>(a, p, st);
    case BF16: return launch_cta_vec<TX, __nv_bfloat16>(a, p, st);
    default: return launch_cta_vec<TX, float>(a, p, st);
  }
}

template <typename TX>
cudaError_t launch_generic(const RmsNormRopeArgs& a, cudaStream_t st) {
  const int64_t rows = a.batch * a.seq_len;
  const size_t smem = static_cast<size_t>(a.hidden) * sizeof(float);
  auto kern = rmsnorm_rope_generic_kernel<TX>;
  if (cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(kern), smem); e != cudaSuccess) return e;
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

}  // namespace

// Chooses the vectorised path when the row, head and table layout allow it.
// Kernel choice for a shape (the static launch table):
//  * kind 2, warp per row: the row is 4, 8 or 16 16-byte vectors per lane and
//    there are at least two rows per warp slot of a full wave;
//  * kind 1, CTA per row: `threads` threads with `vec` 16-byte vectors each;
//  * kind 0, generic: any shape, dtype mix or alignment.
RmsPlan rmsnorm_rope_plan(int64_t rows, int64_t hidden, int64_t head_dim, int64_t num_heads, int esz, bool vec_ok) {
  RmsPlan p{};
  p.kind = 0;
  p.threads = 256;
  const int E = 16 / esz;
  const int64_t D = head_dim;
  const int64_t dv = D / E;
  const bool vec = vec_ok && (hidden % E == 0) && (D % (2 * E) == 0) && dv >= 2 && dv <= 32 && (dv & (dv - 1)) == 0 &&
                   (hidden / E) <= 8 * 256;
  if (!vec) return p;
  const int nvec = static_cast<int>(hidden / E);
  const int vpl = nvec / 32;
  const bool vpl_ok = (nvec % 32 == 0) && (vpl == 4 || vpl == 8 || vpl == 16);
  int cs_stride = 0;
  size_t smem = 0;
  const int warps = vpl_ok ? warp_rows_config(hidden, D, esz, warp_rows_max_warps(vpl), &cs_stride, &smem) : 0;
  if (warps > 0 && rows >= 2ll * num_sms() * warps) {
    p.kind = 2;
    p.threads = warps;
    p.vec = vpl;
    p.full = (num_heads * D == hidden);
    p.cs_stride = cs_stride;
    p.smem = smem;
    return p;
  }
  for (int nv : {1, 2, 4, 8}) {
    const int threads = ((nvec + nv - 1) / nv + 31) / 32 * 32;
    if (threads <= 256) {
      p.kind = 1;
      p.threads = threads;
      p.vec = nv;
      p.full = (nv * threads == nvec) && (num_heads * D == hidden);
      return p;
    }
  }
  return p;
}

cudaError_t rmsnorm_rope_quant_launch(const RmsNormRopeArgs& a, int mode, const RowQuantArgs& q, int* nparts,
                                      cudaStream_t st) {
  const int esz = (a.x_dtype == F32) ? 4 : 2;
  const bool ok = aligned16(a.x) && aligned16(a.out) && a.cos_dtype == a.sin_dtype;
  // only where tfo_rmsnorm_rope itself runs the warp-per-row kernel, so that the
  // rows (and their rounding) are exactly those of the unfused op
  const RmsPlan p = rmsnorm_rope_plan(a.batch * a.seq_len, a.hidden, a.head_dim, a.num_heads, esz, ok);
  if (p.kind != 2) return cudaErrorNotSupported;
  *nparts = static_cast<int>(warp_rows_grid(a.batch * a.seq_len, p.threads));
  switch (a.x_dtype) {
    case F16: return dispatch_warp_rows<__half>(a, p, mode, q, st);
    case BF16: return dispatch_warp_rows<__nv_bfloat16>(a, p, mode, q, st);
    default: return dispatch_warp_rows<float>(a, p, mode, q, st);
  }
}

int rmsnorm_rope_quant_max_parts() { return num_sms(); }

cudaError_t rmsnorm_rope_launch(const RmsNormRopeArgs& a, cudaStream_t st) {
  const int esz = (a.x_dtype == F32) ? 4 : 2;
  const bool vec_ok = aligned16(a.x) && aligned16(a.out) && a.cos_dtype == a.sin_dtype;
  const RmsPlan p = rmsnorm_rope_plan(a.batch * a.seq_len, a.hidden, a.head_dim, a.num_heads, esz, vec_ok);
  if (p.kind != 0) {
    switch (a.x_dtype) {
      case F16: return dispatch_plan<__half>(a, p, st);
      case BF16: return dispatch_plan<__nv_bfloat16>(a, p, st);
      default: return dispatch_plan<float>(a, p, st);
    }
  }
  switch (a.x_dtype) {
    case F16: return launch_generic<__half>(a, st);
    case BF16: return launch_generic<__nv_bfloat16>(a, st);
    default: return launch_generic<float>(a, st);
  }
}

}  // namespace tfo
