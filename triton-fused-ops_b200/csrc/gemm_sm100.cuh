// Persistent, warp-specialised tcgen05 GEMM mainloop for sm_100a.
// `idesc` must describe an M = 128, N = NUM_B * BLOCK_N instruction.
//
//   D[m, n] (+)= sum_k A[m, k] * B_j[n, k]        for j < NUM_B
//
// A and every B_j are K-major (rows of K), staged by TMA into a STAGES-deep
// shared-memory ring with the 128-byte swizzle; one elected thread issues
// tcgen05.mma (M = 128, N = BLOCK_N, 32 bytes of K per instruction) into a
// double-buffered TMEM accumulator (2 x NUM_B x BLOCK_N columns), and the
// epilogue warps drain the finished buffer with tcgen05.ld while the next
// tile's mainloop runs. NUM_B = 2 shares every A tile between two B operands
// (the gate and up projections of the gated MLP).
//
// Warp roles (64 + 32 * EPI_WARPS threads): warp 0 = TMA producer, warp 1 =
// MMA issuer and TMEM owner, warps 2.. = epilogue. Epilogue warp w reads TMEM
// lanes 32*(w%4)..+31 (the lanes its sub-partition may access); with 8
// epilogue warps two warps share those lanes and each drains half of the
// tile's columns, so that every scheduler has two epilogue warps to
// interleave (one warp alone leaves every instruction latency exposed).
//
// Every mbarrier wait is bounded; a wait that runs out of budget records a
// bit in the device error word, raises a CTA-wide abort flag that the other
// roles poll, and all roles fall through to the final barrier, where TMEM is
// released. No TMA multicast is used.
#pragma once

#include "common.cuh"

namespace tfo {

template <MmaKind KIND> struct KindTraits;
template <> struct KindTraits<MmaKind::F16> { static constexpr int ELEM = 2; };
template <> struct KindTraits<MmaKind::TF32> { static constexpr int ELEM = 4; };
template <> struct KindTraits<MmaKind::I8> { static constexpr int ELEM = 1; };
template <> struct KindTraits<MmaKind::F8F6F4> { static constexpr int ELEM = 1; };

struct TileSched {
  int num_m, num_n, group_m;
  __device__ __forceinline__ int num_tiles() const { return num_m * num_n; }
  // Grouped raster: GROUP_M row-blocks sweep the column-blocks together so the
  // B tiles and the A rows of a wave stay resident in L2.
  __device__ __forceinline__ void coords(int tile, int& m_blk, int& n_blk) const {
    const int in_group = group_m * num_n;
    const int g = tile / in_group;
    const int first_m = g * group_m;
    const int gsz = min(num_m - first_m, group_m);
    const int r = tile - g * in_group;
    m_blk = first_m + r % gsz;
    n_blk = r / gsz;
  }
};

// Per-CTA shared-memory layout. The UMMA is M = 128 * CG by N = NUM_B *
// BLOCK_N; each CTA stages A_ROWS rows of A and N / CG rows of B per K block.
// Stage s is [A_ROWS rows of A | B tile] at s * STAGE_BYTES.
// A_ROWS < 128 (one CTA per MMA, M <= A_ROWS): the A stages are smaller, so
// more stages fit; the MMA still reads 128 rows from the A tile's start, and
// the rows past A_ROWS are the first bytes of the same stage's B tile. Those
// landed before the MMA's wait on the stage's full barrier and are not
// rewritten before the MMA commits the stage as empty, so the extra rows read
// settled memory; the accumulator rows they feed lie past M and are never
// stored or exchanged.
template <int BLOCK_N, int NUM_B, int STAGES, int CG = 1, bool KSPLIT = false, int A_ROWS = 128>
struct GemmLayout {
  static constexpr int BM = 128;             // accumulator lanes (output rows) per CTA
  static constexpr int PAIR_M = BM * CG;     // rows per tile
  static constexpr int A_BYTES = A_ROWS * 128;
  static_assert(A_ROWS % 8 == 0 && A_ROWS <= BM && (A_ROWS == BM || CG == 1), "A stage rows");
  static constexpr int N_MMA = NUM_B * BLOCK_N;
  static constexpr int B_ROWS = N_MMA / CG;  // B rows staged by one CTA
  static constexpr int B_STAGE_BYTES = B_ROWS * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_STAGE_BYTES;
  static constexpr int ACC_COLS = N_MMA;
  static constexpr int TMEM_COLS = 2 * ACC_COLS;
  static_assert(CG == 1 || CG == 2, "one or two CTAs per MMA");
  static_assert(TMEM_COLS <= 512 && (TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM columns must be a power of two <= 512");
  static_assert(BLOCK_N % 16 == 0 && BLOCK_N >= 16 && N_MMA <= 256, "UMMA N");
  static_assert(CG == 1 || (B_ROWS % 128 == 0 && (NUM_B == 1 || B_ROWS == BLOCK_N)),
                "pair MMA: each CTA stages whole 128-row B boxes (one operand each when NUM_B == 2)");
  static_assert(!KSPLIT || (CG == 1 && NUM_B == 1), "cluster K split: one CTA per MMA, one B operand");
  static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
  // cluster K split: the raw accumulator tile (read by the cluster's other
  // CTAs) and the tile of this CTA's summed rows (at most half the rows, as
  // k_splits >= 2). Both reuse the ring: a K-split CTA runs one work item,
  // and once its accumulator is complete no TMA write or MMA read of the ring
  // remains.
  static constexpr int RED_BYTES = KSPLIT ? BM * N_MMA * 4 : 0;
  static constexpr int SUM_OFFSET = RED_BYTES;
  static constexpr int SUM_BYTES = KSPLIT ? (BM / 2) * N_MMA * 4 : 0;
  static_assert(RED_BYTES + SUM_BYTES <= RING_BYTES, "reduction tiles fit in the ring");
  static_assert(A_ROWS == BM || STAGE_BYTES >= BM * 128,
                "a 128-row read from a short A tile stays inside its own stage");
  static_assert(A_BYTES % 1024 == 0 && B_STAGE_BYTES % 1024 == 0, "128-byte-swizzled tiles on 1 KB boundaries");
  static constexpr int BAR_OFFSET = RING_BYTES;
  // dynamic shared memory: ring + barriers + 1 KB for manual alignment
  static constexpr size_t SMEM_BYTES = static_cast<size_t>(BAR_OFFSET) + 256 + 1024;
};

// Address of 16-byte vector `v` of row `row` in a K-split reduction tile
// (VECS_PER_ROW vectors per row, XOR-swizzled by row: a warp storing one
// vector of 32 rows, or reading 16 columns of 4 rows, spreads over all banks).
template <int VECS_PER_ROW>
__device__ __forceinline__ int red_vec_index(int row, int v) {
  return row * VECS_PER_ROW + (v ^ (row & 7));
}

__device__ __forceinline__ uint4 ld_dsmem_v4(uint32_t cluster_addr) {
  uint4 r;
  asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"(cluster_addr)
               : "memory");
  return r;
}

// Barrier 1 over the epilogue warps (barrier 0 is __syncthreads).
__device__ __forceinline__ void epilogue_warps_sync(int threads) {
  asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}

// Threads of a GEMM kernel with EPI_WARPS epilogue warps.
constexpr int gemm_threads(int epi_warps) { return 64 + 32 * epi_warps; }

// Waits for `parity` on `bar`, giving up when the CTA abort flag is raised or
// the budget runs out (then sets the error bit and raises the flag).
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag, uint32_t* err,
                                              uint32_t bit) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitBudgetCycles) {
      set_error(err, bit);
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}

// Epi must provide:
//   struct Params;
//   struct State;  per epilogue thread: values derived once from Params, running values
//   static __device__ State init(const Params&);
//   __device__ void operator()(const Params&, State&, const uint32_t (&acc)[NUM_B][16], int row, int col0,
//                              int M, int N, int split)
//   called once per 16 accumulator columns per row (row < M not guaranteed);
//   static __device__ void finish(const Params&, State&)
//   called by every epilogue thread (EPI_WARPS full warps) after its last tile.
//
// B_MN: the B operand is MN-major (B given as [K, N] with N contiguous, as
// the reference's fp8_gemm passes it); each stage then holds B_ROWS / 128
// boxes of [128 K rows x 128 bytes of N], chained by the descriptor's
// leading-byte offset. Only for 8-bit operands and NUM_B == 1.
//
// k_splits > 1 splits the K loop: work item w covers tile w / k_splits and
// the K blocks of slice w % k_splits; the epilogue receives the slice index.
//
// CG == 2: launched as clusters of two CTAs (consecutive blockIdx.x). Both
// CTAs walk the same tile list; CTA r of the pair loads A rows
// [tile_m + 128 r, +128) and B rows [r * B_ROWS, +B_ROWS) of the tile's N
// range (for NUM_B == 2: operand r), with the transaction bytes reported to
// the even CTA's `full` barrier. The even CTA issues the M = 256 MMAs and
// commits to the `empty` / `tfull` barriers of both CTAs; the epilogue warps
// of both CTAs release the accumulator on the even CTA's `tempty` barrier.
//
// KSPLIT: the k_splits K slices of a tile run as one cluster of k_splits CTAs
// (one work item per CTA, grid = tiles x k_splits). Each CTA leaves its raw
// accumulator tile (rows inside M) in shared memory over the drained ring.
// After a cluster barrier CTA r takes the r-th of k_splits contiguous row
// blocks of the tile's rows inside M: a warp reads one row of every slice's
// tile through distributed shared memory (lane l: 16-byte vector l, so each
// request is 512 contiguous bytes; four rows' requests in flight), sums the
// slices in slice order into a local tile of sums, and after a barrier of
// the epilogue warps the epilogue runs on 16-column units of that tile (Epi
// must provide add_partial and final_params). A second cluster barrier keeps
// every tile readable until all CTAs are done. 2 <= k_splits <= 8.
template <MmaKind KIND, int BLOCK_N, int NUM_B, int STAGES, class Epi, bool B_MN = false, int CG = 1,
          bool KSPLIT = false, int EPI_WARPS = 4, int A_ROWS = 128>
__global__ void __launch_bounds__(gemm_threads(EPI_WARPS), 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b0,
                     const __grid_constant__ CUtensorMap tmap_b1, int M, int N, int K, int group_m, uint32_t idesc,
                     const typename Epi::Params ep, uint32_t* err, int k_splits) {
  griddep_launch_dependents();  // a programmatic-dependent GEMM after this one may be scheduled as CTAs retire
  static_assert(!B_MN || (NUM_B == 1 && KindTraits<KIND>::ELEM == 1 && BLOCK_N % 128 == 0),
                "MN-major B: 8-bit operands, one B operand, BLOCK_N a multiple of 128");
  using L = GemmLayout<BLOCK_N, NUM_B, STAGES, CG, KSPLIT, A_ROWS>;
  constexpr int KB_ELEMS = 128 / KindTraits<KIND>::ELEM;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // stage s: A tile at sa + s * STAGE_BYTES, B tile at sb + s * STAGE_BYTES
  uint8_t* sa = smem;
  uint8_t* sb = smem + L::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFFSET);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = (CG == 2) ? (cluster_ctarank() & 1u) : 0u;  // position in the pair
  const bool leader = (rank == 0);
  const int unit = blockIdx.x / CG, num_units = gridDim.x / CG;
  TileSched sched{(M + L::PAIR_M - 1) / L::PAIR_M, (N + BLOCK_N - 1) / BLOCK_N, group_m};
  const int num_tiles = sched.num_tiles();
  const int num_k = (K + KB_ELEMS - 1) / KB_ELEMS;
  const int num_work = num_tiles * k_splits;
  // work item -> (tile, K-block range, slice); slices differ by at most one
  // K block, so none is empty while k_splits <= num_k (the host's split rule)
  struct Work {
    int m_blk, n_blk, kb0, kb1, split;
  };
  auto work = [&](int w) {
    Work r;
    const int tile = w / k_splits;
    r.split = w - tile * k_splits;
    sched.coords(tile, r.m_blk, r.n_blk);
    // floor(split * num_k / k_splits) in 32-bit arithmetic without the product
    r.kb0 = r.split * (num_k / k_splits) + (r.split * (num_k % k_splits)) / k_splits;
    r.kb1 = (r.split + 1) * (num_k / k_splits) + ((r.split + 1) * (num_k % k_splits)) / k_splits;
    return r;
  };
  uint4* red_tile = reinterpret_cast<uint4*>(smem);
  if constexpr (KSPLIT) {
    // the reduction tiles reuse the ring, which holds for one work item per CTA
    if (static_cast<int>(gridDim.x) != num_work) {
      if (threadIdx.x == 0) atomicOr(err, ERR_BAD_LAUNCH);
      return;  // uniform over the grid: no CTA reaches a barrier
    }
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EPI_WARPS * CG);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b0);
    if (NUM_B == 2) tma_prefetch_desc(&tmap_b1);
  }
  if (warp == 1) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(tmem_slot, L::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, L::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // everything above overlaps the previous kernel when launched as a
  // programmatic dependent; global memory is touched only after this
  griddep_wait();
  // epilogue state (a K split's final pass reuses it: its epilogue keeps no
  // per-tile state)
  typename Epi::State est{};

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      for (int w = unit; w < num_work && !*abort_flag; w += num_units) {
        const Work wk = work(w);
        const int m_row = wk.m_blk * L::PAIR_M + static_cast<int>(rank) * L::BM;
        for (int kb = wk.kb0; kb < wk.kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!wait_or_abort(&empty[s], ph ^ 1, abort_flag, err, ERR_WAIT_TIMEOUT_PRODUCER)) break;
          const int kx = kb * KB_ELEMS;
          uint8_t* a_dst = sa + s * L::STAGE_BYTES;
          uint8_t* b_dst = sb + s * L::STAGE_BYTES;
          if constexpr (CG == 1) {
            mbar_arrive_expect_tx(&full[s], L::STAGE_BYTES);
            tma_load_2d(a_dst, &tmap_a, &full[s], kx, m_row);
            if constexpr (B_MN) {
#pragma unroll
              for (int c = 0; c < L::B_ROWS / 128; ++c)
                tma_load_2d(b_dst + c * (128 * 128), &tmap_b0, &full[s], wk.n_blk * BLOCK_N + c * 128, kx);
            } else {
              tma_load_2d(b_dst, &tmap_b0, &full[s], kx, wk.n_blk * BLOCK_N);
              if constexpr (NUM_B == 2) tma_load_2d(b_dst + BLOCK_N * 128, &tmap_b1, &full[s], kx, wk.n_blk * BLOCK_N);
            }
          } else {
            // both CTAs' bytes complete the even CTA's full[s]
            const uint32_t bar = mapa_shared(smem_u32(&full[s]), 0);
            if (leader) mbar_arrive_expect_tx(&full[s], 2 * L::STAGE_BYTES);
            tma_load_2d_pair(a_dst, &tmap_a, bar, kx, m_row);
            if constexpr (B_MN) {
#pragma unroll
              for (int c = 0; c < L::B_ROWS / 128; ++c)
                tma_load_2d_pair(b_dst + c * (128 * 128), &tmap_b0, bar,
                                 wk.n_blk * BLOCK_N + static_cast<int>(rank) * L::B_ROWS + c * 128, kx);
            } else if constexpr (NUM_B == 2) {
              tma_load_2d_pair(b_dst, rank == 0 ? &tmap_b0 : &tmap_b1, bar, kx, wk.n_blk * BLOCK_N);
            } else {
              tma_load_2d_pair(b_dst, &tmap_b0, bar, kx, wk.n_blk * BLOCK_N + static_cast<int>(rank) * L::B_ROWS);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      // pair commits go to this CTA's and the peer's barrier at the same offset
      const uint32_t peer = rank ^ 1u;
      int it = 0, tcount = 0;
      for (int w = unit; w < num_work && !*abort_flag; w += num_units, ++tcount) {
        const Work wk = work(w);
        const int kb0 = wk.kb0, kb1 = wk.kb1;
        const int acc = tcount & 1;
        const uint32_t aph = (tcount >> 1) & 1;
        if (!wait_or_abort(&tempty[acc], aph ^ 1, abort_flag, err, ERR_WAIT_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * L::ACC_COLS;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!wait_or_abort(&full[s], ph, abort_flag, err, ERR_WAIT_TIMEOUT_MMA)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sa + s * L::STAGE_BYTES);
          const uint32_t b_addr = smem_u32(sb + s * L::STAGE_BYTES);
          // With CG == 1 the NUM_B B tiles of a stage are consecutive
          // 128-byte-swizzled K-major tiles, i.e. one (NUM_B * BLOCK_N)-row
          // tile, so a single UMMA of N = NUM_B * BLOCK_N reads the A tile
          // once for all of them; accumulator column j * BLOCK_N + c belongs
          // to B operand j. With CG == 2 the two halves of N sit in the two
          // CTAs at the same offset.
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t adesc = smem_desc_kmajor_sw128(a_addr + kk * 32);
            // MN-major B: 32 K rows of 128 bytes per instruction = 4 swizzle atoms
            const uint64_t bdesc = B_MN ? smem_desc_mnmajor_sw128(b_addr + kk * 4096, 128 * 128)
                                        : smem_desc_kmajor_sw128(b_addr + kk * 32);
            const uint32_t accum = (kb != kb0 || kk != 0) ? 1u : 0u;
            if constexpr (CG == 2) umma_pair<KIND>(d_tmem, adesc, bdesc, idesc, accum);
            else umma<KIND>(d_tmem, adesc, bdesc, idesc, accum);
          }
          if constexpr (CG == 2) {
            umma_commit_pair(smem_u32(&empty[s]));
            umma_commit_pair(mapa_shared(smem_u32(&empty[s]), peer));
          } else {
            umma_commit(&empty[s]);
          }
        }
        if (!ok) break;
        if constexpr (CG == 2) {
          umma_commit_pair(smem_u32(&tfull[acc]));
          umma_commit_pair(mapa_shared(smem_u32(&tfull[acc]), peer));
        } else {
          umma_commit(&tfull[acc]);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "one or two epilogue warps per TMEM sub-partition");
    constexpr int COLS = BLOCK_N / (EPI_WARPS / 4);  // columns per epilogue warp (per B operand)
    static_assert(COLS % 32 == 0, "epilogue walks 32 columns per iteration");
    const int sub = warp & 3;
    const int col_lo = ((warp - 2) >> 2) * COLS;  // this warp's first column of the tile
    const int row_in_tile = static_cast<int>(rank) * L::BM + sub * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(sub * 32) << 16;
    est = Epi::init(ep);
    int tcount = 0;
    for (int w = unit; w < num_work; w += num_units, ++tcount) {
      const int acc = tcount & 1;
      const uint32_t aph = (tcount >> 1) & 1;
      if (!wait_or_abort(&tfull[acc], aph, abort_flag, err, ERR_WAIT_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const Work wk = work(w);
      const int row = wk.m_blk * L::PAIR_M + row_in_tile;
      const uint32_t base = tmem_base + lane_addr + acc * L::ACC_COLS;
      // Two register sets: the TMEM load of the next 16 columns is in flight
      // while the current ones are converted and stored.
      if (wk.m_blk * L::PAIR_M + row_in_tile - lane >= M) {
        // all 32 rows of this warp lie past M: nothing to read or store
        __syncwarp();
        if (lane == 0) {
          if constexpr (CG == 2) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
          else mbar_arrive(&tempty[acc]);
        }
        continue;
      }
      if constexpr (KSPLIT) {
        // raw accumulators to the reduction tile (row = this thread's TMEM lane)
        const int trow = sub * 32 + lane;
#pragma unroll 1
        for (int c = col_lo; c < col_lo + COLS; c += 16) {
          uint32_t r[16];
          tmem_ld16(base + c, r);
          tmem_ld_wait();
          tmem_ld_fence(r);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            red_tile[red_vec_index<L::N_MMA / 4>(trow, c / 4 + q)] =
                make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        continue;
      }
      uint32_t ra[NUM_B][16], rb[NUM_B][16];
#pragma unroll
      for (int j = 0; j < NUM_B; ++j) tmem_ld16(base + j * BLOCK_N + col_lo, ra[j]);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < NUM_B; ++j) tmem_ld_fence(ra[j]);
#pragma unroll 1
      for (int c = col_lo; c < col_lo + COLS; c += 32) {
#pragma unroll
        for (int j = 0; j < NUM_B; ++j) tmem_ld16(base + j * BLOCK_N + c + 16, rb[j]);
        Epi{}(ep, est, ra, row, wk.n_blk * BLOCK_N + c, M, N, wk.split);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < NUM_B; ++j) tmem_ld_fence(rb[j]);
        if (c + 32 < col_lo + COLS) {
#pragma unroll
          for (int j = 0; j < NUM_B; ++j) tmem_ld16(base + j * BLOCK_N + c + 32, ra[j]);
        }
        Epi{}(ep, est, rb, row, wk.n_blk * BLOCK_N + c + 16, M, N, wk.split);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < NUM_B; ++j) tmem_ld_fence(ra[j]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CG == 2) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
        else mbar_arrive(&tempty[acc]);
      }
    }
    Epi::finish(ep, est);
  }

  __syncthreads();
  if constexpr (KSPLIT) {
    cluster_sync();  // every slice's tile is in shared memory
    if (warp >= 2) {
      constexpr int VECS = L::N_MMA / 4;
      constexpr int CHUNKS = BLOCK_N / 16;
      constexpr int MAX_SPLITS = 8;
      constexpr int ROWS_IN_FLIGHT = 4;
      static_assert(VECS == 32, "one 16-byte vector of a row per lane");
      const typename Epi::Params epf = Epi::final_params(ep);
      const Work wk = work(blockIdx.x);
      const int row0 = wk.m_blk * L::PAIR_M;
      const int rows = max(0, min(L::BM, M - row0));
      const int per = (rows + k_splits - 1) / k_splits;  // <= BM / 2 rows
      const int r_begin = min(rows, static_cast<int>(cluster_ctarank()) * per);
      const int r_end = min(rows, r_begin + per);
      const uint32_t tile_base = smem_u32(red_tile);
      uint4* sum_tile = reinterpret_cast<uint4*>(smem + L::SUM_OFFSET);
      // 1. epilogue warp w sums rows r_begin + w, + EPI_WARPS, ...: lane l holds vector l of the row
      for (int r = r_begin + (warp - 2); r < r_end; r += EPI_WARPS * ROWS_IN_FLIGHT) {
        uint4 v[ROWS_IN_FLIGHT][MAX_SPLITS];
#pragma unroll
        for (int i = 0; i < ROWS_IN_FLIGHT; ++i) {
          const int ri = r + EPI_WARPS * i;
          const uint32_t off = static_cast<uint32_t>(red_vec_index<VECS>(ri, lane)) * 16u;
#pragma unroll
          for (int sl = 0; sl < MAX_SPLITS; ++sl)
            if (ri < r_end && sl < k_splits) v[i][sl] = ld_dsmem_v4(mapa_shared(tile_base + off, static_cast<uint32_t>(sl)));
        }
#pragma unroll
        for (int i = 0; i < ROWS_IN_FLIGHT; ++i) {
          const int ri = r + EPI_WARPS * i;
          if (ri >= r_end) break;
          uint4 t = v[i][0];
#pragma unroll
          for (int sl = 1; sl < MAX_SPLITS; ++sl) {
            if (sl < k_splits) {
              t.x = Epi::add_partial(t.x, v[i][sl].x);
              t.y = Epi::add_partial(t.y, v[i][sl].y);
              t.z = Epi::add_partial(t.z, v[i][sl].z);
              t.w = Epi::add_partial(t.w, v[i][sl].w);
            }
          }
          sum_tile[red_vec_index<VECS>(ri - r_begin, lane)] = t;
        }
      }
      epilogue_warps_sync(32 * EPI_WARPS);
      // 2. the epilogue on 16-column units of the summed rows
      const int units = (r_end - r_begin) * CHUNKS;
      for (int u = threadIdx.x - 64; u < units; u += 32 * EPI_WARPS) {
        const int lr = u / CHUNKS, c = (u % CHUNKS) * 16;
        uint32_t sum[1][16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 t = sum_tile[red_vec_index<VECS>(lr, c / 4 + q)];
          sum[0][4 * q] = t.x;
          sum[0][4 * q + 1] = t.y;
          sum[0][4 * q + 2] = t.z;
          sum[0][4 * q + 3] = t.w;
        }
        Epi{}(epf, est, sum, row0 + r_begin + lr, wk.n_blk * BLOCK_N + c, M, N, 0);
      }
    }
    cluster_sync();  // no CTA leaves while the others may still read its tile
  }
  if constexpr (CG == 2) cluster_sync();  // no CTA leaves while its pair may still touch its memory
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (CG == 2) tmem_dealloc_pair(tmem_base, L::TMEM_COLS);
    else tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

}  // namespace tfo
