// Persistent, warp-specialised dense GEMM for sm_100a:
//   C[l] (M x N, BF16 or FP32) = A[l] (M x K, BF16, K-major) * B[l]^T (N x K, BF16, K-major)
//
// This is the kernel that takes the three CuTe DSL candidate slots of the
// reference driver (gemm_comparison/gemm_comparison.py:209-260:
// nonpersistent_1cta, persistent_1cta, persistent_2cta) plus a tuned slot.
//
// Roles inside one CTA (192 threads, one CTA per SM):
//   warp 0      TMA producer: one lane streams A/B k-blocks (64 BF16 wide,
//               128-byte swizzle) into a STAGES-deep shared-memory ring.
//   warp 1      TMEM allocator for the CTA, and (in the MMA CTA of the
//               cluster) the single-thread tcgen05.mma issuer accumulating
//               FP32 in a double-buffered TMEM accumulator.
//   warps 2-5   epilogue warpgroup: tcgen05.ld of its 32 TMEM lanes,
//               conversion to BF16 (or FP32 pass-through), 128-byte-swizzled
//               staging in shared memory and a TMA store per 32x128-byte box.
//
// CTA-pair mode (kCG == 2): a cluster of two CTAs computes a 256 x BN tile
// with tcgen05.mma.cta_group::2. Each CTA TMA-loads its own 128 rows of A
// and its own BN/2 rows of B into its own shared memory; both loads
// complete on the full barrier of CTA rank 0, whose single thread issues the
// MMAs and signals both CTAs' barriers with one tcgen05.commit each. Every
// TMA load fetches from global memory into its own CTA only.
//
// The tile scheduler is static and persistent: cluster c processes tiles
// c, c + nclusters, ... in a grouped raster order (group_m tile-rows swept
// across all tile-columns) so the A rows and B columns a wave touches stay
// in L2.
#include <cuda.h>
#include <cuda_bf16.h>

#include <cmath>
#include <cstdlib>

#include "common.cuh"
#include "gemm_sm100.cuh"
#include "ptx.cuh"

namespace bb {
namespace gemm {

// Most clusters a stream-K region is cut over (one per SM of a B200).
constexpr int kMaxSkClusters = 148;

struct Params {
  int32_t m, n, k, l;
  int32_t tiles_m, tiles_n;
  int32_t num_tiles;
  int32_t k_blocks;
  int32_t group_m;
  int32_t num_clusters;
  // Data-parallel tiles [0, dp_tiles) go to cluster t % num_clusters with
  // the full K range. The remaining sk_tiles tiles form one stream-K region:
  // its sk_tiles * k_blocks (tile, k-block) iterations, tile-major, are cut
  // into num_clusters contiguous ranges (sk_begin), one per cluster, run
  // after that cluster's data-parallel tiles. A range cut inside a tile
  // makes a partial piece; the pieces of a tile are fixed up by whichever
  // finishes last (no piece ever waits for another).
  int32_t dp_tiles;
  // Narrow tail: tiles [dp_tiles, dp_tiles + narrow_tiles) are each computed
  // as two half-width tiles (N / 2 columns each) by clusters 2 t and 2 t + 1
  // of the tail, so a partial last wave of 256-wide tiles becomes one wave
  // of half tiles on twice as many clusters. Exclusive with stream-K.
  int32_t narrow_tiles;
  int32_t sk_tiles;  // 0: no stream-K region
  // First stream-K iteration of clusters 0..num_clusters (entry c + 1 ends
  // cluster c's range); the region has fewer than 2^31 iterations.
  int32_t sk_bounds[kMaxSkClusters + 1];
  float* partials;   // FP32 partial tiles, two slots per cluster and CTA rank
  int* counters;     // k-blocks accumulated so far, one per stream-K tile and CTA rank
  int* status;
  // Epilogue D = alpha * acc + beta * Csrc (epi_mode 0: alpha 1, beta 0;
  // 1: alpha only; 2: alpha and beta). Csrc has the output's dtype and
  // (L, M, N) row-major layout and may alias the output.
  int32_t epi_mode;
  int32_t spin;  // bit 0: the producer's slot waits spin; bit 1: the MMA warp's stage waits spin
  float alpha, beta;
  const void* c_src;
};

// alpha * v[j] (+ beta * Csrc[l][row][col + j]) for kCount consecutive
// columns of one row; Csrc elements past N (or a row past M) read as 0.
// Fully unrolled so v stays in registers.
template <bool kOutF32, int kCount>
__device__ __forceinline__ void apply_epilogue(const Params& p, float (&v)[kCount], int row, int col, int l) {
  if (p.epi_mode == 0) return;
#pragma unroll
  for (int j = 0; j < kCount; ++j) v[j] *= p.alpha;
  if (p.epi_mode != 2 || row >= p.m) return;
  const int64_t base = (static_cast<int64_t>(l) * p.m + row) * p.n + col;
  if constexpr (kOutF32) {
    const float* c = static_cast<const float*>(p.c_src) + base;
#pragma unroll
    for (int j = 0; j < kCount; j += 4) {
      float x[4] = {0.f, 0.f, 0.f, 0.f};
      if (col + j + 4 <= p.n) {
        const float4 q4 = __ldg(reinterpret_cast<const float4*>(c + j));
        x[0] = q4.x;
        x[1] = q4.y;
        x[2] = q4.z;
        x[3] = q4.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (col + j + e < p.n) x[e] = __ldg(c + j + e);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) v[j + e] = fmaf(p.beta, x[e], v[j + e]);
    }
  } else {
    const __nv_bfloat16* c = static_cast<const __nv_bfloat16*>(p.c_src) + base;
#pragma unroll
    for (int j = 0; j < kCount; j += 8) {
      uint32_t w[4] = {0u, 0u, 0u, 0u};
      if (col + j + 8 <= p.n) {
        const uint4 q4 = __ldg(reinterpret_cast<const uint4*>(c + j));
        w[0] = q4.x;
        w[1] = q4.y;
        w[2] = q4.z;
        w[3] = q4.w;
      } else {
        const uint16_t* c16 = reinterpret_cast<const uint16_t*>(c + j);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (col + j + e < p.n) w[e / 2] |= static_cast<uint32_t>(__ldg(c16 + e)) << (16 * (e & 1));
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[j + 2 * e] = fmaf(p.beta, __uint_as_float(w[e] << 16), v[j + 2 * e]);
        v[j + 2 * e + 1] = fmaf(p.beta, __uint_as_float(w[e] & 0xFFFF0000u), v[j + 2 * e + 1]);
      }
    }
  }
}

struct WorkItem {
  int tile;
  int kb0, kb1;  // k-block range [kb0, kb1)
  int part;      // -1 for a whole tile, else 1: a partial piece of a stream-K tile
  int half;      // -1 for the full tile width, else which half (narrow tail)
};

// First stream-K iteration of cluster c (0 <= c <= num_clusters): c / P of
// the region, moved to the nearest tile edge when it lies within a few
// k-blocks of one (a sliver of a tile costs a whole partial-tile write);
// computed on the host (sk_begin_host), non-decreasing in c.
__device__ __forceinline__ int sk_begin(const Params& p, int c) { return p.sk_bounds[c]; }

// Work item `idx` of cluster c: its data-parallel tiles first, then the
// pieces of its stream-K range in tile order.
// kStreamK = false compiles the stream-K part out (kernels never given a
// stream-K region).
template <bool kStreamK>
__device__ __forceinline__ bool next_item(const Params& p, int c, int idx, WorkItem& it) {
  const int n_dp = c < p.dp_tiles ? (p.dp_tiles - 1 - c) / p.num_clusters + 1 : 0;
  it.half = -1;
  if (idx < n_dp) {
    it.tile = c + idx * p.num_clusters;
    it.kb0 = 0;
    it.kb1 = p.k_blocks;
    it.part = -1;
    return true;
  }
  if (kStreamK && p.narrow_tiles > 0) {
    if (idx != n_dp || c >= 2 * p.narrow_tiles) return false;
    it.tile = p.dp_tiles + c / 2;
    it.half = c & 1;
    it.kb0 = 0;
    it.kb1 = p.k_blocks;
    it.part = -1;
    return true;
  }
  if (!kStreamK || p.sk_tiles == 0) return false;
  const int b0 = sk_begin(p, c), b1 = sk_begin(p, c + 1);
  if (b0 >= b1) return false;
  const int t = b0 / p.k_blocks + (idx - n_dp);
  const int t0 = t * p.k_blocks;
  if (t0 >= b1) return false;
  it.tile = p.dp_tiles + t;
  it.kb0 = (b0 > t0 ? b0 : t0) - t0;
  it.kb1 = (b1 - t0 < p.k_blocks ? b1 - t0 : p.k_blocks);
  it.part = (it.kb0 == 0 && it.kb1 == p.k_blocks) ? -1 : 1;
  return true;
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

constexpr int kBK = 64;  // K elements per stage: one 128-byte swizzle row of BF16
// How long a stream-K tile's first piece waits for the other pieces before
// falling back to publishing its own partial (they are normally done).
constexpr uint64_t kSkFixupWaitNs = 50000;

template <int kCG, int kBN, bool kOutF32>
struct Cfg {
  static constexpr int BM = 128;              // accumulator rows held by one CTA
  static constexpr int TILE_M = BM * kCG;     // rows of one cluster tile
  // One MMA instruction covers at most N = 256 columns; a 512-wide tile is
  // two N = 256 MMAs per K step that share the A operand.
  static constexpr int MMA_N = kBN > 256 ? 256 : kBN;
  static constexpr int N_SUB = kBN / MMA_N;
  static constexpr int B_BOX_ROWS = MMA_N / kCG;  // B rows of one CTA for one MMA (one TMA box)
  static constexpr int B_SUB_BYTES = B_BOX_ROWS * kBK * 2;
  static constexpr int A_BYTES = BM * kBK * 2;
  static constexpr int B_BYTES = N_SUB * B_SUB_BYTES;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_COLS = kOutF32 ? 32 : 64;  // C columns per 128-byte store row
  static constexpr int EPI_BOX_BYTES = 32 * 128;      // 32 rows x 128 bytes
  // A 512-wide accumulator is drained by eight epilogue warps (two per TMEM
  // lane quarter, each owning half the columns) so the single accumulator
  // buffer goes back to the MMA sooner; narrower tiles use four.
  static constexpr int EPI_WARPS = kBN > 256 ? 8 : 4;
  static constexpr int EPI_COL_SPLIT = EPI_WARPS / 4;
  static constexpr int WARP_COLS = kBN / EPI_COL_SPLIT;
  static constexpr int EPI_BUFS = EPI_WARPS == 8 ? 1 : 2;  // staging boxes per warp
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_BUFS * EPI_BOX_BYTES;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  // Two accumulator buffers (epilogue of tile i overlaps the MMAs of tile
  // i+1) when they fit in the 512 TMEM columns, else one.
  static constexpr int ACC_BUFS = 2 * kBN <= 512 ? 2 : 1;
  static constexpr int TMEM_COLS = ACC_BUFS * kBN;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM_LIMIT = 232448;  // sm_100 opt-in maximum per block
  static constexpr int STAGES_FIT = (SMEM_LIMIT - 1024 - BAR_BYTES - EPI_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
  static_assert(STAGES >= 2, "ring too shallow");
  static_assert((2 * STAGES + 15) * 8 <= BAR_BYTES, "barrier area");
  static_assert(SMEM_BYTES <= SMEM_LIMIT, "shared memory budget");
  static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation size");
  static_assert(kBN % EPI_COLS == 0, "epilogue chunking");
  static_assert(B_BYTES % 1024 == 0 && A_BYTES % 1024 == 0, "swizzle atoms need 1 KiB alignment");
  // MMA shape legality for kind::f16: M=128 needs N%16==0, 16<=N<=256;
  // M=256 (cta_group::2) the same.
  static_assert(N_SUB == 1 || N_SUB == 2, "the MMA loop issues one or two N = 256 halves per K step");
  static_assert(MMA_N % 16 == 0 && MMA_N >= 16 && MMA_N <= 256 && kBN % MMA_N == 0, "UMMA N");
};

__device__ __forceinline__ void tile_coords(const Params& p, int t, int& l, int& m_blk, int& n_blk) {
  const int per_batch = p.tiles_m * p.tiles_n;
  l = t / per_batch;
  const int r = t - l * per_batch;
  const int group_size = p.group_m * p.tiles_n;
  const int g = r / group_size;
  const int first_m = g * p.group_m;
  const int gm = min(p.group_m, p.tiles_m - first_m);
  const int local = r - g * group_size;
  m_blk = first_m + local % gm;
  n_blk = local / gm;
}

template <int kCG, int kBN, bool kOutF32>
__global__ void __launch_bounds__(Cfg<kCG, kBN, kOutF32>::THREADS, 1)
    bb_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ CUtensorMap tm_b_half,
                   const __grid_constant__ Params p) {
  using C = Cfg<kCG, kBN, kOutF32>;
  constexpr int STAGES = C::STAGES;

  // Launch contract, checked before any barrier, TMEM or cluster operation.
  const uint32_t rank = (kCG == 2) ? cluster_ctarank() : 0u;
  if (blockDim.x != C::THREADS || (kCG == 2 && cluster_nctarank() != 2) || (gridDim.x % kCG) != 0) {
    if (threadIdx.x == 0 && p.status) atomicCAS(p.status, 0, kDevBadLaunch);
    return;
  }

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + STAGES * C::A_BYTES;
  uint8_t* smem_epi = smem + STAGES * C::STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_epi + C::EPI_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tmem_full = bars + 2 * STAGES;
  uint64_t* tmem_empty = bars + 2 * STAGES + 2;
  uint64_t* mma_done = bars + 2 * STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
  volatile int* epi_flag = reinterpret_cast<volatile int*>(bars + 2 * STAGES + 6);
  uint64_t* fix_bar = bars + 2 * STAGES + 7;  // eight: two staging buffers per epilogue warp

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const bool mma_cta = (kCG == 1) || (rank == 0);

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
    prefetch_tmap(&tm_c);
    if (p.narrow_tiles > 0) prefetch_tmap(&tm_b_half);
  }
  if (warp == 1 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tmem_full[a]), 1);
      mbar_init(smem_u32(&tmem_empty[a]), C::EPI_WARPS * kCG);
    }
    mbar_init(smem_u32(mma_done), 1);
    for (int i = 0; i < 8; ++i) mbar_init(smem_u32(&fix_bar[i]), 1);
    fence_mbarrier_init_cluster();
  }
  if (warp == 1) {
    tmem_alloc<kCG>(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish<kCG>();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (kCG == 2) cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  // Programmatic dependent launch: the set-up above (barrier init, TMEM
  // allocation) overlaps the previous kernel in the stream; no global memory
  // is touched before that kernel has completed. Dependents may launch now;
  // their CTAs only become resident as this kernel's CTAs exit.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  const int cluster_idx = blockIdx.x / kCG;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The whole warp runs the loop and waits; one elected lane issues (a lone
    // lane looping inside a divergent branch issues markedly slower).
    bool ok = true;
    int stage = 0;
    uint32_t phase = 0;
    const uint32_t full_target_rank = 0;
    WorkItem it;
    for (int idx = 0; ok && next_item<C::ACC_BUFS == 2>(p, cluster_idx, idx, it); ++idx) {
      int l, m_blk, n_blk;
      tile_coords(p, it.tile, l, m_blk, n_blk);
      const int a_row = m_blk * C::TILE_M + static_cast<int>(rank) * C::BM;
      // A half-width item loads this CTA's B_BOX_ROWS / 2 rows of its half.
      const bool narrow = C::N_SUB == 1 && it.half >= 0;
      const int b_row = narrow ? n_blk * kBN + it.half * (kBN / 2) + static_cast<int>(rank) * (C::B_BOX_ROWS / 2)
                               : n_blk * kBN + static_cast<int>(rank) * C::B_BOX_ROWS;
      const uint32_t stage_tx = (narrow ? C::A_BYTES + C::B_BYTES / 2 : C::STAGE_BYTES) * kCG;
      for (int kb = it.kb0; kb < it.kb1; ++kb) {
        const bool got = (p.spin & 1) ? bb_wait_warp<kCG == 2, false>(smem_u32(&empty[stage]), phase ^ 1u, p.status, kDevTimeoutProducer)
                                       : bb_wait_warp<kCG == 2>(smem_u32(&empty[stage]), phase ^ 1u, p.status, kDevTimeoutProducer);
        if (!got) {
          ok = false;
          break;
        }
        if (elect_one()) {
          const uint32_t fb = smem_u32(&full[stage]);
          if (mma_cta) mbar_arrive_expect_tx(fb, stage_tx);
          const uint32_t da = smem_u32(smem_a + stage * C::A_BYTES);
          const uint32_t db = smem_u32(smem_b + stage * C::B_BYTES);
          if constexpr (kCG == 2) {
            const uint32_t fbc = mapa_shared(fb, full_target_rank);
            tma_load_3d_pair(da, &tm_a, fbc, kb * kBK, a_row, l);
            if (narrow) {
              tma_load_3d_pair(db, &tm_b_half, fbc, kb * kBK, b_row, l);
            } else {
#pragma unroll
              for (int h = 0; h < C::N_SUB; ++h)
                tma_load_3d_pair(db + h * C::B_SUB_BYTES, &tm_b, fbc, kb * kBK, b_row + h * C::MMA_N, l);
            }
          } else {
            tma_load_3d(da, &tm_a, fb, kb * kBK, a_row, l);
            if (narrow) {
              tma_load_3d(db, &tm_b_half, fb, kb * kBK, b_row, l);
            } else {
#pragma unroll
              for (int h = 0; h < C::N_SUB; ++h)
                tma_load_3d(db + h * C::B_SUB_BYTES, &tm_b, fb, kb * kBK, b_row + h * C::MMA_N, l);
            }
          }
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (ok) {
      // Tail: wait until the MMA has released every stage, so no commit
      // arrival can still be in flight towards this CTA when it exits.
      for (int i = 0; i < STAGES; ++i) {
        if (!bb_wait_warp<kCG == 2>(smem_u32(&empty[stage]), phase ^ 1u, p.status, kDevTimeoutProducer)) break;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    } else if (lane == 0) {
      // Aborted: let any TMA copy already issued land before teardown.
      bounded_sleep_ns(2000000);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // Whole warp loops and waits; the elected lane (always the lowest lane of
    // the converged warp, so its commits track all of its MMAs) issues.
    if (mma_cta) {
      constexpr uint32_t idesc_full = make_idesc_bf16_f32(C::TILE_M, C::MMA_N);
      constexpr uint32_t idesc_half = make_idesc_bf16_f32(C::TILE_M, C::MMA_N / 2);
      const uint64_t a_desc0 = sw128_kmajor_desc(smem_u32(smem_a));
      const uint64_t b_desc0 = sw128_kmajor_desc(smem_u32(smem_b));
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_iter = 0;
      WorkItem it;
      for (int idx = 0; ok && next_item<C::ACC_BUFS == 2>(p, cluster_idx, idx, it); ++idx, ++acc_iter) {
        const uint32_t acc = acc_iter % C::ACC_BUFS;
        const uint32_t acc_phase = (acc_iter / C::ACC_BUFS) & 1u;
        if (!bb_wait_warp<kCG == 2>(smem_u32(&tmem_empty[acc]), acc_phase ^ 1u, p.status, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kBN;
        const uint32_t idesc = (C::N_SUB == 1 && it.half >= 0) ? idesc_half : idesc_full;
        for (int kb = it.kb0; kb < it.kb1; ++kb) {
          const bool got = (p.spin & 2) ? bb_wait_warp<kCG == 2, false>(smem_u32(&full[stage]), phase, p.status, kDevTimeoutMma)
                                         : bb_wait_warp<kCG == 2>(smem_u32(&full[stage]), phase, p.status, kDevTimeoutMma);
          if (!got) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (elect_one()) {
            // Descriptors advance by adds in 16-byte units (the start-address
            // field's unit): 32 bytes (2 units) per K16 step.
            const uint64_t a_desc = a_desc0 + static_cast<uint64_t>(stage) * (C::A_BYTES >> 4);
            const uint64_t b_desc = b_desc0 + static_cast<uint64_t>(stage) * (C::B_BYTES >> 4);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              const uint32_t acc_in = (kb != it.kb0 || kk != 0) ? 1u : 0u;
              if constexpr (C::N_SUB == 2) {
                // Both N = 256 halves use this K step's A: read it once.
                umma_f16_keep_a<kCG, true>(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc, acc_in);
                umma_f16_keep_a<kCG, false>(d_tmem + C::MMA_N, a_desc + 2 * kk,
                                            b_desc + (C::B_SUB_BYTES >> 4) + 2 * kk, idesc, acc_in);
              } else {
                umma_f16<kCG>(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc, acc_in);
              }
            }
            const uint32_t eb = smem_u32(&empty[stage]);
            umma_commit<kCG>(eb);
            if constexpr (kCG == 2) umma_commit<kCG>(mapa_shared(eb, 1));
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (elect_one()) {
          const uint32_t fb = smem_u32(&tmem_full[acc]);
          umma_commit<kCG>(fb);
          if constexpr (kCG == 2) umma_commit<kCG>(mapa_shared(fb, 1));
        }
        __syncwarp();
      }
      // Drain: every MMA issued so far must finish before TMEM is freed.
      if (elect_one()) umma_commit<kCG>(smem_u32(mma_done));
      __syncwarp();
      bb_wait_warp(smem_u32(mma_done), 0, p.status, kDevTimeoutMma, /*honor_abort=*/false);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int ep_tid = threadIdx.x - 64;  // index within the epilogue warps
    constexpr int kEpiThreads = C::EPI_WARPS * 32;
    const int wc0 = ((warp - 2) / 4) * C::WARP_COLS;  // this warp's columns: [wc0, wc0 + WARP_COLS)
    uint8_t* ebuf = smem_epi + (warp - 2) * C::EPI_BUFS * C::EPI_BOX_BYTES;
    const uint32_t ebuf_u32 = smem_u32(ebuf);
    uint32_t acc_iter = 0;
    int chunk_seq = 0;

    // Stages one 32-row x 128-byte chunk in swizzled shared memory and
    // stores it to C with TMA.
    auto store_chunk = [&](const uint32_t (&packed)[32], int row0, int col0, int l) {
      const uint32_t buf = ebuf_u32 + (chunk_seq % C::EPI_BUFS) * C::EPI_BOX_BYTES;
      ++chunk_seq;
      if (lane == 0) bulk_wait_group_read<C::EPI_BUFS - 1>();
      __syncwarp();
      const uint32_t row_addr = buf + lane * 128;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        st_shared_v4(row_addr + ((j ^ (lane & 7)) << 4), packed[4 * j], packed[4 * j + 1], packed[4 * j + 2],
                     packed[4 * j + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && row0 < p.m && col0 < p.n) {
        // Boxes that start inside C are clipped by TMA at the far edges;
        // boxes wholly outside C (ragged last tile) are skipped.
        tma_store_3d(&tm_c, buf, col0, row0, l);
      }
      if (lane == 0) bulk_commit_group();
    };
    auto pack_chunk = [&](const float* v, uint32_t (&packed)[32]) {
      if constexpr (kOutF32) {
#pragma unroll
        for (int j = 0; j < 32; ++j) packed[j] = __float_as_uint(v[j]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) packed[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
      }
    };
    auto release_acc = [&](uint32_t acc) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        const uint32_t eb = smem_u32(&tmem_empty[acc]);
        if constexpr (kCG == 2) {
          // Relaxed: the TMEM reads this publishes completed at
          // tcgen05.wait::ld; a cluster-scope release arrive is far slower.
          mbar_arrive_cluster_relaxed(mapa_shared(eb, 0));
        } else {
          mbar_arrive(eb);
        }
      }
    };

    WorkItem it;
    for (int idx = 0; next_item<C::ACC_BUFS == 2>(p, cluster_idx, idx, it); ++idx, ++acc_iter) {
      int l, m_blk, n_blk;
      tile_coords(p, it.tile, l, m_blk, n_blk);
      const uint32_t acc = acc_iter % C::ACC_BUFS;
      const uint32_t acc_phase = (acc_iter / C::ACC_BUFS) & 1u;
      if (!bb_wait<kCG == 2>(smem_u32(&tmem_full[acc]), acc_phase, p.status, kDevTimeoutEpilogue)) break;
      tc_fence_after();
      const int row0 = m_blk * C::TILE_M + static_cast<int>(rank) * C::BM + q * 32;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kBN;
      constexpr int ncols = kOutF32 ? 32 : 64;  // accumulator columns behind one 128-byte store row

      if (it.part < 0) {
        if constexpr (!kOutF32 && C::EPI_COL_SPLIT == 2) {
          // ---- whole 512-wide tile, BF16: the warp's 256 columns are
          // converted into registers (128 packed words), the accumulator is
          // released, and only then staged and stored.
          uint32_t pk[C::WARP_COLS / 64][32];
#pragma unroll
          for (int h = 0; h < C::WARP_COLS / 32; ++h) {
            uint32_t r0[32];
            tmem_ld_32x32b_x32(t_row + wc0 + h * 32, r0);
            tmem_ld_wait();
            if (p.epi_mode != 0) {
              float v[32];
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) v[jj] = __uint_as_float(r0[jj]);
              apply_epilogue<kOutF32, 32>(p, v, row0 + lane, n_blk * kBN + wc0 + h * 32, l);
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) r0[jj] = __float_as_uint(v[jj]);
            }
#pragma unroll
            for (int jj = 0; jj < 16; ++jj)
              pk[h / 2][(h & 1) * 16 + jj] = pack_bf16x2(__uint_as_float(r0[2 * jj]), __uint_as_float(r0[2 * jj + 1]));
          }
          release_acc(acc);
#pragma unroll
          for (int cc = 0; cc < C::WARP_COLS / 64; ++cc) store_chunk(pk[cc], row0, n_blk * kBN + wc0 + cc * 64, l);
        } else {
          // ---- whole tile: TMEM -> registers -> C, one store row at a time
          // (a half-width item: the first half of the accumulator columns,
          // stored at its half's columns of C)
          constexpr int kWarpChunks = C::WARP_COLS / C::EPI_COLS;
          const int n_chunks = it.half >= 0 ? kWarpChunks / 2 : kWarpChunks;
          const int c_off = it.half >= 0 ? it.half * (kBN / 2) : 0;
#pragma unroll 1
          for (int c = 0; c < n_chunks; ++c) {
            const int col = wc0 + c * ncols;
            float v[64];
            uint32_t r0[32];
            tmem_ld_32x32b_x32(t_row + col, r0);
            if constexpr (!kOutF32) {
              uint32_t r1[32];
              tmem_ld_32x32b_x32(t_row + col + 32, r1);
              tmem_ld_wait();
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) v[32 + jj] = __uint_as_float(r1[jj]);
            } else {
              tmem_ld_wait();
            }
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) v[jj] = __uint_as_float(r0[jj]);
            if (c == n_chunks - 1) release_acc(acc);  // accumulator now lives in registers
            apply_epilogue<kOutF32, ncols>(p, *reinterpret_cast<float(*)[ncols]>(v), row0 + lane,
                                           n_blk * kBN + c_off + col, l);
            uint32_t packed[32];
            pack_chunk(v, packed);
            store_chunk(packed, row0, n_blk * kBN + c_off + col, l);
          }
        }
      } else if constexpr (C::ACC_BUFS == 2) {
        // ---- a partial piece of a stream-K tile (tiles up to 256 wide; the
        // host never gives the 512-wide tile a stream-K region).
        //
        // Protocol, per tile and CTA rank (no piece ever waits unboundedly):
        // * every piece but the tile's first (k-blocks from 0) writes its FP32
        //   accumulator to its workspace slot, then adds its k-block count to
        //   the tile's counter (release);
        // * the first piece is normally processed last (it is the end of its
        //   cluster's range) and fixes the tile up: it waits, bounded, for the
        //   counter to hold every other piece's k-blocks, then sums the pieces
        //   in k order, its own from TMEM, and stores C;
        // * if that wait runs out (other pieces not resident yet, e.g. beside
        //   another kernel), the first piece writes and adds like the others,
        //   and whichever piece completes the counter does the fix-up.
        // The sum order is fixed (k order), so C does not depend on timing.
        // A slot is laid out [lane quarter][column quad][lane][4] floats: each
        // epilogue warp's 32 rows are contiguous (one warp access covers 512
        // contiguous bytes).
        const int t_local = it.tile - p.dp_tiles;
        const int mine = it.kb1 - it.kb0;
        int* ctr = p.counters + t_local * kCG + static_cast<int>(rank);
        constexpr int64_t kSlotFloats = static_cast<int64_t>(C::BM) * kBN;
        constexpr int kQuads = kBN / 4;
        // This warp's part of cluster c_owner's slot for this tile (two slots
        // per cluster: a range holds at most two partial pieces, one in its
        // first tile and one in its last).
        auto slot_warp = [&](int c_owner) {
          const bool first = sk_begin(p, c_owner) / p.k_blocks == t_local;
          const int64_t s = (2 * static_cast<int64_t>(c_owner) + (first ? 0 : 1)) * kCG + rank;
          return reinterpret_cast<float4*>(p.partials + s * kSlotFloats) + q * (kQuads * 32);
        };
        // 128 columns per TMEM wait (the load latency, not the stores, sets
        // the pace of this loop).
        auto write_partial = [&]() {
          float4* dst = slot_warp(cluster_idx) + lane;
#pragma unroll 1
          for (int c = 0; c < kBN / 128; ++c) {
            uint32_t r[4][32];
#pragma unroll
            for (int u = 0; u < 4; ++u) tmem_ld_32x32b_x32(t_row + c * 128 + u * 32, r[u]);
            tmem_ld_wait();
#pragma unroll
            for (int u = 0; u < 4; ++u) {
#pragma unroll
              for (int jj = 0; jj < 8; ++jj) {
                __stcg(dst + (c * 32 + u * 8 + jj) * 32,
                       make_float4(__uint_as_float(r[u][4 * jj]), __uint_as_float(r[u][4 * jj + 1]),
                                   __uint_as_float(r[u][4 * jj + 2]), __uint_as_float(r[u][4 * jj + 3])));
              }
            }
          }
        };
        // Publishes this piece's partial; true when it completed the tile.
        auto publish = [&]() {
          __threadfence();
          named_bar_sync(1, kEpiThreads);
          if (ep_tid == 0) {
            const int old = atomicAdd(ctr, mine);
            __threadfence();
            epi_flag[0] = (old + mine == p.k_blocks) ? 1 : 0;
          }
          named_bar_sync(1, kEpiThreads);
          return epi_flag[0] != 0;
        };
        bool fix;
        if (it.kb0 == 0) {
          if (ep_tid == 0) {
            const int target = p.k_blocks - mine;
            const uint64_t t0 = globaltimer_ns();
            int v;
            while (true) {
              asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
              if (v >= target || globaltimer_ns() - t0 > kSkFixupWaitNs) break;
              __nanosleep(64);
            }
            epi_flag[0] = v >= target ? 1 : 0;
          }
          named_bar_sync(1, kEpiThreads);
          fix = epi_flag[0] != 0;
          if (!fix) {
            write_partial();
            fix = publish();
          }
        } else {
          write_partial();
          fix = publish();
        }
        if (fix) {
          // The tile's pieces belong to consecutive clusters c_first..c_last
          // (clusters with an empty range in between own none).
          const int tile0 = t_local * p.k_blocks;
          int c_first = cluster_idx, c_last = cluster_idx;
          while (c_first > 0 && sk_begin(p, c_first) > tile0) --c_first;
          while (c_last + 1 < p.num_clusters && sk_begin(p, c_last + 1) < tile0 + p.k_blocks) ++c_last;
          auto foreign = [&](int co) { return co != cluster_idx && sk_begin(p, co) < sk_begin(p, co + 1); };
          // Up to kMaxStaged other pieces, in k order, and this piece's place.
          int nf = 0, own_pos = 0, f0 = 0, f1 = 0, f2 = 0;
          for (int co = c_first; co <= c_last; ++co) {
            if (co == cluster_idx) own_pos = nf;
            if (!foreign(co)) continue;
            if (nf == 0) f0 = co;
            else if (nf == 1) f1 = co;
            else if (nf == 2) f2 = co;
            ++nf;
          }
          // Staged fix-up: on the cluster's final work item the operand ring
          // is idle (every MMA that read it completed before this tile's
          // accumulator was signalled), so each epilogue warp brings its 32
          // rows of the other pieces' partials into its own quarter of the
          // ring by bulk copies, 64 columns at a time, double buffered: many
          // bytes in flight and no CTA-wide barrier. Otherwise the partials
          // are read with plain loads.
          constexpr int kGroupCols = 64;
          constexpr int kGroups = kBN / kGroupCols;
          constexpr uint32_t kWarpGroupBytes = 32 * kGroupCols * 4;
          constexpr int kWarpRing = STAGES * C::STAGE_BYTES / 4;
          constexpr int kMaxStaged = kWarpRing / (2 * static_cast<int>(kWarpGroupBytes));
          static_assert(kMaxStaged >= 1 && kMaxStaged <= 3, "staging depth");
          WorkItem nx;
          const bool staged = nf <= kMaxStaged && !next_item<true>(p, cluster_idx, idx + 1, nx);
          if (staged) {
            const int ew = warp - 2;  // epilogue warp index 0..3
            uint8_t* wring = smem + ew * kWarpRing;
            auto foreign_at = [&](int i) { return i == 0 ? f0 : (i == 1 ? f1 : f2); };
            auto issue_group = [&](int g) {
              const uint32_t bar = smem_u32(&fix_bar[2 * ew + (g & 1)]);
              mbar_arrive_expect_tx(bar, nf * kWarpGroupBytes);
              for (int i = 0; i < nf; ++i) {
                const float4* src = slot_warp(foreign_at(i)) + g * (kGroupCols / 4) * 32;
                bulk_load_g2s(smem_u32(wring + ((g & 1) * kMaxStaged + i) * kWarpGroupBytes), src, kWarpGroupBytes,
                              bar);
              }
            };
            if (lane == 0) {
              fence_proxy_async_global();
              issue_group(0);
              if (kGroups > 1) issue_group(1);
            }
            __syncwarp();
#pragma unroll 1
            for (int g = 0; g < kGroups; ++g) {
              if (!bb_wait(smem_u32(&fix_bar[2 * ew + (g & 1)]), (g >> 1) & 1, p.status, kDevTimeoutEpilogue)) break;
              const uint32_t buf = smem_u32(wring + (g & 1) * kMaxStaged * kWarpGroupBytes);
#pragma unroll 1
              // This piece's 64 columns from TMEM with one wait, then every
              // piece's values added in k order.
              uint32_t o[2][32];
              tmem_ld_32x32b_x32(t_row + g * kGroupCols, o[0]);
              tmem_ld_32x32b_x32(t_row + g * kGroupCols + 32, o[1]);
              tmem_ld_wait();
#pragma unroll
              for (int c = 0; c < kGroupCols / ncols; ++c) {
                uint32_t packed[32];
#pragma unroll
                for (int h = 0; h < ncols / 32; ++h) {
                  const int hh = c * (ncols / 32) + h;  // 32-column half of the group
                  float v[32];
                  for (int pos = 0; pos <= nf; ++pos) {
                    if (pos == own_pos) {
#pragma unroll
                      for (int jj = 0; jj < 32; ++jj)
                        v[jj] = pos == 0 ? __uint_as_float(o[hh][jj]) : v[jj] + __uint_as_float(o[hh][jj]);
                      continue;
                    }
                    const int i = pos < own_pos ? pos : pos - 1;
                    const uint32_t src = buf + i * kWarpGroupBytes + ((hh * 8 * 32) + lane) * 16;
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                      const float4 x = ld_shared_v4f(src + jj * 32 * 16);
                      if (pos == 0) {
                        v[4 * jj] = x.x;
                        v[4 * jj + 1] = x.y;
                        v[4 * jj + 2] = x.z;
                        v[4 * jj + 3] = x.w;
                      } else {
                        v[4 * jj] += x.x;
                        v[4 * jj + 1] += x.y;
                        v[4 * jj + 2] += x.z;
                        v[4 * jj + 3] += x.w;
                      }
                    }
                  }
                  const int col = g * kGroupCols + 32 * hh;
                  apply_epilogue<kOutF32, 32>(p, v, row0 + lane, n_blk * kBN + col, l);
                  if constexpr (kOutF32) {
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj) packed[jj] = __float_as_uint(v[jj]);
                  } else {
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) packed[16 * h + jj] = pack_bf16x2(v[2 * jj], v[2 * jj + 1]);
                  }
                }
                store_chunk(packed, row0, n_blk * kBN + g * kGroupCols + c * ncols, l);
              }
              // This warp has read buffer g & 1: refill it.
              __syncwarp();
              if (lane == 0 && g + 2 < kGroups) issue_group(g + 2);
              __syncwarp();
            }
          } else {
#pragma unroll 1
            for (int c = wc0 / ncols; c < (wc0 + C::WARP_COLS) / ncols; ++c) {
              // One 128-byte store row, summed 32 columns at a time (fewer live
              // registers than the whole row).
              uint32_t packed[32];
#pragma unroll
              for (int h = 0; h < ncols / 32; ++h) {
                const int col = c * ncols + 32 * h;
                float v[32];
                bool first_term = true;
                for (int co = c_first; co <= c_last; ++co) {
                  if (co == cluster_idx) {
                    // Own piece, straight from TMEM at its place in the order.
                    uint32_t r0[32];
                    tmem_ld_32x32b_x32(t_row + col, r0);
                    tmem_ld_wait();
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj)
                      v[jj] = first_term ? __uint_as_float(r0[jj]) : v[jj] + __uint_as_float(r0[jj]);
                    first_term = false;
                    continue;
                  }
                  if (!foreign(co)) continue;
                  const float4* src = slot_warp(co) + (col / 4) * 32 + lane;
                  float4 x[8];
#pragma unroll
                  for (int jj = 0; jj < 8; ++jj) x[jj] = __ldcg(src + jj * 32);
#pragma unroll
                  for (int jj = 0; jj < 8; ++jj) {
                    v[4 * jj] = first_term ? x[jj].x : v[4 * jj] + x[jj].x;
                    v[4 * jj + 1] = first_term ? x[jj].y : v[4 * jj + 1] + x[jj].y;
                    v[4 * jj + 2] = first_term ? x[jj].z : v[4 * jj + 2] + x[jj].z;
                    v[4 * jj + 3] = first_term ? x[jj].w : v[4 * jj + 3] + x[jj].w;
                  }
                  first_term = false;
                }
                apply_epilogue<kOutF32, 32>(p, v, row0 + lane, n_blk * kBN + col, l);
                if constexpr (kOutF32) {
#pragma unroll
                  for (int jj = 0; jj < 32; ++jj) packed[jj] = __float_as_uint(v[jj]);
                } else {
#pragma unroll
                  for (int jj = 0; jj < 16; ++jj) packed[16 * h + jj] = pack_bf16x2(v[2 * jj], v[2 * jj + 1]);
                }
              }
              store_chunk(packed, row0, n_blk * kBN + c * C::EPI_COLS, l);
            }
          }
          // Every other piece has added its k-blocks: reset for the next launch.
          if (ep_tid == 0) atomicExch(ctr, 0);
        }
        release_acc(acc);
        // epi_flag is rewritten by the next piece: nobody may still read it.
        named_bar_sync(1, kEpiThreads);
      }
    }
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if constexpr (kCG == 2) cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc<kCG>(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side

// Stream-K planning. The device's sk_begin restated on the host, and the
// modelled time of the slowest cluster (k-block units): its k-blocks plus
// `ovh` per partial piece (a partial-tile write, or the fix-up reads).
constexpr int kDefaultSkSnap = 4;
// Measured cost of a partial piece, in k-blocks of a 256 x 256 tile (about
// 0.33 us each): its partial-tile write, or the fix-up's reads and store,
// which run at the aggregate L2 write/read rate when every cluster does it
// at once (about 4 us per piece at 4096^3 and on sub-wave problems).
constexpr double kDefaultSkOverhead = 17.0;
// Main-loop efficiency of the 256 x 128 pair tile relative to the tensor
// peak (the 256 x 256 tile: 0.907, the 256 x 512 tile: 0.96), measured at
// 4096^3 (1220 against 1460 TFLOP/s for the 256 x 256 tile).
constexpr double kEff128 = 0.66;
// The 256 x 512 tile's, including its exposed epilogue (single accumulator
// buffer): 2048 x 4096 x 4096 ran at 1246 TFLOP/s against 1292 for two
// waves of 256 x 256 tiles.
constexpr double kEff512 = 0.93;

static int64_t sk_begin_host(int c, int P, int sk_tiles, int kb, int snap) {
  const int64_t total = static_cast<int64_t>(sk_tiles) * kb;
  if (c <= 0) return 0;
  if (c >= P) return total;
  int64_t x = (static_cast<int64_t>(c) * total) / P;
  const int64_t off = x % kb;
  if (off < snap) x -= off;
  else if (kb - off < snap) x += kb - off;
  return x;
}

static double sk_region_cost(int P, int sk_tiles, int kb, int snap, double ovh) {
  double worst = 0.0;
  for (int c = 0; c < P; ++c) {
    const int64_t b0 = sk_begin_host(c, P, sk_tiles, kb, snap), b1 = sk_begin_host(c + 1, P, sk_tiles, kb, snap);
    if (b0 >= b1) continue;
    double cost = static_cast<double>(b1 - b0);
    for (int64_t t = b0 / kb; t * kb < b1; ++t) {
      const int64_t t0 = t * kb;
      if (b0 > t0 || b1 < t0 + kb) cost += ovh;
    }
    worst = cost > worst ? cost : worst;
  }
  return worst;
}

struct StreamKChoice {
  int sk_tiles;  // 0: whole tiles only
  double cost;
};

// Region options: none; the rem tiles of the partial last wave; those plus
// one full wave (a region of a few k-blocks per cluster is mostly fix-up).
static StreamKChoice choose_stream_k(int T, int P, int kb, int snap, double ovh, bool force) {
  const int full = T / P, rem = T % P;
  StreamKChoice best{0, static_cast<double>(full + (rem ? 1 : 0)) * kb};
  if (rem == 0) return best;
  StreamKChoice sk{rem, static_cast<double>(full) * kb + sk_region_cost(P, rem, kb, snap, ovh)};
  if (full >= 1) {
    const double c2 = static_cast<double>(full - 1) * kb + sk_region_cost(P, rem + P, kb, snap, ovh);
    if (c2 < sk.cost) sk = {rem + P, c2};
  }
  if (force || sk.cost < 0.97 * best.cost) best = sk;
  return best;
}

// Half-width tile time relative to a full 256-wide tile (same K): half the
// MMA work at the 256 x 128 tile's lower main-loop efficiency.
constexpr double kNarrowRate = 0.5 * 0.907 / kEff128;

struct TailPlan {
  int narrow_tiles;  // > 0: narrow tail of this many tiles
  int sk_tiles;      // > 0: stream-K region of this many tiles
  double cost;       // modelled time, k-blocks of one full tile
};

// The cheapest way to run the last, partial wave of T tiles of kb k-blocks
// on P clusters: whole tiles; a narrow tail (allowed for 256-wide tiles when
// the partial wave fits P as half tiles); or a stream-K region. Modes: -1
// model, 0 off, 1 forced (when legal). A plan must model at least 3 %
// faster than whole tiles unless forced.
static TailPlan plan_tail(int T, int P, int kb, bool allow_narrow, int snap, double ovh, int narrow_mode,
                          int sk_mode) {
  const int full = T / P, rem = T % P;
  TailPlan best{0, 0, static_cast<double>(full + (rem ? 1 : 0)) * kb};
  if (rem == 0) return best;
  const double whole = best.cost;
  if (allow_narrow && narrow_mode != 0 && 2 * rem <= P) {
    const TailPlan nt{rem, 0, static_cast<double>(full) * kb + kb * kNarrowRate};
    if (narrow_mode == 1 || nt.cost < 0.97 * whole) best = nt;
    if (narrow_mode == 1) return best;
  }
  if (sk_mode != 0) {
    const StreamKChoice sk = choose_stream_k(T, P, kb, snap, ovh, sk_mode == 1);
    if (sk.sk_tiles > 0 && (sk_mode == 1 || sk.cost < best.cost)) best = {0, sk.sk_tiles, sk.cost};
  }
  return best;
}

static int env_mode(const char* name) {
  const char* e = std::getenv(name);
  return e ? std::atoi(e) : -1;
}

struct KernelChoice {
  int cg;
  int bn;
  bool persistent;
  int group_m;
  bool stream_k;
};

static KernelChoice choose(int variant, int64_t m, int64_t n, int64_t k, int sm_count) {
  switch (variant) {
    case BB_VARIANT_NONPERSISTENT_1CTA: return {1, 128, false, 8, false};
    case BB_VARIANT_PERSISTENT_1CTA: return {1, 128, true, 8, false};
    case BB_VARIANT_PERSISTENT_2CTA: return {2, 128, true, 8, false};
    default: break;
  }
  // Tuned: CTA-pair tiles wherever they fill the machine.
  if (n < 256 || m < 256) return {1, 128, true, 8, true};
  // Three CTA-pair tile shapes: 256 x 256 (double-buffered TMEM
  // accumulator; a narrow tail or stream-K region for a partial last wave),
  // 256 x 128 (twice the tiles, for short problems), and 256 x 512 (two
  // N = 256 MMAs per K step sharing A: 36 % fewer operand bytes staged per
  // FLOP, but one accumulator buffer, so each tile's epilogue is exposed).
  // BB_GEMM_TILE_N=128|256|512 forces one.
  const char* tn = std::getenv("BB_GEMM_TILE_N");
  if (tn && std::atoi(tn) == 256) return {2, 256, true, 8, true};
  if (tn && std::atoi(tn) == 512) return {2, 512, true, 8, true};
  if (tn && std::atoi(tn) == 128) return {2, 128, true, 8, true};
  const int P = sm_count / 2;
  const int kb = static_cast<int>((k + kBK - 1) / kBK);
  int snap = kDefaultSkSnap > kb / 4 ? kb / 4 : kDefaultSkSnap;
  auto tiles = [&](int tn_) { return static_cast<int>(((m + 255) / 256) * ((n + tn_ - 1) / tn_)); };
  // Modelled time in k-blocks of one 256 x 256 tile at full tensor rate
  // (the 256-wide tile's stream-K region included; the 512-wide tile runs
  // whole tiles only); the per-shape efficiencies are the measured
  // main-loop tensor-pipe activity, and the 512-wide tile's single
  // accumulator exposes about two k-blocks of epilogue per tile.
  const double time256 =
      plan_tail(tiles(256), P, kb, true, snap, kDefaultSkOverhead, env_mode("BB_GEMM_NARROW"), env_mode("BB_GEMM_STREAM_K"))
          .cost /
      0.907;
  const int t512 = tiles(512);
  const double time512 = static_cast<double>((t512 + P - 1) / P) * kb * 2.0 / kEff512 * (1.0 + 2.0 / kb);
  // 256 x 128 pair tiles: half the work per tile at a lower rate (the MMA
  // streams more operand bytes per FLOP), but twice the tiles, which fills
  // the machine on short-M or short-N problems.
  const double time128 =
      plan_tail(tiles(128), P, kb, false, snap, kDefaultSkOverhead, 0, env_mode("BB_GEMM_STREAM_K")).cost * 0.5 /
      kEff128;
  // The 256 x 128 tile where it clearly wins (its efficiency varies more
  // with the shape than the model's constant), and where every 256-wide
  // tile would be a narrow-tail item anyway (its own kernel runs those
  // faster: deeper ring).
  if (tiles(256) * 2 <= P || (time128 < 0.9 * time256 && time128 < 0.9 * time512)) return {2, 128, true, 8, true};
  return time512 < time256 ? KernelChoice{2, 512, true, 8, true} : KernelChoice{2, 256, true, 8, true};
}

template <int kCG, int kBN, bool kOutF32>
static int launch(const Plan& pl) {
  using C = Cfg<kCG, kBN, kOutF32>;
  auto kern = bb_gemm_kernel<kCG, kBN, kOutF32>;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(pl.grid), 1, 1);
  cfg.blockDim = dim3(C::THREADS, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = pl.stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCG;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pl.pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  Params prm{};
  prm.m = static_cast<int32_t>(pl.m);
  prm.n = static_cast<int32_t>(pl.n);
  prm.k = static_cast<int32_t>(pl.k);
  prm.l = static_cast<int32_t>(pl.l);
  prm.tiles_m = pl.tiles_m;
  prm.tiles_n = pl.tiles_n;
  prm.num_tiles = pl.num_tiles;
  prm.k_blocks = pl.k_blocks;
  prm.group_m = pl.group_m;
  prm.num_clusters = pl.grid / kCG;
  prm.dp_tiles = pl.dp_tiles;
  prm.narrow_tiles = pl.narrow_tiles;
  prm.sk_tiles = pl.sk_tiles;
  if (pl.sk_tiles > 0) {
    for (int c = 0; c <= prm.num_clusters; ++c)
      prm.sk_bounds[c] = static_cast<int32_t>(sk_begin_host(c, prm.num_clusters, pl.sk_tiles, pl.k_blocks, pl.sk_snap));
  }
  prm.partials = pl.partials;
  prm.counters = pl.counters;
  prm.status = pl.status;
  prm.epi_mode = pl.epi_mode;
  prm.spin = pl.spin;
  prm.alpha = pl.alpha;
  prm.beta = pl.beta;
  prm.c_src = pl.c_src;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, pl.tm_a, pl.tm_b, pl.tm_c, pl.tm_b_half, prm), "cudaLaunchKernelEx(gemm)");
}

template <int kCG, int kBN, bool kOutF32>
static int prepare(Plan& pl, int sm_count) {
  using C = Cfg<kCG, kBN, kOutF32>;
  auto kern = bb_gemm_kernel<kCG, kBN, kOutF32>;
  BB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
  if (kCG == 2) {
    BB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 0));
  }
  pl.tile_m = C::TILE_M;
  pl.tile_n = kBN;
  pl.threads = C::THREADS;
  pl.stages = C::STAGES;
  pl.smem_bytes = C::SMEM_BYTES;
  pl.tmem_cols = C::TMEM_COLS;
  pl.b_rows = C::B_BOX_ROWS;
  pl.epi_cols = C::EPI_COLS;
  pl.tiles_m = static_cast<int>((pl.m + C::TILE_M - 1) / C::TILE_M);
  pl.tiles_n = static_cast<int>((pl.n + kBN - 1) / kBN);
  pl.num_tiles = pl.tiles_m * pl.tiles_n * static_cast<int>(pl.l);
  pl.k_blocks = static_cast<int>((pl.k + kBK - 1) / kBK);
  // Clusters that can be resident at once.
  int max_clusters = sm_count / kCG;
  {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(kCG * max_clusters), 1, 1);
    cfg.blockDim = dim3(C::THREADS, 1, 1);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCG;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n_clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&n_clusters, kern, &cfg) == cudaSuccess && n_clusters > 0) {
      max_clusters = n_clusters;
    } else {
      cudaGetLastError();
    }
  }
  pl.max_active_clusters = max_clusters;
  int clusters = pl.persistent ? (pl.num_tiles < max_clusters ? pl.num_tiles : max_clusters) : pl.num_tiles;
  pl.dp_tiles = pl.num_tiles;
  pl.narrow_tiles = 0;
  pl.sk_tiles = 0;
  // The last, partial wave (tuned variant, double-buffered accumulator):
  // whole tiles, a narrow tail or a stream-K region, whichever the model
  // says is fastest. BB_GEMM_NARROW / BB_GEMM_STREAM_K = 0 | 1 turn either
  // off or force it (tuning overrides). The 512-wide tile has one
  // accumulator buffer and no register room for the stream-K fix-up: whole
  // tiles only.
  if (pl.stream_k && pl.persistent && C::ACC_BUFS == 2 && pl.num_tiles % max_clusters != 0 &&
      max_clusters <= kMaxSkClusters) {
    const int P = max_clusters;
    const int kb = pl.k_blocks;
    int snap = kDefaultSkSnap;
    if (const char* e = std::getenv("BB_GEMM_SK_SNAP")) snap = std::atoi(e);
    if (snap > kb / 4) snap = kb / 4;
    if (snap < 0) snap = 0;
    double ovh = kDefaultSkOverhead;
    if (const char* e = std::getenv("BB_GEMM_SK_OVH")) ovh = std::atof(e);
    const TailPlan tp = plan_tail(pl.num_tiles, P, kb, kBN == 256 && C::N_SUB == 1, snap, ovh,
                                  env_mode("BB_GEMM_NARROW"), env_mode("BB_GEMM_STREAM_K"));
    if (tp.narrow_tiles > 0) {
      clusters = P;
      pl.dp_tiles = pl.num_tiles - tp.narrow_tiles;
      pl.narrow_tiles = tp.narrow_tiles;
    } else if (tp.sk_tiles > 0 && static_cast<int64_t>(tp.sk_tiles) * kb < (int64_t(1) << 31)) {
      // (the device indexes the region with 32-bit iteration numbers)
      clusters = P;
      pl.dp_tiles = pl.num_tiles - tp.sk_tiles;
      pl.sk_tiles = tp.sk_tiles;
      pl.sk_snap = snap;
      pl.partial_floats = static_cast<int64_t>(2 * P) * kCG * C::BM * kBN;
      pl.counter_ints = static_cast<int64_t>(tp.sk_tiles) * kCG;
    }
  }
  pl.grid = clusters * kCG;
  pl.launch = &launch<kCG, kBN, kOutF32>;
  return BB_OK;
}

int plan_init(Plan& pl, int variant, int sm_count) {
  const KernelChoice ch = choose(variant, pl.m, pl.n, pl.k, sm_count);
  pl.cg = ch.cg;
  pl.persistent = ch.persistent;
  // BB_GEMM_PDL=0 turns programmatic dependent launch off.
  const char* pdl_env = std::getenv("BB_GEMM_PDL");
  pl.pdl = !(pdl_env && std::atoi(pdl_env) == 0);
  pl.stream_k = ch.stream_k;
  pl.group_m = ch.group_m;
  if (variant == BB_VARIANT_TUNED) {
    // Tuned: a raster group's A rows total about 32 MiB (a quarter of L2),
    // so the A block of a wave stays resident while B streams (measured:
    // 32768x512x4096 +24 %, 4096^3 +1 % over 8 tile-rows).
    const int64_t tile_rows = 128 * static_cast<int64_t>(ch.cg);
    const int64_t g = (32ll << 20) / (tile_rows * pl.k * 2);
    const int64_t tiles_m = (pl.m + tile_rows - 1) / tile_rows;
    pl.group_m = static_cast<int>(g < 1 ? 1 : (g > tiles_m ? tiles_m : g));
  }
  // BB_GEMM_GROUP_M=g overrides the raster group (tile-rows per group).
  if (const char* g_env = std::getenv("BB_GEMM_GROUP_M")) {
    const int g = std::atoi(g_env);
    if (g > 0) pl.group_m = g;
  }
  pl.variant = variant;
  // Ring waits that spin instead of suspending: the producer's (bit 0; a
  // suspended producer wakes late and refills the freed slot later: +1-2 %
  // on the tuned tiles, +8 % on 256 x 128 tiles) and the MMA warp's (bit 1;
  // no gain measured). BB_GEMM_SPIN=<bits> overrides.
  pl.spin = 1;
  if (const char* e = std::getenv("BB_GEMM_SPIN")) pl.spin = std::atoi(e);
  const bool f32 = pl.c_dtype == BB_DTYPE_F32;
  int rc = BB_ERR_INTERNAL;
  if (ch.cg == 1 && ch.bn == 128) rc = f32 ? prepare<1, 128, true>(pl, sm_count) : prepare<1, 128, false>(pl, sm_count);
  else if (ch.cg == 1 && ch.bn == 256) rc = f32 ? prepare<1, 256, true>(pl, sm_count) : prepare<1, 256, false>(pl, sm_count);
  else if (ch.cg == 2 && ch.bn == 128) rc = f32 ? prepare<2, 128, true>(pl, sm_count) : prepare<2, 128, false>(pl, sm_count);
  else if (ch.cg == 2 && ch.bn == 256) rc = f32 ? prepare<2, 256, true>(pl, sm_count) : prepare<2, 256, false>(pl, sm_count);
  else if (ch.cg == 2 && ch.bn == 512) rc = f32 ? prepare<2, 512, true>(pl, sm_count) : prepare<2, 512, false>(pl, sm_count);
  if (rc == BB_ERR_INTERNAL) set_error("no kernel for cta_group=%d bn=%d", ch.cg, ch.bn);
  return rc;
}

}  // namespace gemm
}  // namespace bb
