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

struct Params {
  int32_t m, n, k, l;
  int32_t tiles_m, tiles_n;
  int32_t num_tiles;
  int32_t k_blocks;
  int32_t group_m;
  int32_t num_clusters;
  // Data-parallel tiles [0, dp_tiles) go to cluster t % num_clusters with
  // the full K range. Each tile of the tail [dp_tiles, num_tiles) is split
  // into sk_parts equal k-block ranges, all in one round: part j of tail
  // tile t is the work of cluster t * sk_parts + j, after its data-parallel
  // tiles (the host guarantees tail_tiles * sk_parts <= num_clusters).
  int32_t dp_tiles;
  int32_t sk_parts;  // 0: no split tail
  float* partials;   // split-tail FP32 partial slices: (parts - 1) tile-sized areas per tail tile and CTA rank
  int* counters;     // two counters (arrived, done) per tail tile and CTA rank
  int* status;
  // Epilogue D = alpha * acc + beta * Csrc (epi_mode 0: alpha 1, beta 0;
  // 1: alpha only; 2: alpha and beta). Csrc has the output's dtype and
  // (L, M, N) row-major layout and may alias the output.
  int32_t epi_mode;
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
  int part;      // -1 for a whole tile, else the part index within the tile
};

// Work item `idx` of cluster c: its data-parallel tiles first, then its
// parts of split tail tiles.
__device__ __forceinline__ bool next_item(const Params& p, int c, int idx, WorkItem& it) {
  const int n_dp = c < p.dp_tiles ? (p.dp_tiles - 1 - c) / p.num_clusters + 1 : 0;
  if (idx < n_dp) {
    it.tile = c + idx * p.num_clusters;
    it.kb0 = 0;
    it.kb1 = p.k_blocks;
    it.part = -1;
    return true;
  }
  if (p.sk_parts == 0 || idx != n_dp) return false;
  const int n_parts = (p.num_tiles - p.dp_tiles) * p.sk_parts;
  if (c >= n_parts) return false;
  const int t_local = c / p.sk_parts;
  const int j = c - t_local * p.sk_parts;
  it.tile = p.dp_tiles + t_local;
  it.kb0 = (j * p.k_blocks) / p.sk_parts;
  it.kb1 = ((j + 1) * p.k_blocks) / p.sk_parts;
  it.part = j;
  return true;
}

// Bounded spin until *ctr >= target (acquire). Returns false on timeout or
// when another role recorded an error.
__device__ __forceinline__ bool spin_until_at_least(const int* ctr, int target, int* status, int code) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (v >= target) return true;
    if ((++spins & 15u) == 0) {
      if (globaltimer_ns() - t0 > kWaitBudgetNs) {
        atomicCAS(status, 0, code);
        return false;
      }
      if (*reinterpret_cast<volatile int*>(status) != 0) return false;
    }
    __nanosleep(64);
  }
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

constexpr int kBK = 64;  // K elements per stage: one 128-byte swizzle row of BF16

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
  static_assert(SMEM_BYTES <= SMEM_LIMIT, "shared memory budget");
  static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation size");
  static_assert(kBN % EPI_COLS == 0, "epilogue chunking");
  static_assert(B_BYTES % 1024 == 0 && A_BYTES % 1024 == 0, "swizzle atoms need 1 KiB alignment");
  // MMA shape legality for kind::f16: M=128 needs N%16==0, 16<=N<=256;
  // M=256 (cta_group::2) the same.
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
                   const __grid_constant__ CUtensorMap tm_c, const Params p) {
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

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const bool mma_cta = (kCG == 1) || (rank == 0);

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
    prefetch_tmap(&tm_c);
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
    for (int idx = 0; ok && next_item(p, cluster_idx, idx, it); ++idx) {
      int l, m_blk, n_blk;
      tile_coords(p, it.tile, l, m_blk, n_blk);
      const int a_row = m_blk * C::TILE_M + static_cast<int>(rank) * C::BM;
      const int b_row = n_blk * kBN + static_cast<int>(rank) * C::B_BOX_ROWS;
      for (int kb = it.kb0; kb < it.kb1; ++kb) {
        if (!bb_wait_warp<kCG == 2>(smem_u32(&empty[stage]), phase ^ 1u, p.status, kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        if (elect_one()) {
          const uint32_t fb = smem_u32(&full[stage]);
          if (mma_cta) mbar_arrive_expect_tx(fb, C::STAGE_BYTES * kCG);
          const uint32_t da = smem_u32(smem_a + stage * C::A_BYTES);
          const uint32_t db = smem_u32(smem_b + stage * C::B_BYTES);
          if constexpr (kCG == 2) {
            const uint32_t fbc = mapa_shared(fb, full_target_rank);
            tma_load_3d_pair(da, &tm_a, fbc, kb * kBK, a_row, l);
#pragma unroll
            for (int h = 0; h < C::N_SUB; ++h)
              tma_load_3d_pair(db + h * C::B_SUB_BYTES, &tm_b, fbc, kb * kBK, b_row + h * C::MMA_N, l);
          } else {
            tma_load_3d(da, &tm_a, fb, kb * kBK, a_row, l);
#pragma unroll
            for (int h = 0; h < C::N_SUB; ++h)
              tma_load_3d(db + h * C::B_SUB_BYTES, &tm_b, fb, kb * kBK, b_row + h * C::MMA_N, l);
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
      constexpr uint32_t idesc = make_idesc_bf16_f32(C::TILE_M, C::MMA_N);
      const uint64_t a_desc0 = sw128_kmajor_desc(smem_u32(smem_a));
      const uint64_t b_desc0 = sw128_kmajor_desc(smem_u32(smem_b));
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_iter = 0;
      WorkItem it;
      for (int idx = 0; ok && next_item(p, cluster_idx, idx, it); ++idx, ++acc_iter) {
        const uint32_t acc = acc_iter % C::ACC_BUFS;
        const uint32_t acc_phase = (acc_iter / C::ACC_BUFS) & 1u;
        if (!bb_wait_warp<kCG == 2>(smem_u32(&tmem_empty[acc]), acc_phase ^ 1u, p.status, kDevTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kBN;
        for (int kb = it.kb0; kb < it.kb1; ++kb) {
          if (!bb_wait_warp<kCG == 2>(smem_u32(&full[stage]), phase, p.status, kDevTimeoutMma)) {
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
#pragma unroll
              for (int h = 0; h < C::N_SUB; ++h) {
                umma_f16<kCG>(d_tmem + h * C::MMA_N, a_desc + 2 * kk, b_desc + h * (C::B_SUB_BYTES >> 4) + 2 * kk,
                              idesc, (kb != it.kb0 || kk != 0) ? 1u : 0u);
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
    for (int idx = 0; next_item(p, cluster_idx, idx, it); ++idx, ++acc_iter) {
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
          constexpr int kWarpChunks = C::WARP_COLS / C::EPI_COLS;
#pragma unroll 1
          for (int c = 0; c < kWarpChunks; ++c) {
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
            if (c == kWarpChunks - 1) release_acc(acc);  // accumulator now lives in registers
            apply_epilogue<kOutF32, ncols>(p, *reinterpret_cast<float(*)[ncols]>(v), row0 + lane, n_blk * kBN + col, l);
            uint32_t packed[32];
            pack_chunk(v, packed);
            store_chunk(packed, row0, n_blk * kBN + col, l);
          }
        }
      } else {
        // ---- part j of a tile split in s along K. Columns are cut into s
        // slices; part j writes its FP32 values of every slice but its own to
        // the workspace, waits until all s parts have written, then sums
        // slice j over the parts in part order (the same fixed order for
        // every slice, so the result does not depend on timing) and stores
        // it. Each block is laid out [col / 4][row][4] floats, so one warp
        // access of a column quad covers 512 contiguous bytes.
        const int t_local = it.tile - p.dp_tiles;
        const int parts = p.sk_parts;
        const int j = it.part;
        const int row = q * 32 + lane;
        const int slice = kBN / parts;  // multiple of 64: parts in {2, 4}, kBN 128, 256 or 512
        // Block (i, w): part w's values of column slice i (w != i), BM rows x
        // slice columns; the tile's (parts - 1) * parts blocks are packed.
        const int64_t tile_base = (static_cast<int64_t>(t_local) * kCG + rank) * (parts - 1) * (C::BM * kBN);
        auto block_ptr = [&](int i, int w) {
          const int idx = i * (parts - 1) + (w < i ? w : w - 1);
          return reinterpret_cast<float4*>(p.partials + tile_base + static_cast<int64_t>(idx) * C::BM * slice) + row;
        };
#pragma unroll 1
        for (int c = wc0 / 32; c < (wc0 + C::WARP_COLS) / 32; ++c) {
          const int i = (c * 32) / slice;
          if (i == j) continue;  // own slice stays in TMEM
          float4* dst = block_ptr(i, j) + ((c * 32 - i * slice) / 4) * C::BM;
          uint32_t r0[32];
          tmem_ld_32x32b_x32(t_row + c * 32, r0);
          tmem_ld_wait();
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            __stcg(dst + jj * C::BM,
                   make_float4(__uint_as_float(r0[4 * jj]), __uint_as_float(r0[4 * jj + 1]),
                               __uint_as_float(r0[4 * jj + 2]), __uint_as_float(r0[4 * jj + 3])));
          }
        }
        __threadfence();
        named_bar_sync(1, kEpiThreads);
        int* arrived = p.counters + 2 * (t_local * kCG + static_cast<int>(rank));
        int* done = arrived + 1;
        if (ep_tid == 0) {
          atomicAdd(arrived, 1);
          epi_flag[0] = spin_until_at_least(arrived, parts, p.status, kDevTimeoutEpilogue) ? 1 : 0;
          __threadfence();
        }
        named_bar_sync(1, kEpiThreads);
        const bool peers_ok = epi_flag[0] != 0;
        if (peers_ok) {
          const int own0 = j * slice > wc0 ? j * slice : wc0;
          const int own1 = (j + 1) * slice < wc0 + C::WARP_COLS ? (j + 1) * slice : wc0 + C::WARP_COLS;
          for (int c = own0 / ncols; c < own1 / ncols; ++c) {
            float own[64];
            {
              uint32_t r0[32];
              tmem_ld_32x32b_x32(t_row + c * ncols, r0);
              if constexpr (!kOutF32) {
                uint32_t r1[32];
                tmem_ld_32x32b_x32(t_row + c * ncols + 32, r1);
                tmem_ld_wait();
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) own[32 + jj] = __uint_as_float(r1[jj]);
              } else {
                tmem_ld_wait();
              }
#pragma unroll
              for (int jj = 0; jj < 32; ++jj) own[jj] = __uint_as_float(r0[jj]);
            }
            float v[64];
#pragma unroll
            for (int jj = 0; jj < ncols; ++jj) v[jj] = 0.0f;
            for (int part = 0; part < parts; ++part) {
              if (part == j) {
#pragma unroll
                for (int jj = 0; jj < ncols; ++jj) v[jj] += own[jj];
                continue;
              }
              const float4* src = block_ptr(j, part) + ((c * ncols - j * slice) / 4) * C::BM;
              float4 x[ncols / 4];
#pragma unroll
              for (int jj = 0; jj < ncols / 4; ++jj) x[jj] = __ldcg(src + jj * C::BM);
#pragma unroll
              for (int jj = 0; jj < ncols / 4; ++jj) {
                v[4 * jj] += x[jj].x;
                v[4 * jj + 1] += x[jj].y;
                v[4 * jj + 2] += x[jj].z;
                v[4 * jj + 3] += x[jj].w;
              }
            }
            apply_epilogue<kOutF32, ncols>(p, *reinterpret_cast<float(*)[ncols]>(v), row0 + lane,
                                           n_blk * kBN + c * C::EPI_COLS, l);
            uint32_t packed[32];
            pack_chunk(v, packed);
            store_chunk(packed, row0, n_blk * kBN + c * C::EPI_COLS, l);
          }
        }
        release_acc(acc);
        named_bar_sync(1, kEpiThreads);
        if (ep_tid == 0 && peers_ok) {
          // Every part has passed its wait: the last one resets both
          // counters for the next launch.
          if (atomicAdd(done, 1) == parts - 1) {
            atomicExch(arrived, 0);
            atomicExch(done, 0);
          }
        }
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
  // Two CTA-pair tile shapes: 256 x 256 (double-buffered TMEM accumulator,
  // split tail) and 256 x 512 (two N = 256 MMAs per K step sharing A: 36 %
  // fewer operand bytes staged per FLOP, but one accumulator buffer, so
  // each tile's epilogue is exposed). BB_GEMM_TILE_N=256|512 forces one.
  const char* tn = std::getenv("BB_GEMM_TILE_N");
  if (tn && std::atoi(tn) == 256) return {2, 256, true, 8, true};
  if (tn && std::atoi(tn) == 512) return {2, 512, true, 8, true};
  const int P = sm_count / 2;
  const double kb = static_cast<double>((k + kBK - 1) / kBK);
  auto tiles = [&](int tn_) { return ((m + 255) / 256) * ((n + tn_ - 1) / tn_); };
  // Modelled time in units of one 256 x 256 tile at full tensor rate; the
  // per-shape efficiencies are the measured main-loop tensor-pipe activity.
  const int64_t t256 = tiles(256);
  const int64_t full = t256 / P, rem = t256 % P;
  double tail = 0.0;
  if (rem) {
    int sp = static_cast<int>(P / rem);
    sp = sp > 4 ? 4 : (sp == 3 ? 2 : sp);
    const bool split = kb >= 48 && sp >= 2 && static_cast<double>(t256) / ((full + 1.0) * P) < 0.95;
    tail = split ? 1.0 / sp + 16.0 / kb : 1.0;
  }
  const double time256 = (full + tail) / 0.907;
  const int64_t t512 = tiles(512);
  const double time512 = static_cast<double>((t512 + P - 1) / P) * 2.0 / 0.96 * (1.0 + 2.0 / kb);
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
  prm.sk_parts = pl.sk_parts;
  prm.partials = pl.partials;
  prm.counters = pl.counters;
  prm.status = pl.status;
  prm.epi_mode = pl.epi_mode;
  prm.alpha = pl.alpha;
  prm.beta = pl.beta;
  prm.c_src = pl.c_src;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, pl.tm_a, pl.tm_b, pl.tm_c, prm), "cudaLaunchKernelEx(gemm)");
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
  pl.sk_parts = 0;
  // BB_GEMM_STREAM_K=0 disables the split tail, =1 uses it whenever the
  // last wave is partial (tuning override; unset: efficiency threshold and
  // at least 48 k-blocks, below which the partial exchange costs more than
  // the idle half tile it saves).
  const char* sk_env = std::getenv("BB_GEMM_STREAM_K");
  const int sk_mode = sk_env ? std::atoi(sk_env) : -1;
  if (pl.stream_k && pl.persistent && (pl.k_blocks >= 48 || sk_mode == 1) && sk_mode != 0) {
    // Split tail: when the last wave of whole tiles would leave clusters
    // idle, each of the rem tail tiles is cut into s equal K parts, s = 4 or
    // 2, the largest with rem * s <= P, so the tail takes about 1/s of a
    // tile time plus the exchange of partial slices.
    const int P = max_clusters;
    const int full = pl.num_tiles / P;
    const int rem = pl.num_tiles % P;
    const double waves = static_cast<double>(full + (rem ? 1 : 0));
    const double eff = static_cast<double>(pl.num_tiles) / (waves * P);
    if (rem != 0 && (eff < 0.95 || sk_mode == 1)) {
      // One round of parts only (every part of a tile runs at the same
      // time, so the wait for peer parts is short and cannot form chains).
      int sp = P / rem;
      if (sp > 4) sp = 4;
      if (sp == 3) sp = 2;  // slices must stay multiples of 64 columns
      if (sp >= 2 && kBN / sp >= 64) {
        clusters = P;
        pl.dp_tiles = full * P;
        pl.sk_parts = sp;
        pl.partial_floats = static_cast<int64_t>(rem) * (sp - 1) * kCG * C::BM * kBN;
        pl.counter_ints = static_cast<int64_t>(rem) * kCG * 2;
      }
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
