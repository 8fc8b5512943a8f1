// Block-scaled low-precision GEMMs for sm_100a (FP8 128 x 128-block, NVFP4):
//   D (M x N, BF16) = dequant(A) (M x K) * dequant(B)^T (N x K), FP32 accumulate.
//
// Two operand formats, one persistent warp-specialised kernel:
//
//   NVFP4  A, B: E2M1 packed two per byte (element 2i in the low nibble),
//          K-major; one UE4M3 scale per 16 K elements of each row, stored
//          as 512-byte scale atoms (128 rows x 4 scales; scale j of row r
//          at byte (r % 32) * 16 + (r / 32) * 4 + j), atoms ordered
//          [row block][K / 64]; a per-tensor FP32 scale (product of A's and
//          B's) applied in the epilogue. The scales are applied by the tensor
//          core itself: tcgen05.mma.kind::mxf4nvf4.block_scale.block16 reads
//          them from TMEM, where tcgen05.cp.32x128b.warpx4 places each atom.
//
//   FP8    A, B: E4M3, K-major; one FP32 scale per 128 x 128 block of each
//          operand. FP32 scales cannot be applied by the tensor core, so every
//          128-wide K block is accumulated on its own (tcgen05.mma.kind::f8f6f4
//          into one of two TMEM partial buffers) and promoted by the epilogue
//          warps into FP32 registers: acc += partial * sa[m][kb] * sb[n][kb].
//          The MMA of K block kb+1 overlaps the promotion of kb.
//
// Tiles: 128 x 256 per CTA, or 256 x 256 per CTA pair (tcgen05.mma
// .cta_group::2; each CTA stages its own 128 A rows and 128 of the B rows,
// loads complete on the leader CTA's barriers, the leader's single thread
// issues the scale copies and MMAs and commits to both CTAs' barriers).
// Roles (320 threads, one CTA per SM):
//   warp 0      producer: TMA loads of A (128 x 128 B) and B (256 or 128 x
//               128 B) per K block, plus (NVFP4) the scale atoms (one 2 KiB
//               box for A's 128-row block, one 4 KiB box for B's 256 rows).
//   warp 1      TMEM allocation (512 columns) and the single MMA thread.
//   warps 2-9   epilogue: warp w reads TMEM lane quarter w % 4 and column
//               half (w - 2) / 4, converts to BF16, stages 32 x 64 boxes
//               with the 128-byte swizzle and writes them with TMA stores.
//
// Every wait is bounded (globaltimer budget); a timeout records a status
// code, drains what is in flight and returns.
#include <cuda.h>
#include <cuda_bf16.h>

#include <atomic>
#include <cstdlib>
#include <new>
#include <type_traits>

#include "common.cuh"
#include "ptx.cuh"

namespace bb {
extern std::atomic<int64_t> g_kernel_launches;

namespace lowp {

enum Kind : int { kNvfp4 = BB_LOWP_NVFP4, kFp8Block = BB_LOWP_FP8_BLOCK128 };

constexpr int BM = 128;         // accumulator rows per CTA
constexpr int ROW_BYTES = 128;  // K bytes of one stage row (one 128-byte swizzle row)
// Every ring and hand-off wait acquires at CTA scope, also for barriers the
// peer CTA of a pair signals (its TMA completions, its commits, its relaxed
// arrivals): what the waiter then touches is read by the tensor core
// (operands, TMEM), whose ordering comes from the barrier's phase and the
// tcgen05 fences, not from a cluster-scope acquire. A completed-phase wait
// costs about 27 clocks at CTA scope against about 50 at cluster scope.
constexpr bool kCtaScope = false;  // bb_wait_warp's kClusterScope argument
constexpr int SF_ATOM = 512;    // bytes of one scale atom (128 rows x 4 scales)
constexpr int EPI_WARPS = 8;
constexpr int kLaunchRegs = 168;  // registers per thread the kernels are built for
constexpr int TMEM_COLS = 512;
constexpr int BAR_BYTES = 256;
// Grouped raster: group_m tile-rows are swept across all tile-columns. The
// host sizes a group's A rows to about 32 MiB (a quarter of L2), so a wave's
// A block stays resident while B streams.
constexpr int64_t kGroupABytes = 32ll << 20;
constexpr int SMEM_LIMIT = 232448;

// kCG = 1: one CTA computes a 128 x 256 tile. kCG = 2: a CTA pair computes a
// 256 x 256 tile with tcgen05.mma.cta_group::2; each CTA stages its own 128
// rows of A and 128 of the 256 B rows, its own A scale atoms and all 256 rows
// of B scale atoms (each CTA's TMEM needs the scales of every B row).
template <int kKind, int kCG>
struct Cfg {
  // Warp roles: 0 producer, 1 MMA, [EPI_W0, EPI_W0 + 8) epilogue. FP8 runs
  // a whole control warpgroup (warps 0-3, 2-3 idle) so setmaxnreg can move
  // registers from it to the two epilogue warpgroups (its promotion keeps a
  // 128-float accumulator per thread and issues two TMEM loads per wait).
  // Tiles are 256 columns wide. The code also supports 128-wide FP8 tiles
  // (four 128-column TMEM partial buffers, 64 accumulators per epilogue
  // thread): as CTA pairs they measured 1.25 PFLOP/s at 8192^3 against 2.2
  // for 256-wide tiles, the MMA warp's two barrier waits per 128-K block
  // then costing as much as the block's 256 clocks of MMA work. Splitting a
  // 256-wide tile's K block into two N = 128 halves with their own commits
  // and sub-buffers (one per epilogue warpgroup, reused after 768 instead
  // of 512 MMA clocks) measured 1843 single / 1976 pair TFLOP/s against
  // 2165: the added wait and commit per block cost more than the slack.
  static constexpr int TILE_N = 256;
  static constexpr int WARP_COLS = TILE_N / 2;         // epilogue columns per warp
  static constexpr int FP8_BUFS = TMEM_COLS / TILE_N;  // FP8 partial buffers
  static constexpr bool kRegSplit = kKind == kFp8Block && WARP_COLS == 128;
  static constexpr int EPI_W0 = kRegSplit ? 4 : 2;
  static constexpr int THREADS = 32 * EPI_W0 + 32 * EPI_WARPS;
  // FP8's MMA warp waits once per 128-K block on the promotion hand-off:
  // it spins (no suspend hint) so wake-up latency stays off that chain
  // (8192^3: 2244 against 2165 TFLOP/s). Spinning in every producer and
  // MMA wait of both kinds, and of the BF16 GEMM, measured within 0.5 %.
  static constexpr bool kSpinWaits = kKind == kFp8Block;
  static constexpr int CTRL_REGS = 56;   // warpgroup 0 after setmaxnreg.dec
  static constexpr int EPI_REGS = 224;   // epilogue warpgroups after setmaxnreg.inc
  static_assert(!kRegSplit || 128 * CTRL_REGS + 256 * EPI_REGS <= THREADS * kLaunchRegs,
                "register split exceeds the registers the block is launched with");
  static constexpr int TILE_M = BM * kCG;
  static constexpr int B_ROWS = TILE_N / kCG;                      // B rows staged per CTA
  static constexpr int K_PER_STAGE = kKind == kNvfp4 ? 256 : 128;  // elements
  static constexpr int MMA_K = kKind == kNvfp4 ? 64 : 32;          // elements per instruction
  static constexpr int MMAS = K_PER_STAGE / MMA_K;                 // 4
  static constexpr int A_BYTES = BM * ROW_BYTES;
  static constexpr int B_BYTES = B_ROWS * ROW_BYTES;
  static constexpr int SFA_BYTES = kKind == kNvfp4 ? MMAS * SF_ATOM : 0;      // one row block
  static constexpr int SFB_BYTES = kKind == kNvfp4 ? 2 * MMAS * SF_ATOM : 0;  // two row blocks
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
  // Epilogue staging: per epilogue warp EPI_BOXES boxes of 32 rows x 128
  // bytes (64 BF16 columns), written to D by TMA stores. One box per warp:
  // a second one cost the NVFP4 pair its fifth ring stage (6170 -> 6512
  // TFLOP/s at 8192^3 with one box and five stages).
  static constexpr int EPI_BOXES = 1;
  static constexpr int EPI_BOX_BYTES = 32 * 128;
  static constexpr int EPI_BYTES = EPI_WARPS * EPI_BOXES * EPI_BOX_BYTES;
  static constexpr int STAGES_FIT = (SMEM_LIMIT - 1024 - BAR_BYTES - EPI_BYTES) / STAGE_BYTES;
  // NVFP4 keeps one TMEM scale area (48 columns) per stage next to the
  // 256-column accumulator.
  static constexpr int STAGES_MAX = kKind == kNvfp4 ? 5 : 8;
  static constexpr int STAGES = STAGES_FIT < STAGES_MAX ? STAGES_FIT : STAGES_MAX;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES;
  static_assert(STAGES >= 3, "ring too shallow");
  static_assert((2 * STAGES + 12) * 8 <= BAR_BYTES, "barrier area");
  static_assert(SMEM_BYTES <= SMEM_LIMIT, "shared memory budget");
  static_assert(MMAS * 32 == ROW_BYTES, "one instruction consumes 32 bytes of each row");
  static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "swizzle atoms need 1 KiB alignment");
};

// NVFP4 TMEM map: two overlapping accumulators, tile j in buffer j % 2 at
// columns [192 b, 192 b + 256): they share one 64-column subtile, which the
// epilogue drains first, so the next tile's MMAs start while the other 192
// columns of the previous tile are still being read. One 48-column scale
// area at 448 (SFA of instruction g at +4g, SFB at +16 + 8g: two 128-row
// atoms), rewritten every stage: scale copies and MMAs of the issuing thread
// execute in issue order, so a copy never overtakes the MMA that reads the
// previous stage's scales. FP8 TMEM map: partial buffer b at 256 b.
constexpr uint32_t kAccStride = 192;     // NVFP4 accumulator b at column 192 b
constexpr uint32_t kOverlapCols = 64;    // columns shared by the two accumulators
constexpr uint32_t kSfBase = 448;
static_assert(kAccStride + 256 <= kSfBase && kSfBase + 48 <= TMEM_COLS, "NVFP4 TMEM map");
static_assert(kAccStride + kOverlapCols == 256, "accumulators overlap by one 64-column subtile");

struct Params {
  int32_t m, n, k;
  int32_t tiles_m, tiles_n, num_tiles;
  int32_t k_stages;    // K / K_PER_STAGE
  int32_t rb_m, rb_n;  // 128-row blocks of A and B
  int32_t num_clusters;
  int32_t group_m;
  const uint8_t* sfa;  // FP8: FP32 block scales (NVFP4 scales travel by TMA)
  const uint8_t* sfb;
  float global_scale;
  __nv_bfloat16* d;
  int* status;
};

// Instruction descriptors.
//   kind::f8f6f4 (E4M3 x E4M3 -> F32): [4,6) D fmt 1, [7,10) A fmt 0,
//     [10,13) B fmt 0, [17,23) N >> 3, [24,29) M >> 4.
//   kind::mxf4nvf4 block-scaled: [4,6) B scale id 0, [7,10) A fmt 1 (E2M1),
//     [10,13) B fmt 1, [17,23) N >> 3, [23] scale fmt 0 (UE4M3),
//     [24,29) M >> 4, [29,31) A scale id 0, [31] K size 0 (K = 64).
__host__ __device__ constexpr uint32_t idesc_f8(int m, int n) {
  return (1u << 4) | ((static_cast<uint32_t>(n) >> 3) << 17) | ((static_cast<uint32_t>(m) >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_nvf4(int m, int n) {
  return (1u << 7) | (1u << 10) | ((static_cast<uint32_t>(n) >> 3) << 17) |
         ((static_cast<uint32_t>(m) >> 4) << 24);
}
static_assert(idesc_f8(128, 256) == 0x08400010u, "f8f6f4 idesc");
static_assert(idesc_nvf4(128, 256) == 0x08400480u, "mxf4nvf4 idesc");
static_assert(idesc_nvf4(256, 256) == 0x10400480u, "mxf4nvf4 idesc, CTA pair");

template <int kCG>
__device__ __forceinline__ void mma_f8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  if constexpr (kCG == 1) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
  }
}
template <int kCG>
__device__ __forceinline__ void mma_nvf4(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t tsfa,
                                         uint32_t tsfb, uint32_t acc) {
  if constexpr (kCG == 1) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
            d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(tsfa), "r"(tsfb)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
            d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(tsfa), "r"(tsfb)
        : "memory");
  }
}
// Shared-memory descriptor of one 512-byte scale atom (32 rows x 16 bytes):
// interleaved (no-swizzle) K-major layout, 8-row core matrices of 128
// contiguous bytes stacked every 128 bytes along the rows (SBO).
__device__ __forceinline__ uint64_t sf_atom_desc(uint32_t smem_addr) {
  return make_smem_desc(smem_addr, 128, 128, kLayoutNone);
}
// One scale atom into 4 TMEM columns, replicated into the four 32-lane
// quarters (each quarter of the MMA reads its own lanes). With cta_group::2
// each CTA of the pair copies from its own shared memory into its own TMEM.
template <int kCG>
__device__ __forceinline__ void tmem_cp_desc(uint32_t taddr, uint64_t desc) {
  if constexpr (kCG == 1) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(desc) : "memory");
  } else {
    asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(desc) : "memory");
  }
}

// Rank-2 tile loads: into this CTA's shared memory, completing on this CTA's
// mbarrier (1 CTA) or on the leader CTA's mbarrier (pair form). The data goes
// to the issuing CTA only.
template <int kCG>
__device__ __forceinline__ void load_2d(uint32_t dst, const void* tmap, uint32_t mbar, int32_t x, int32_t y) {
  if constexpr (kCG == 1) {
    tma_load_2d(dst, tmap, mbar, x, y);
  } else {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(tmap), "r"(mbar), "r"(x), "r"(y)
        : "memory");
  }
}

__device__ __forceinline__ void tile_coords(const Params& p, int t, int& m_blk, int& n_blk) {
  const int group_size = p.group_m * p.tiles_n;
  const int g = t / group_size;
  const int first_m = g * p.group_m;
  const int gm = min(p.group_m, p.tiles_m - first_m);
  const int local = t - g * group_size;
  m_blk = first_m + local % gm;
  n_blk = local / gm;
}

// Converts 32 FP32 accumulator values (scaled by s) to 16 packed BF16 pairs.
__device__ __forceinline__ void pack32(const float* v, float s, uint32_t* out) {
#pragma unroll
  for (int j = 0; j < 16; ++j) out[j] = pack_bf16x2(v[2 * j] * s, v[2 * j + 1] * s);
}

// FP32 promotion acc += v * s for 32 values, two lanes per instruction
// (packed fma.rn.f32x2 of sm_100).
__device__ __forceinline__ void promote32(float* acc, const uint32_t (&v)[32], float s) {
  const uint64_t s2 = (static_cast<uint64_t>(__float_as_uint(s)) << 32) | __float_as_uint(s);
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    uint64_t a2 = (static_cast<uint64_t>(__float_as_uint(acc[2 * j + 1])) << 32) | __float_as_uint(acc[2 * j]);
    const uint64_t v2 = (static_cast<uint64_t>(v[2 * j + 1]) << 32) | v[2 * j];
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(a2) : "l"(v2), "l"(s2));
    acc[2 * j] = __uint_as_float(static_cast<uint32_t>(a2));
    acc[2 * j + 1] = __uint_as_float(static_cast<uint32_t>(a2 >> 32));
  }
}

template <int kKind, int kCG>
__global__ void __launch_bounds__(Cfg<kKind, kCG>::THREADS, 1)
    bb_lowp_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        const __grid_constant__ CUtensorMap tm_sfa, const __grid_constant__ CUtensorMap tm_sfb,
                        const __grid_constant__ CUtensorMap tm_d, const Params p) {
  using C = Cfg<kKind, kCG>;
  constexpr int STAGES = C::STAGES;
  constexpr bool kPair = kCG == 2;
  const uint32_t rank = kPair ? cluster_ctarank() : 0u;
  if (blockDim.x != C::THREADS || (kPair && cluster_nctarank() != 2) || (gridDim.x % kCG) != 0) {
    if (threadIdx.x == 0 && p.status) atomicCAS(p.status, 0, kDevBadLaunch);
    return;
  }
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem_a + STAGES * C::A_BYTES;
  uint8_t* smem_sfa = smem_b + STAGES * C::B_BYTES;        // NVFP4 only
  uint8_t* smem_sfb = smem_sfa + STAGES * C::SFA_BYTES;    // NVFP4 only
  uint8_t* smem_epi = smem + STAGES * C::STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_epi + C::EPI_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;       // [4]
  uint64_t* acc_empty = bars + 2 * STAGES + 4;  // [4], in the leader CTA: buffer fully drained
  uint64_t* ovl_free = bars + 2 * STAGES + 8;   // [2], in the leader CTA: NVFP4 shared subtile drained
  uint64_t* mma_done = bars + 2 * STAGES + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 11);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const bool leader = rank == 0;

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
    prefetch_tmap(&tm_d);
    if constexpr (kKind == kNvfp4) {
      prefetch_tmap(&tm_sfa);
      prefetch_tmap(&tm_sfb);
    }
  }
  if (warp == 1 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 4; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_empty[b]), EPI_WARPS * kCG);
    }
    for (int b = 0; b < 2; ++b) mbar_init(smem_u32(&ovl_free[b]), (EPI_WARPS / 2) * kCG);
    mbar_init(smem_u32(mma_done), 1);
    fence_mbarrier_init_cluster();
  }
  if (warp == 1) {
    tmem_alloc<kCG>(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish<kCG>();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (kPair) cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  const int cluster_idx = blockIdx.x / kCG;

  if (warp < C::EPI_W0) {
    if constexpr (C::kRegSplit) {
      // Warpgroup 0 (producer, MMA, two idle warps) gives registers to the
      // epilogue warpgroups (setmaxnreg sits inside each role's branch so
      // the register allocator sees one limit per region). The host checks
      // the block's launch register pool covers the split before launching.
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::CTRL_REGS));
    }
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The whole warp runs the loop and waits; one elected lane issues.
    bool ok = true;
    int stage = 0;
    uint32_t phase = 0;
    for (int t = cluster_idx; ok && t < p.num_tiles; t += p.num_clusters) {
      int m_blk, n_blk;
      tile_coords(p, t, m_blk, n_blk);
      const int a_row = m_blk * C::TILE_M + static_cast<int>(rank) * BM;
      const int b_row = n_blk * C::TILE_N + static_cast<int>(rank) * C::B_ROWS;
      const int sfa_blk = m_blk * kCG + static_cast<int>(rank);
      for (int ks = 0; ks < p.k_stages; ++ks) {
        if (!bb_wait_warp<kCtaScope>(smem_u32(&empty[stage]), phase ^ 1u, p.status, kDevTimeoutProducer)) {
          ok = false;
          break;
        }
        if (elect_one()) {
          const uint32_t fb_own = smem_u32(&full[stage]);
          const uint32_t fb = kPair ? mapa_shared(fb_own, 0) : fb_own;
          if (leader) mbar_arrive_expect_tx(fb_own, C::STAGE_BYTES * kCG);
          load_2d<kCG>(smem_u32(smem_a + stage * C::A_BYTES), &tm_a, fb, ks * ROW_BYTES, a_row);
          load_2d<kCG>(smem_u32(smem_b + stage * C::B_BYTES), &tm_b, fb, ks * ROW_BYTES, b_row);
          if constexpr (kKind == kNvfp4) {
            // Scale atoms as rows of 8-byte words: one row per 128-row block,
            // K/64 atoms of 64 words each; a stage is 4 atoms (256 words).
            load_2d<kCG>(smem_u32(smem_sfa + stage * C::SFA_BYTES), &tm_sfa, fb, ks * 256, sfa_blk);
            load_2d<kCG>(smem_u32(smem_sfb + stage * C::SFB_BYTES), &tm_sfb, fb, ks * 256, 2 * n_blk);
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
        if (!bb_wait_warp<kCtaScope>(smem_u32(&empty[stage]), phase ^ 1u, p.status, kDevTimeoutProducer)) break;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    } else if (lane == 0) {
      bounded_sleep_ns(2000000);  // aborted: let copies already issued land
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA)
    // Whole warp runs the loop and waits; one elected lane issues the scale
    // copies, MMAs and commits of each stage (always the same lane: elect.sync
    // picks the lowest active lane of the converged warp).
    if (leader) {
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_iter = 0;  // NVFP4: tiles; FP8: K blocks (partial buffers)
      // Stage-0 descriptors; stage s adds s times the stage size (in 16-byte
      // units, the unit of the descriptors' start-address field).
      const uint64_t a_desc0 = sw128_kmajor_desc(smem_u32(smem_a));
      const uint64_t b_desc0 = sw128_kmajor_desc(smem_u32(smem_b));
      const uint64_t sfa_desc0 = sf_atom_desc(smem_u32(smem_sfa));
      const uint64_t sfb_desc0 = sf_atom_desc(smem_u32(smem_sfb));
      const uint32_t sf_cols0 = tmem_base + kSfBase;
      auto commit_both = [&](uint64_t* bar) {
        const uint32_t a = smem_u32(bar);
        umma_commit<kCG>(a);
        if constexpr (kPair) umma_commit<kCG>(mapa_shared(a, 1));
      };
      for (int t = cluster_idx; ok && t < p.num_tiles; t += p.num_clusters) {
        uint32_t acc_col = 0;
        if constexpr (kKind == kNvfp4) {
          // Tile j goes to buffer j % 2: wait until tile j - 2 left it, and
          // until tile j - 1 (the other buffer) drained the shared subtile.
          const uint32_t b = acc_iter & 1u;
          if (!bb_wait_warp<kCtaScope>(smem_u32(&acc_empty[b]), ((acc_iter >> 1) & 1u) ^ 1u, p.status,
                                   kDevTimeoutMma)) {
            ok = false;
            break;
          }
          if (acc_iter > 0 && !bb_wait_warp<kCtaScope>(smem_u32(&ovl_free[b ^ 1u]), ((acc_iter - 1) >> 1) & 1u,
                                                   p.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          acc_col = b * kAccStride;
        }
        for (int ks = 0; ks < p.k_stages; ++ks) {
          uint32_t d_tmem = tmem_base + acc_col;
          uint32_t buf = 0;
          // The stage's operands are normally resident long before its
          // partial buffer is free (FP8), so the data wait comes first and
          // only the buffer hand-off stands between the release and the MMAs.
          if (!bb_wait_warp<kCtaScope, !C::kSpinWaits>(smem_u32(&full[stage]), phase, p.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          if constexpr (kKind == kFp8Block) {
            buf = acc_iter % C::FP8_BUFS;
            if (!bb_wait_warp<kCtaScope, !C::kSpinWaits>(smem_u32(&acc_empty[buf]), ((acc_iter / C::FP8_BUFS) & 1u) ^ 1u,
                                                     p.status, kDevTimeoutMma)) {
              ok = false;
              break;
            }
            d_tmem = tmem_base + buf * C::TILE_N;
          }
          tc_fence_after();
          if (elect_one()) {
            const uint64_t a_desc = a_desc0 + static_cast<uint64_t>(stage) * (C::A_BYTES >> 4);
            const uint64_t b_desc = b_desc0 + static_cast<uint64_t>(stage) * (C::B_BYTES >> 4);
            if constexpr (kKind == kNvfp4) {
              const uint32_t sf_cols = sf_cols0;
              const uint64_t sfa_desc = sfa_desc0 + static_cast<uint64_t>(stage) * (C::SFA_BYTES >> 4);
              const uint64_t sfb_desc = sfb_desc0 + static_cast<uint64_t>(stage) * (C::SFB_BYTES >> 4);
              constexpr uint32_t idesc = idesc_nvf4(C::TILE_M, C::TILE_N);
              // Per K step: its three scale copies, then its MMA (copies and
              // MMAs of one thread execute in issue order).
#pragma unroll
              for (int g = 0; g < C::MMAS; ++g) {
                tmem_cp_desc<kCG>(sf_cols + 4 * g, sfa_desc + g * (SF_ATOM >> 4));
                tmem_cp_desc<kCG>(sf_cols + 16 + 8 * g, sfb_desc + g * (SF_ATOM >> 4));
                tmem_cp_desc<kCG>(sf_cols + 20 + 8 * g, sfb_desc + (C::SFB_BYTES / 2 + g * SF_ATOM) / 16);
                mma_nvf4<kCG>(d_tmem, a_desc + 2 * g, b_desc + 2 * g, idesc, sf_cols + 4 * g, sf_cols + 16 + 8 * g,
                              (ks | g) != 0 ? 1u : 0u);
              }
            } else {
              constexpr uint32_t idesc = idesc_f8(C::TILE_M, C::TILE_N);
#pragma unroll
              for (int g = 0; g < C::MMAS; ++g)
                mma_f8<kCG>(d_tmem, a_desc + 2 * g, b_desc + 2 * g, idesc, g != 0 ? 1u : 0u);
            }
            // FP8: this commit also tells the epilogue that K block
            // acc_iter's partial is complete (its wait is on the stage's
            // barrier), so no second commit per block is needed.
            commit_both(&empty[stage]);
          }
          __syncwarp();
          if constexpr (kKind == kFp8Block) ++acc_iter;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (kKind == kNvfp4) {
          if (elect_one()) commit_both(&acc_full[acc_iter & 1u]);
          __syncwarp();
          ++acc_iter;
        }
      }
      // Drain: every MMA issued so far must finish before TMEM is freed.
      if (elect_one()) umma_commit<kCG>(smem_u32(mma_done));
      __syncwarp();
      bb_wait_warp(smem_u32(mma_done), 0, p.status, kDevTimeoutMma, /*honor_abort=*/false);
    }
  }
  } else {
    if constexpr (C::kRegSplit) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C::EPI_REGS));
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int half = (warp - C::EPI_W0) / 4;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    uint32_t acc_iter = 0;
    bool ok = true;
    // One arrival per warp on a barrier of the leader CTA, after this
    // warp's TMEM reads completed.
    auto arrive_leader = [&](uint64_t* bar) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        const uint32_t eb = smem_u32(bar);
        if constexpr (kPair) {
          mbar_arrive_cluster_relaxed(mapa_shared(eb, 0));
        } else {
          mbar_arrive(eb);
        }
      }
    };
    auto release = [&](uint32_t buf) { arrive_leader(&acc_empty[buf]); };
    // D rows row0 .. row0 + 31 (lane = row), columns col0 .. col0 + 127 as two
    // 32 x 64 boxes: each staged with the 128-byte swizzle in this warp's
    // boxes of shared memory and written by one TMA store (clipped at the
    // edges of D; boxes wholly outside D are skipped).
    const uint32_t ebuf = smem_u32(smem_epi + (warp - C::EPI_W0) * C::EPI_BOXES * C::EPI_BOX_BYTES);
    uint32_t box_seq = 0;
    const uint64_t d_policy = l2_policy_evict_first();
    auto store_boxes = [&](int row0, int col0_, const uint32_t(&pk_)[C::WARP_COLS / 2]) {
#pragma unroll
      for (int h = 0; h < C::WARP_COLS / 64; ++h) {
        const uint32_t buf = ebuf + (box_seq % C::EPI_BOXES) * C::EPI_BOX_BYTES;
        ++box_seq;
        if (lane == 0) bulk_wait_group_read<C::EPI_BOXES - 1>();
        __syncwarp();
        const uint32_t row_addr = buf + lane * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          st_shared_v4(row_addr + ((j ^ (lane & 7)) << 4), pk_[32 * h + 4 * j], pk_[32 * h + 4 * j + 1],
                       pk_[32 * h + 4 * j + 2], pk_[32 * h + 4 * j + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // D is written once: evict-first in L2.
          if (row0 < p.m && col0_ + 64 * h < p.n) tma_store_2d_hint(&tm_d, buf, col0_ + 64 * h, row0, d_policy);
          bulk_commit_group();
        }
      }
    };
    for (int t = cluster_idx; ok && t < p.num_tiles; t += p.num_clusters) {
      int m_blk, n_blk;
      tile_coords(p, t, m_blk, n_blk);
      const int row = m_blk * C::TILE_M + static_cast<int>(rank) * BM + q * 32 + lane;
      const int col0 = n_blk * C::TILE_N + half * C::WARP_COLS;
      uint32_t pk[C::WARP_COLS / 2];
      if constexpr (kKind == kNvfp4) {
        const uint32_t b = acc_iter & 1u;
        if (!bb_wait_warp<kCtaScope>(smem_u32(&acc_full[b]), (acc_iter >> 1) & 1u, p.status, kDevTimeoutEpilogue)) break;
        tc_fence_after();
        const uint32_t taddr = tmem_base + lane_off + b * kAccStride + half * C::WARP_COLS;
        // The subtile shared with the other buffer is columns [192, 256) of
        // buffer 0 (this warp's chunks 2, 3 when half == 1) and [0, 64) of
        // buffer 1 (chunks 0, 1 when half == 0); its owners read it first
        // and report it drained before reading the rest.
        const bool owner = (b == 0) ? (half == 1) : (half == 0);
        // Chunk pair c, c + 1 (32 columns each) into pk; compile-time chunk
        // indices keep pk in registers.
        auto drain_pair = [&](auto chunk, bool report) {
          constexpr int c = decltype(chunk)::value;
          uint32_t r0[32], r1[32];
          tmem_ld_32x32b_x32(taddr + 32 * c, r0);
          tmem_ld_32x32b_x32(taddr + 32 * (c + 1), r1);
          tmem_ld_wait();
          if (report) arrive_leader(&ovl_free[b]);
          pack32(reinterpret_cast<const float*>(r0), p.global_scale, pk + 16 * c);
          pack32(reinterpret_cast<const float*>(r1), p.global_scale, pk + 16 * (c + 1));
        };
        if (b == 0) {
          drain_pair(std::integral_constant<int, 2>{}, owner);
          drain_pair(std::integral_constant<int, 0>{}, false);
        } else {
          drain_pair(std::integral_constant<int, 0>{}, owner);
          drain_pair(std::integral_constant<int, 2>{}, false);
        }
        release(b);
        ++acc_iter;
      } else {
        const float* sa = reinterpret_cast<const float*>(p.sfa);
        const float* sb = reinterpret_cast<const float*>(p.sfb);
        // Ragged edges: rows / columns past M / N are never stored, any valid
        // scale row serves them.
        const int mb = min(m_blk * kCG + static_cast<int>(rank), p.rb_m - 1);
        const int nb = min(col0 / 128, p.rb_n - 1);
        const float* sa_row = sa + static_cast<int64_t>(mb) * p.k_stages;
        const float* sb_row = sb + static_cast<int64_t>(nb) * p.k_stages;
        float acc[C::WARP_COLS];
#pragma unroll
        for (int j = 0; j < C::WARP_COLS; ++j) acc[j] = 0.f;
        // Lane l holds the scale product of K block w + l of the current
        // 32-block window (s_win) and the raw scales of the next window,
        // loaded a whole window ahead: the per-block loop reads its scale
        // with one shuffle and never waits on a global load (a load issued
        // one block ahead still stalled each block for an L2 round trip,
        // right before the wait on the MMA hand-off).
        float ra, rb;
        auto load_raw = [&](int kk) {
          ra = 0.f;
          rb = 0.f;
          if (kk < p.k_stages) {
            ra = __ldg(sa_row + kk);
            rb = __ldg(sb_row + kk);
          }
        };
        load_raw(lane);
        float s_win = ra * rb;
        load_raw(32 + lane);
        for (int ks = 0; ks < p.k_stages; ++ks) {
          if ((ks & 31) == 0 && ks > 0) {
            s_win = ra * rb;
            load_raw(ks + 32 + lane);
          }
          const float s = __shfl_sync(0xffffffffu, s_win, ks & 31);
          const uint32_t buf = acc_iter % C::FP8_BUFS;
          // K block acc_iter's partial is complete when the MMA's commit
          // releases its operand stage (one stage per K block, stage =
          // acc_iter % STAGES, that barrier's phase acc_iter / STAGES). The
          // parity cannot be overtaken: the MMA can run at most FP8_BUFS
          // blocks ahead of this wait, and STAGES > FP8_BUFS.
          // Spin without the suspend hint: this wait is on the per-K-block
          // MMA -> promotion -> MMA hand-off, where wake-up latency counts.
          static_assert(STAGES > C::FP8_BUFS, "stage barrier reused before the epilogue saw it");
          if (!bb_wait_warp<kCtaScope, false>(smem_u32(&empty[acc_iter % STAGES]), (acc_iter / STAGES) & 1u, p.status,
                                          kDevTimeoutEpilogue)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t taddr = tmem_base + lane_off + buf * C::TILE_N + half * C::WARP_COLS;
          constexpr int kChunks = C::WARP_COLS / 32;
#pragma unroll
          for (int c = 0; c < kChunks; c += 2) {
            uint32_t r0[32], r1[32];
            tmem_ld_32x32b_x32(taddr + 32 * c, r0);
            tmem_ld_32x32b_x32(taddr + 32 * (c + 1), r1);
            tmem_ld_wait();
            if (c == kChunks - 2) release(buf);
            promote32(acc + 32 * c, r0, s);
            promote32(acc + 32 * (c + 1), r1, s);
          }
          ++acc_iter;
        }
        if (!ok) break;
#pragma unroll
        for (int c = 0; c < C::WARP_COLS / 32; ++c) pack32(acc + 32 * c, p.global_scale, pk + 16 * c);
      }
      store_boxes(row - lane, col0, pk);
    }
    if (lane == 0) bulk_wait_group<0>();  // stores read their staging boxes before exit
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (kPair) cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc<kCG>(tmem_base, TMEM_COLS);
  }
}

}  // namespace lowp
}  // namespace bb

struct bb_lowp_plan {
  int kind = 0;
  int cg = 1;
  int tile_n = 256;
  int stages = 0;
  int64_t m = 0, n = 0, k = 0;
  cudaStream_t stream = nullptr;
  CUtensorMap tm_a{}, tm_b{}, tm_sfa{}, tm_sfb{}, tm_d{};
  bb::lowp::Params params{};
  int grid = 0;
  int smem_bytes = 0;
  int* status_dev = nullptr;
  int64_t launches = 0;
};

using namespace bb;
using namespace bb::lowp;

namespace {

template <int kKind, int kCG>
cudaLaunchConfig_t launch_config(const bb_lowp_plan& pl, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(Cfg<kKind, kCG>::THREADS);
  cfg.dynamicSmemBytes = Cfg<kKind, kCG>::SMEM_BYTES;
  cfg.stream = pl.stream;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCG;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

template <int kKind, int kCG>
int set_attributes() {
  static bool done = false;  // one attribute call per kernel and process
  if (!done) {
    if constexpr (Cfg<kKind, kCG>::kRegSplit) {
      // setmaxnreg.inc waits until the block's register pool can serve it;
      // refuse to launch a build whose pool is smaller than the split needs.
      cudaFuncAttributes fa{};
      BB_CUDA_TRY(cudaFuncGetAttributes(&fa, bb_lowp_gemm_kernel<kKind, kCG>));
      if (fa.numRegs * Cfg<kKind, kCG>::THREADS < 128 * Cfg<kKind, kCG>::CTRL_REGS + 256 * Cfg<kKind, kCG>::EPI_REGS) {
        set_error("bb_lowp: kernel built with %d registers per thread; its register split needs %d", fa.numRegs,
                  kLaunchRegs);
        return BB_ERR_INTERNAL;
      }
    }
    BB_CUDA_TRY(cudaFuncSetAttribute(bb_lowp_gemm_kernel<kKind, kCG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Cfg<kKind, kCG>::SMEM_BYTES));
    done = true;
  }
  return BB_OK;
}

template <int kKind, int kCG>
int launch_kind(const bb_lowp_plan& pl) {
  int rc = set_attributes<kKind, kCG>();
  if (rc != BB_OK) return rc;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = launch_config<kKind, kCG>(pl, attr);
  return check_cuda(cudaLaunchKernelEx(&cfg, bb_lowp_gemm_kernel<kKind, kCG>, pl.tm_a, pl.tm_b, pl.tm_sfa, pl.tm_sfb,
                                       pl.tm_d, pl.params),
                    "launch bb_lowp_gemm_kernel");
}

int launch(const bb_lowp_plan& pl) {
  if (pl.kind == kNvfp4) return pl.cg == 2 ? launch_kind<kNvfp4, 2>(pl) : launch_kind<kNvfp4, 1>(pl);
  return pl.cg == 2 ? launch_kind<kFp8Block, 2>(pl) : launch_kind<kFp8Block, 1>(pl);
}

// Clusters of kCG CTAs resident at once (one CTA per SM: the shared-memory
// ring takes the whole SM).
template <int kKind, int kCG>
int max_clusters(const bb_lowp_plan& pl, int sm_count) {
  int clusters = sm_count / kCG;
  if (kCG > 1 && set_attributes<kKind, kCG>() == BB_OK) {
    bb_lowp_plan probe = pl;
    probe.grid = kCG * clusters;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = launch_config<kKind, kCG>(probe, attr);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, bb_lowp_gemm_kernel<kKind, kCG>, &cfg) == cudaSuccess && n > 0) {
      clusters = n;
    } else {
      cudaGetLastError();
    }
  }
  return clusters;
}

template <int kKind, int kCG>
void plan_geometry(bb_lowp_plan& h, int sm_count) {
  using C = Cfg<kKind, kCG>;
  h.stages = C::STAGES;
  h.tile_n = C::TILE_N;
  h.smem_bytes = C::SMEM_BYTES;
  Params& p = h.params;
  p.tiles_m = static_cast<int32_t>((h.m + C::TILE_M - 1) / C::TILE_M);
  p.tiles_n = static_cast<int32_t>((h.n + C::TILE_N - 1) / C::TILE_N);
  p.num_tiles = p.tiles_m * p.tiles_n;
  const int64_t a_tile_bytes = static_cast<int64_t>(C::TILE_M) * (kKind == kNvfp4 ? h.k / 2 : h.k);
  const int64_t g = kGroupABytes / (a_tile_bytes > 0 ? a_tile_bytes : 1);
  p.group_m = static_cast<int32_t>(g < 1 ? 1 : (g > p.tiles_m ? p.tiles_m : g));
  const int clusters = max_clusters<kKind, kCG>(h, sm_count);
  p.num_clusters = p.num_tiles < clusters ? p.num_tiles : clusters;
  h.grid = p.num_clusters * kCG;
}

}  // namespace

extern "C" {

BB_API size_t bb_lowp_info_size(void) { return sizeof(bb_lowp_info); }

BB_API int64_t bb_lowp_scale_bytes(int kind, int64_t rows, int64_t k) {
  if (rows <= 0 || k <= 0) return -1;
  const int64_t rb = (rows + 127) / 128;
  if (kind == BB_LOWP_NVFP4) return k % 64 ? -1 : rb * (k / 64) * 512;
  if (kind == BB_LOWP_FP8_BLOCK128) return k % 128 ? -1 : rb * (k / 128) * 4;
  return -1;
}

BB_API int bb_lowp_plan_create(int kind, int64_t m, int64_t n, int64_t k, const void* a, const void* b,
                               const void* sfa, const void* sfb, float global_scale, void* d, void* stream,
                               bb_lowp_plan** plan, bb_lowp_info* info) {
  try {
    clear_error();
    if (!plan) {
      set_error("bb_lowp_plan_create: plan out-pointer is null");
      return BB_ERR_ARGUMENT;
    }
    *plan = nullptr;
    if (kind != BB_LOWP_NVFP4 && kind != BB_LOWP_FP8_BLOCK128) {
      set_error("bb_lowp_plan_create: unknown kind %d", kind);
      return BB_ERR_ARGUMENT;
    }
    if (!a || !b || !sfa || !sfb || !d) {
      set_error("bb_lowp_plan_create: null operand pointer");
      return BB_ERR_ARGUMENT;
    }
    if (m <= 0 || n <= 0 || k <= 0 || m > (int64_t(1) << 30) || n > (int64_t(1) << 30) || k > (int64_t(1) << 30)) {
      set_error("bb_lowp_plan_create: extents out of range (m=%lld n=%lld k=%lld)", (long long)m, (long long)n,
                (long long)k);
      return BB_ERR_ARGUMENT;
    }
    const int k_step = kind == BB_LOWP_NVFP4 ? 256 : 128;
    if (k % k_step != 0) {
      set_error("bb_lowp_plan_create: K=%lld must be a multiple of %d for this kind", (long long)k, k_step);
      return BB_ERR_ARGUMENT;
    }
    if (n % 8 != 0) {
      set_error("bb_lowp_plan_create: N=%lld must be a multiple of 8 (16-byte rows of D)", (long long)n);
      return BB_ERR_ARGUMENT;
    }
    for (const void* ptr : {a, b, sfa, sfb, static_cast<const void*>(d)}) {
      if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) {
        set_error("bb_lowp_plan_create: every buffer must be 16-byte aligned");
        return BB_ERR_ARGUMENT;
      }
    }
    DeviceInfo dev;
    int rc = query_device(&dev);
    if (rc != BB_OK) return rc;
    if (dev.major != 10) {
      set_error("bb_lowp_plan_create: needs an sm_100 device (found sm_%d%d)", dev.major, dev.minor);
      return BB_ERR_UNSUPPORTED;
    }
    auto* h = new (std::nothrow) bb_lowp_plan();
    if (!h) {
      set_error("bb_lowp_plan_create: out of host memory");
      return BB_ERR_INTERNAL;
    }
    h->kind = kind;
    h->m = m;
    h->n = n;
    h->k = k;
    h->stream = static_cast<cudaStream_t>(stream);
    // CTA pairs (256-row tiles) unless A has a single 128-row block. For
    // FP8 the pair is the only shape that can approach the tensor rate: a
    // single CTA's 128 x 256 tile moves 96 KiB of shared memory per 128-K
    // block (48 KiB of TMA writes, 48 KiB of MMA operand reads) against the
    // pair's 64 KiB, i.e. about 750 against 500 clocks at 128 B/clock for
    // 512 clocks of MMA. The pair's price is its per-block accumulator
    // hand-off across the CTAs (8192^3: pair 2320-2377, single 2200-2250
    // TFLOP/s). BB_LOWP_CTA_GROUP=1|2 forces one.
    h->cg = m > 128 ? 2 : 1;
    if (const char* env = std::getenv("BB_LOWP_CTA_GROUP")) {
      if (env[0] == '1') h->cg = 1;
      if (env[0] == '2') h->cg = 2;
    }
    if (kind == kNvfp4) {
      if (h->cg == 2) plan_geometry<kNvfp4, 2>(*h, dev.sm_count); else plan_geometry<kNvfp4, 1>(*h, dev.sm_count);
    } else {
      if (h->cg == 2) plan_geometry<kFp8Block, 2>(*h, dev.sm_count); else plan_geometry<kFp8Block, 1>(*h, dev.sm_count);
    }
    // Operands are byte arrays: K / 2 bytes per row for E2M1, K for E4M3.
    const uint64_t row_bytes = kind == BB_LOWP_NVFP4 ? k / 2 : k;
    const uint64_t rb_m = (m + 127) / 128, rb_n = (n + 127) / 128;
    {
      const uint64_t dims[2] = {row_bytes, static_cast<uint64_t>(m)};
      const uint64_t strides[1] = {row_bytes};
      const uint32_t box[2] = {ROW_BYTES, BM};
      rc = encode_tiled(&h->tm_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 2, a, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    }
    if (rc == BB_OK) {
      const uint64_t dims[2] = {row_bytes, static_cast<uint64_t>(n)};
      const uint64_t strides[1] = {row_bytes};
      const uint32_t box[2] = {ROW_BYTES, static_cast<uint32_t>(h->tile_n / h->cg)};
      rc = encode_tiled(&h->tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 2, b, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    }
    if (rc == BB_OK && kind == BB_LOWP_NVFP4) {
      // Scale atoms viewed as rows of 8-byte words, one row per 128-row block
      // (K words: K/64 atoms of 64 words); a stage's box is 256 words (4 atoms).
      const uint64_t strides[1] = {static_cast<uint64_t>(k) * 8};
      const uint64_t dims_a[2] = {static_cast<uint64_t>(k), rb_m};
      const uint32_t box_a[2] = {256, 1};
      rc = encode_tiled(&h->tm_sfa, CU_TENSOR_MAP_DATA_TYPE_UINT64, 8, 2, sfa, dims_a, strides, box_a,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
      if (rc == BB_OK) {
        const uint64_t dims_b[2] = {static_cast<uint64_t>(k), rb_n};
        const uint32_t box_b[2] = {256, 2};
        rc = encode_tiled(&h->tm_sfb, CU_TENSOR_MAP_DATA_TYPE_UINT64, 8, 2, sfb, dims_b, strides, box_b,
                          CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
      }
    } else {
      h->tm_sfa = h->tm_a;  // unused by the FP8 kernel
      h->tm_sfb = h->tm_b;
    }
    if (rc == BB_OK) {
      // D (M x N BF16, row-major) for the epilogue's TMA stores: boxes of 64
      // columns (128 bytes) x 32 rows, 128-byte swizzle.
      const uint64_t dims[2] = {static_cast<uint64_t>(n), static_cast<uint64_t>(m)};
      const uint64_t strides[1] = {static_cast<uint64_t>(n) * 2};
      const uint32_t box[2] = {64, 32};
      rc = encode_tiled(&h->tm_d, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 2, d, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE);
    }
    if (rc == BB_OK) rc = check_cuda(cudaMalloc(&h->status_dev, sizeof(int)), "cudaMalloc(status)");
    if (rc == BB_OK) rc = check_cuda(cudaMemset(h->status_dev, 0, sizeof(int)), "cudaMemset(status)");
    if (rc != BB_OK) {
      if (h->status_dev) cudaFree(h->status_dev);
      delete h;
      return rc;
    }
    Params& p = h->params;
    p.m = static_cast<int32_t>(m);
    p.n = static_cast<int32_t>(n);
    p.k = static_cast<int32_t>(k);
    p.k_stages = static_cast<int32_t>(k / k_step);
    p.rb_m = static_cast<int32_t>(rb_m);
    p.rb_n = static_cast<int32_t>(rb_n);
    p.sfa = static_cast<const uint8_t*>(sfa);
    p.sfb = static_cast<const uint8_t*>(sfb);
    p.global_scale = global_scale;
    p.d = static_cast<__nv_bfloat16*>(d);
    p.status = h->status_dev;
    if (info) {
      info->kind = kind;
      info->tile_m = 128 * h->cg;
      info->tile_n = h->tile_n;
      info->tile_k = k_step;
      info->stages = h->stages;
      info->grid_ctas = h->grid;
      info->num_tiles = p.num_tiles;
      info->smem_bytes = h->smem_bytes;
      info->tmem_columns = TMEM_COLS;
      info->threads_per_cta = kind == BB_LOWP_NVFP4 ? Cfg<kNvfp4, 1>::THREADS : Cfg<kFp8Block, 1>::THREADS;
      info->cta_group = h->cg;
      for (int i = 0; i < 5; ++i) info->reserved[i] = 0;
    }
    *plan = h;
    return BB_OK;
  } catch (...) {
    set_error("bb_lowp_plan_create: unexpected C++ exception");
    return BB_ERR_INTERNAL;
  }
}

BB_API int bb_lowp_execute_n(bb_lowp_plan* plan, int iterations) {
  try {
    if (!plan) {
      set_error("bb_lowp_execute_n: null plan");
      return BB_ERR_ARGUMENT;
    }
    if (iterations < 0) {
      set_error("bb_lowp_execute: negative iteration count %d", iterations);
      return BB_ERR_ARGUMENT;
    }
    for (int i = 0; i < iterations; ++i) {
      int rc = launch(*plan);
      if (rc != BB_OK) return rc;
      ++plan->launches;
      g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    }
    return BB_OK;
  } catch (...) {
    set_error("bb_lowp_execute_n: unexpected C++ exception");
    return BB_ERR_INTERNAL;
  }
}

BB_API int bb_lowp_synchronize(bb_lowp_plan* plan) {
  try {
    if (!plan) {
      set_error("bb_lowp_synchronize: null plan");
      return BB_ERR_ARGUMENT;
    }
    BB_CUDA_TRY(cudaStreamSynchronize(plan->stream));
    int st = 0;
    BB_CUDA_TRY(cudaMemcpy(&st, plan->status_dev, sizeof(int), cudaMemcpyDeviceToHost));
    if (st != 0) {
      set_error("block-scaled GEMM kernel reported device status 0x%x (%s)", st,
                st == 0x200 ? "launch contract violated" : "a bounded wait timed out");
      return st == 0x200 ? BB_ERR_INTERNAL : BB_ERR_TIMEOUT;
    }
    return BB_OK;
  } catch (...) {
    set_error("bb_lowp_synchronize: unexpected C++ exception");
    return BB_ERR_INTERNAL;
  }
}

BB_API int64_t bb_lowp_launches(const bb_lowp_plan* plan) { return plan ? plan->launches : -1; }

BB_API int bb_lowp_destroy(bb_lowp_plan* plan) {
  if (!plan) return BB_OK;
  int rc = BB_OK;
  if (plan->status_dev) {
    cudaError_t e = cudaFree(plan->status_dev);
    if (e != cudaSuccess) rc = check_cuda(e, "cudaFree(status)");
  }
  delete plan;
  return rc;
}

}  // extern "C"
