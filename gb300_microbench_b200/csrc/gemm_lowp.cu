// Block-scaled low-precision GEMMs for sm_100a:
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
// Roles (320 threads, one CTA per SM, 128 x 256 output tile per CTA):
//   warp 0      producer: TMA loads of A (128 x 128 B) and B (256 x 128 B)
//               per K block, plus (NVFP4) bulk copies of the scale atoms.
//   warp 1      TMEM allocation (512 columns) and the single MMA thread.
//   warps 2-9   epilogue: warp w reads TMEM lane quarter w % 4 and column
//               half (w - 2) / 4, converts to BF16 and stores D directly.
//
// Every wait is bounded (globaltimer budget); a timeout records a status
// code, drains what is in flight and returns.
#include <cuda.h>
#include <cuda_bf16.h>

#include <atomic>
#include <new>

#include "common.cuh"
#include "ptx.cuh"

namespace bb {
extern std::atomic<int64_t> g_kernel_launches;

namespace lowp {

enum Kind : int { kNvfp4 = BB_LOWP_NVFP4, kFp8Block = BB_LOWP_FP8_BLOCK128 };

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int ROW_BYTES = 128;               // K bytes of one stage row (one swizzle row)
constexpr int A_BYTES = BM * ROW_BYTES;      // 16 KiB
constexpr int B_BYTES = BN * ROW_BYTES;      // 32 KiB
constexpr int SFA_BYTES = 4 * 512;           // NVFP4: 4 atoms (256 K) x 1 row block
constexpr int SFB_BYTES = 2 * 4 * 512;       // NVFP4: 4 atoms x 2 row blocks
constexpr int STAGES = 4;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr int TMEM_COLS = 512;
constexpr int BAR_BYTES = 256;
constexpr int GROUP_M = 8;

template <int kKind>
struct Cfg {
  static constexpr int K_PER_STAGE = kKind == kNvfp4 ? 256 : 128;  // elements
  static constexpr int MMA_K = kKind == kNvfp4 ? 64 : 32;          // elements per instruction
  static constexpr int MMAS = K_PER_STAGE / MMA_K;                 // 4
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + (kKind == kNvfp4 ? SFA_BYTES + SFB_BYTES : 0);
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + BAR_BYTES;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(MMAS * 32 == ROW_BYTES, "one instruction consumes 32 bytes of each row");
};

// NVFP4 TMEM map: accumulator columns [0, 256); per stage s a scale area at
// 256 + 48 s: SFA of instruction g at +4g (4 columns), SFB at +16 + 8g
// (8 columns: two 128-row atoms). FP8 TMEM map: partial buffer b at 256 b.
constexpr uint32_t kSfBase = 256;
constexpr uint32_t kSfStageCols = 48;
static_assert(kSfBase + STAGES * kSfStageCols <= TMEM_COLS, "TMEM scale ring");

struct Params {
  int32_t m, n, k;
  int32_t tiles_m, tiles_n, num_tiles;
  int32_t k_stages;    // K / K_PER_STAGE
  int32_t k_groups;    // NVFP4: K / 64 (atoms per row block)
  int32_t rb_n;        // NVFP4: 128-row blocks of B's scales
  const uint8_t* sfa;  // NVFP4 atoms, or FP8 FP32 block scales (as bytes)
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

__device__ __forceinline__ void mma_f8(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_nvf4(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t tsfa,
                                         uint32_t tsfb, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(tsfa), "r"(tsfb)
      : "memory");
}
// One 512-byte scale atom (32 rows x 16 bytes) from shared memory into 4
// TMEM columns, replicated into the four 32-lane quarters.
__device__ __forceinline__ void tmem_cp_atom(uint32_t taddr, uint32_t smem_addr) {
  // Interleaved (no-swizzle) K-major layout: 8-row core matrices of 128
  // contiguous bytes, stacked every 128 bytes along the rows (SBO).
  const uint64_t desc = make_smem_desc(smem_addr, 128, 128, kLayoutNone);
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(desc) : "memory");
}
// Non-tensor bulk copy global -> this CTA's shared memory, completing on an
// mbarrier of this CTA.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(mbar)
      : "memory");
}

__device__ __forceinline__ void tile_coords(const Params& p, int t, int& m_blk, int& n_blk) {
  const int group_size = GROUP_M * p.tiles_n;
  const int g = t / group_size;
  const int first_m = g * GROUP_M;
  const int gm = min(GROUP_M, p.tiles_m - first_m);
  const int local = t - g * group_size;
  m_blk = first_m + local % gm;
  n_blk = local / gm;
}

// Converts 32 FP32 accumulator values (scaled by s) to 16 packed BF16 pairs.
__device__ __forceinline__ void pack32(const float* v, float s, uint32_t* out) {
#pragma unroll
  for (int j = 0; j < 16; ++j) out[j] = pack_bf16x2(v[2 * j] * s, v[2 * j + 1] * s);
}

// Stores one row segment of 128 BF16 (64 packed words) at (row, col0).
__device__ __forceinline__ void store_row(const Params& p, int row, int col0, const uint32_t (&pk)[64]) {
  if (row >= p.m) return;
  __nv_bfloat16* dst = p.d + static_cast<int64_t>(row) * p.n + col0;
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    const int col = col0 + 8 * c;
    if (col + 8 <= p.n) {
      *reinterpret_cast<uint4*>(dst + 8 * c) = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (col + e < p.n) {
          const uint32_t w = pk[4 * c + e / 2];
          const uint16_t bits = static_cast<uint16_t>((e & 1) ? (w >> 16) : (w & 0xFFFFu));
          reinterpret_cast<uint16_t*>(dst)[8 * c + e] = bits;
        }
      }
    }
  }
}

template <int kKind>
__global__ void __launch_bounds__(THREADS, 1)
    bb_lowp_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        const Params p) {
  using C = Cfg<kKind>;
  if (blockDim.x != THREADS) {
    if (threadIdx.x == 0 && p.status) atomicCAS(p.status, 0, kDevBadLaunch);
    return;
  }
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem_a + STAGES * A_BYTES;
  uint8_t* smem_sfa = smem_b + STAGES * B_BYTES;          // NVFP4 only
  uint8_t* smem_sfb = smem_sfa + STAGES * SFA_BYTES;      // NVFP4 only
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;       // [2]
  uint64_t* acc_empty = bars + 2 * STAGES + 2;  // [2]
  uint64_t* mma_done = bars + 2 * STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;

  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
  }
  if (warp == 1 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_empty[b]), EPI_WARPS);
    }
    mbar_init(smem_u32(mma_done), 1);
    fence_mbarrier_init_cluster();
  }
  if (warp == 1) {
    tmem_alloc<1>(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish<1>();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
        int m_blk, n_blk;
        tile_coords(p, t, m_blk, n_blk);
        const int rb_b = 2 * n_blk;  // first 128-row block of B's scales
        const int sfb_blocks = kKind == kNvfp4 ? min(2, p.rb_n - rb_b) : 0;
        for (int ks = 0; ks < p.k_stages; ++ks) {
          if (!bb_wait(smem_u32(&empty[stage]), phase ^ 1u, p.status, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full[stage]);
          uint32_t bytes = A_BYTES + B_BYTES;
          if constexpr (kKind == kNvfp4) bytes += SFA_BYTES + sfb_blocks * (SFB_BYTES / 2);
          mbar_arrive_expect_tx(fb, bytes);
          tma_load_2d(smem_u32(smem_a + stage * A_BYTES), &tm_a, fb, ks * ROW_BYTES, m_blk * BM);
          tma_load_2d(smem_u32(smem_b + stage * B_BYTES), &tm_b, fb, ks * ROW_BYTES, n_blk * BN);
          if constexpr (kKind == kNvfp4) {
            const int64_t kg0 = static_cast<int64_t>(ks) * 4;
            bulk_load(smem_u32(smem_sfa + stage * SFA_BYTES),
                      p.sfa + (static_cast<int64_t>(m_blk) * p.k_groups + kg0) * 512, SFA_BYTES, fb);
            for (int r = 0; r < sfb_blocks; ++r)
              bulk_load(smem_u32(smem_sfb + stage * SFB_BYTES + r * (SFB_BYTES / 2)),
                        p.sfb + (static_cast<int64_t>(rb_b + r) * p.k_groups + kg0) * 512, SFB_BYTES / 2, fb);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (ok) {
        for (int i = 0; i < STAGES; ++i) {
          if (!bb_wait(smem_u32(&empty[stage]), phase ^ 1u, p.status, kDevTimeoutProducer)) break;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      } else {
        bounded_sleep_ns(2000000);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_iter = 0;  // NVFP4: tiles; FP8: K blocks (partial buffers)
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
        if constexpr (kKind == kNvfp4) {
          if (!bb_wait(smem_u32(&acc_empty[0]), (acc_iter & 1u) ^ 1u, p.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        for (int ks = 0; ks < p.k_stages; ++ks) {
          uint32_t d_tmem = tmem_base;
          uint32_t buf = 0;
          if constexpr (kKind == kFp8Block) {
            buf = acc_iter & 1u;
            if (!bb_wait(smem_u32(&acc_empty[buf]), ((acc_iter >> 1) & 1u) ^ 1u, p.status, kDevTimeoutMma)) {
              ok = false;
              break;
            }
            d_tmem = tmem_base + buf * 256u;
          }
          if (!bb_wait(smem_u32(&full[stage]), phase, p.status, kDevTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem_a + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(smem_b + stage * B_BYTES);
          if constexpr (kKind == kNvfp4) {
            const uint32_t sf_cols = tmem_base + kSfBase + stage * kSfStageCols;
            const uint32_t sfa_s = smem_u32(smem_sfa + stage * SFA_BYTES);
            const uint32_t sfb_s = smem_u32(smem_sfb + stage * SFB_BYTES);
#pragma unroll
            for (int g = 0; g < C::MMAS; ++g) {
              tmem_cp_atom(sf_cols + 4 * g, sfa_s + g * 512);
              tmem_cp_atom(sf_cols + 16 + 8 * g, sfb_s + g * 512);
              tmem_cp_atom(sf_cols + 16 + 8 * g + 4, sfb_s + SFB_BYTES / 2 + g * 512);
            }
            constexpr uint32_t idesc = idesc_nvf4(BM, BN);
#pragma unroll
            for (int g = 0; g < C::MMAS; ++g) {
              mma_nvf4(d_tmem, sw128_kmajor_desc(a_addr + g * 32), sw128_kmajor_desc(b_addr + g * 32), idesc,
                       sf_cols + 4 * g, sf_cols + 16 + 8 * g, (ks != 0 || g != 0) ? 1u : 0u);
            }
          } else {
            constexpr uint32_t idesc = idesc_f8(BM, BN);
#pragma unroll
            for (int g = 0; g < C::MMAS; ++g) {
              mma_f8(d_tmem, sw128_kmajor_desc(a_addr + g * 32), sw128_kmajor_desc(b_addr + g * 32), idesc,
                     g != 0 ? 1u : 0u);
            }
          }
          umma_commit<1>(smem_u32(&empty[stage]));
          if constexpr (kKind == kFp8Block) {
            umma_commit<1>(smem_u32(&acc_full[buf]));
            ++acc_iter;
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (kKind == kNvfp4) {
          umma_commit<1>(smem_u32(&acc_full[0]));
          ++acc_iter;
        }
      }
      umma_commit<1>(smem_u32(mma_done));
      bb_wait(smem_u32(mma_done), 0, p.status, kDevTimeoutMma, /*honor_abort=*/false);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int half = (warp - 2) / 4;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    uint32_t acc_iter = 0;
    bool ok = true;
    auto release = [&](uint32_t buf) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&acc_empty[buf]));
    };
    for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
      int m_blk, n_blk;
      tile_coords(p, t, m_blk, n_blk);
      const int row = m_blk * BM + q * 32 + lane;
      const int col0 = n_blk * BN + half * 128;
      uint32_t pk[64];
      if constexpr (kKind == kNvfp4) {
        if (!bb_wait(smem_u32(&acc_full[0]), acc_iter & 1u, p.status, kDevTimeoutEpilogue)) break;
        tc_fence_after();
        const uint32_t taddr = tmem_base + lane_off + half * 128;
#pragma unroll
        for (int c = 0; c < 4; c += 2) {
          uint32_t r0[32], r1[32];
          tmem_ld_32x32b_x32(taddr + 32 * c, r0);
          tmem_ld_32x32b_x32(taddr + 32 * (c + 1), r1);
          tmem_ld_wait();
          pack32(reinterpret_cast<const float*>(r0), p.global_scale, pk + 16 * c);
          pack32(reinterpret_cast<const float*>(r1), p.global_scale, pk + 16 * (c + 1));
        }
        release(0);
        ++acc_iter;
      } else {
        const float* sa = reinterpret_cast<const float*>(p.sfa);
        const float* sb = reinterpret_cast<const float*>(p.sfb);
        const int rb_n = (p.n + 127) / 128;
        const int nb = min(2 * n_blk + half, rb_n - 1);  // ragged N: columns past N are never stored
        const float* sa_row = sa + static_cast<int64_t>(m_blk) * p.k_stages;
        const float* sb_row = sb + static_cast<int64_t>(nb) * p.k_stages;
        float acc[128];
#pragma unroll
        for (int j = 0; j < 128; ++j) acc[j] = 0.f;
        float s_next = __ldg(sa_row) * __ldg(sb_row);
        for (int ks = 0; ks < p.k_stages; ++ks) {
          const float s = s_next;
          if (ks + 1 < p.k_stages) s_next = __ldg(sa_row + ks + 1) * __ldg(sb_row + ks + 1);
          const uint32_t buf = acc_iter & 1u;
          if (!bb_wait(smem_u32(&acc_full[buf]), (acc_iter >> 1) & 1u, p.status, kDevTimeoutEpilogue)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t taddr = tmem_base + lane_off + buf * 256u + half * 128;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t r0[32];
            tmem_ld_32x32b_x32(taddr + 32 * c, r0);
            tmem_ld_wait();
            if (c == 3) release(buf);
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[32 * c + j] = fmaf(__uint_as_float(r0[j]), s, acc[32 * c + j]);
          }
          ++acc_iter;
        }
        if (!ok) break;
#pragma unroll
        for (int c = 0; c < 4; ++c) pack32(acc + 32 * c, p.global_scale, pk + 16 * c);
      }
      store_row(p, row, col0, pk);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<1>(tmem_base, TMEM_COLS);
  }
}

}  // namespace lowp
}  // namespace bb

struct bb_lowp_plan {
  int kind = 0;
  int64_t m = 0, n = 0, k = 0;
  const void* a = nullptr;
  const void* b = nullptr;
  const void* sfa = nullptr;
  const void* sfb = nullptr;
  void* d = nullptr;
  cudaStream_t stream = nullptr;
  CUtensorMap tm_a{}, tm_b{};
  bb::lowp::Params params{};
  int grid = 0;
  int smem_bytes = 0;
  int* status_dev = nullptr;
  int64_t launches = 0;
};

using namespace bb;
using namespace bb::lowp;

namespace {

template <int kKind>
int launch_kind(const bb_lowp_plan& pl) {
  auto kern = bb_lowp_gemm_kernel<kKind>;
  static bool attr_set = false;  // one attribute call per kernel and process
  if (!attr_set) {
    BB_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<kKind>::SMEM_BYTES));
    attr_set = true;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = Cfg<kKind>::SMEM_BYTES;
  cfg.stream = pl.stream;
  cfg.numAttrs = 0;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, pl.tm_a, pl.tm_b, pl.params), "launch bb_lowp_gemm_kernel");
}

int launch(const bb_lowp_plan& pl) {
  return pl.kind == kNvfp4 ? launch_kind<kNvfp4>(pl) : launch_kind<kFp8Block>(pl);
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
    if (m <= 0 || n <= 0 || k <= 0 || m > (int64_t(1) << 31) || n > (int64_t(1) << 31) || k > (int64_t(1) << 31)) {
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
    h->a = a;
    h->b = b;
    h->sfa = sfa;
    h->sfb = sfb;
    h->d = d;
    h->stream = static_cast<cudaStream_t>(stream);
    // Operands are byte arrays: K / 2 bytes per row for E2M1, K for E4M3.
    const uint64_t row_bytes = kind == BB_LOWP_NVFP4 ? k / 2 : k;
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
      const uint32_t box[2] = {ROW_BYTES, BN};
      rc = encode_tiled(&h->tm_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, 2, b, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
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
    p.tiles_m = static_cast<int32_t>((m + BM - 1) / BM);
    p.tiles_n = static_cast<int32_t>((n + BN - 1) / BN);
    p.num_tiles = p.tiles_m * p.tiles_n;
    p.k_stages = static_cast<int32_t>(k / k_step);
    p.k_groups = static_cast<int32_t>(k / 64);
    p.rb_n = static_cast<int32_t>((n + 127) / 128);
    p.sfa = static_cast<const uint8_t*>(sfa);
    p.sfb = static_cast<const uint8_t*>(sfb);
    p.global_scale = global_scale;
    p.d = static_cast<__nv_bfloat16*>(d);
    p.status = h->status_dev;
    h->grid = p.num_tiles < dev.sm_count ? p.num_tiles : dev.sm_count;
    h->smem_bytes = kind == BB_LOWP_NVFP4 ? Cfg<kNvfp4>::SMEM_BYTES : Cfg<kFp8Block>::SMEM_BYTES;
    if (info) {
      info->kind = kind;
      info->tile_m = BM;
      info->tile_n = BN;
      info->tile_k = k_step;
      info->stages = STAGES;
      info->grid_ctas = h->grid;
      info->num_tiles = p.num_tiles;
      info->smem_bytes = h->smem_bytes;
      info->tmem_columns = TMEM_COLS;
      info->threads_per_cta = THREADS;
      for (int i = 0; i < 6; ++i) info->reserved[i] = 0;
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
