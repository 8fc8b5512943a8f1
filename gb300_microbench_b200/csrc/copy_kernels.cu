// HBM -> shared-memory streaming kernels for sm_100a: the LDGSTS
// (cp.async.cg, 16-byte) arm and the 2D TMA (cp.async.bulk.tensor) arm of
// the reference's memory-path experiment (memory_paths/ldgsts.cu,
// memory_paths/tma.cu), with their C ABI.
//
// Work decomposition (both arms): the buffer is cut into tiles of
// stage_bytes; CTA i of G owns the contiguous tile range
// [i*T/G, (i+1)*T/G). One CTA runs per SM (the shared-memory reservation is
// larger than half an SM), so bytes in flight per SM = stages * stage_bytes.
//
// LDGSTS arm: 128 threads; thread t copies vectors t, t+128, ... of every
// tile with cp.async.cg into a STAGES-deep ring and later XORs exactly the
// vectors it copied itself. Because no thread reads another thread's
// copies, cp.async.wait_group alone orders copy and use: the ring needs no
// CTA-wide barrier (the reference synchronises the CTA twice per tile,
// ldgsts.cu:356-359).
//
// TMA arm: a producer warp issues one 2D tensor copy per stage (box =
// tile_rows x row_bytes) against a full mbarrier with expect_tx; four
// consumer warps wait on it, XOR the tile and release the slot through an
// empty mbarrier (one arrival per warp). The reference instead lets one of
// the 128 consumer threads issue and uses __syncthreads for slot reuse
// (tma.cu:578-586).
//
// Every CTA writes one 32-bit checksum: the XOR of all words it read in
// pass 0, XORed with pass p's checksum rotated left by p % 32.
#include <cuda.h>

#include <atomic>

#include <cstdlib>

#include "common.cuh"
#include "ptx.cuh"

namespace bb {
extern std::atomic<int64_t> g_kernel_launches;

namespace copy {

constexpr int kLdgstsThreads = 128;
constexpr int kTmaConsumerThreads = 128;
constexpr int kTmaThreads = kTmaConsumerThreads + 32;
constexpr int kTmaMaxVecPerThread = 32768 / 16 / kTmaConsumerThreads;  // stages of at most 32 KiB
constexpr uint64_t kPatternSalt = 0xD1B54A32D192ED03ull;

// SplitMix64 finaliser (the pattern generator of ldgsts.cu:220-232).
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t x) {
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__device__ __forceinline__ uint4 pattern_vector(uint64_t i) {
  const uint64_t lo = mix64(i);
  const uint64_t hi = mix64(i ^ kPatternSalt);
  return make_uint4(static_cast<uint32_t>(lo), static_cast<uint32_t>(lo >> 32), static_cast<uint32_t>(hi),
                    static_cast<uint32_t>(hi >> 32));
}

__device__ __forceinline__ uint32_t rotl32(uint32_t x, int r) {
  r &= 31;
  return r == 0 ? x : ((x << r) | (x >> (32 - r)));
}

__device__ __forceinline__ void cta_range(int64_t total_tiles, int64_t& t0, int64_t& n) {
  const int64_t g = gridDim.x;
  t0 = (static_cast<int64_t>(blockIdx.x) * total_tiles) / g;
  const int64_t t1 = (static_cast<int64_t>(blockIdx.x + 1) * total_tiles) / g;
  n = t1 - t0;
}

// XOR-reduce one 32-bit value per thread over the CTA; thread 0 gets it.
template <int kThreads>
__device__ __forceinline__ uint32_t cta_xor(uint32_t v, uint32_t* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v ^= __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x / 32;
  if ((threadIdx.x & 31) == 0 && warp < kThreads / 32) scratch[warp] = v;
  __syncthreads();
  uint32_t r = 0;
  if (threadIdx.x == 0) {
    for (int w = 0; w < kThreads / 32; ++w) r ^= scratch[w];
  }
  return r;
}

// ------------------------------------------------------------------ LDGSTS
template <int STAGES, int COPIES, bool VALIDATE>
__device__ __forceinline__ void ldgsts_body(const uint4* __restrict__ src, int64_t total_vec, int64_t total_tiles,
                                            int64_t passes, int64_t rotation, uint32_t* __restrict__ sink,
                                            unsigned long long* __restrict__ mismatches, int pipe) {
  constexpr int kVecPerTile = kLdgstsThreads * COPIES;
  constexpr int kStageBytes = kVecPerTile * 16;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint32_t red[4];
  const int tid = threadIdx.x;
  int64_t t0, n;
  cta_range(total_tiles, t0, n);
  uint32_t total = 0;
  unsigned long long bad = 0;
  const uint32_t zmask = static_cast<uint32_t>(total_vec >> 62);  // 0 for every real buffer
  if (n > 0) {
    for (int64_t p = 0; p < passes; ++p) {
      const int64_t rot = (rotation + p) % n;
      uint4 acc = make_uint4(0, 0, 0, 0);
      auto tile_of = [&](int64_t s) {
        int64_t i = rot + s;
        if (i >= n) i -= n;
        return t0 + i;
      };
      auto issue = [&](int64_t s) {
        const int64_t vbase = tile_of(s) * kVecPerTile;
        const uint32_t slot = smem_u32(smem + (s % STAGES) * kStageBytes);
#pragma unroll
        for (int c = 0; c < COPIES; ++c) {
          const int v = tid + c * kLdgstsThreads;
          if (vbase + v < total_vec) {
            cp_async_16(slot + v * 16, src + vbase + v);
          }
        }
      };
      // Consumes tile s and refills its slot with tile s + STAGES: this
      // thread's vectors of the slot are loaded into registers first, then
      // the whole refill is issued at once (one burst per stage, as the
      // stage issue itself), and only then are the values XORed, so STAGES
      // tiles stay in flight while a tile is reduced (never more: the slot
      // is refilled only after it was read). Each thread reads and rewrites
      // only the positions it copied itself; the refill's shared addresses
      // carry a data dependence on the values read (AND with a zero the
      // compiler cannot see), so no refill can issue before its reads
      // returned.
      auto consume = [&](int64_t s) {
        const int64_t vbase = tile_of(s) * kVecPerTile;
        const uint4* slot = reinterpret_cast<const uint4*>(smem + (s % STAGES) * kStageBytes);
#pragma unroll
        for (int c = 0; c < COPIES; ++c) {
          const int v = tid + c * kLdgstsThreads;
          if (vbase + v < total_vec) {
            const uint4 x = slot[v];
            acc.x ^= x.x;
            acc.y ^= x.y;
            acc.z ^= x.z;
            acc.w ^= x.w;
            if constexpr (VALIDATE) {
              const uint4 e = pattern_vector(static_cast<uint64_t>(vbase + v));
              bad += (x.x != e.x || x.y != e.y || x.z != e.z || x.w != e.w) ? 1 : 0;
            }
          }
        }
      };
      auto consume_refill = [&](int64_t s) {
        const int64_t vbase = tile_of(s) * kVecPerTile;
        const bool refill = s + STAGES < n;
        const int64_t nbase = refill ? tile_of(s + STAGES) * kVecPerTile : 0;
        const uint32_t slot_u32 = smem_u32(smem + (s % STAGES) * kStageBytes);
        const uint4* slot = reinterpret_cast<const uint4*>(smem + (s % STAGES) * kStageBytes);
        uint4 x[COPIES];
        uint32_t dep = 0;
#pragma unroll
        for (int c = 0; c < COPIES; ++c) {
          const int v = tid + c * kLdgstsThreads;
          x[c] = (vbase + v < total_vec) ? slot[v] : make_uint4(0, 0, 0, 0);
          dep |= x[c].x;
        }
        dep &= zmask;
        if (refill) {
#pragma unroll
          for (int c = 0; c < COPIES; ++c) {
            const int v = tid + c * kLdgstsThreads;
            if (nbase + v < total_vec) {
              cp_async_16(slot_u32 + v * 16 + dep, src + nbase + v);
            }
          }
        }
#pragma unroll
        for (int c = 0; c < COPIES; ++c) {
          const int v = tid + c * kLdgstsThreads;
          if (vbase + v < total_vec) {
            acc.x ^= x[c].x;
            acc.y ^= x[c].y;
            acc.z ^= x[c].z;
            acc.w ^= x[c].w;
            if constexpr (VALIDATE) {
              const uint4 e = pattern_vector(static_cast<uint64_t>(vbase + v));
              bad += (x[c].x != e.x || x[c].y != e.y || x[c].z != e.z || x[c].w != e.w) ? 1 : 0;
            }
          }
        }
      };
      if (pipe & 1) {
        // Refill form: STAGES tiles in flight while one is reduced.
        for (int64_t s = 0; s < STAGES; ++s) {
          if (s < n) issue(s);
          cp_async_commit();  // possibly empty: keeps the group count uniform
        }
        for (int64_t s = 0; s < n; ++s) {
          cp_async_wait<STAGES - 1>();
          consume_refill(s);
          cp_async_commit();
        }
      } else {
        // Classic form (the reference's order): tile s is issued into the
        // slot freed by the previous reduction, then tile s - STAGES + 1 is
        // waited for and reduced in place.
        for (int64_t s = 0; s < n + STAGES - 1; ++s) {
          if (s < n) issue(s);
          cp_async_commit();  // possibly empty: keeps the group count uniform
          if (s >= STAGES - 1) {
            cp_async_wait<STAGES - 1>();
            consume(s - (STAGES - 1));
          }
        }
      }
      cp_async_wait<0>();
      total ^= rotl32(acc.x ^ acc.y ^ acc.z ^ acc.w, static_cast<int>(p));
    }
  }
  const uint32_t cs = cta_xor<kLdgstsThreads>(total, red);
  if (tid == 0) sink[blockIdx.x] = cs;
  if constexpr (VALIDATE) {
    if (bad) atomicAdd(mismatches, bad);
  }
}

// Kernel names match the reference's (ncu_capture.py filters on the
// function base name "ldgsts_benchmark_kernel" / "tma_benchmark_kernel").
template <int STAGES, int COPIES>
__global__ void __launch_bounds__(kLdgstsThreads, 1)
    ldgsts_benchmark_kernel(const uint4* __restrict__ src, int64_t total_vec, int64_t total_tiles, int64_t passes,
                            int64_t rotation, uint32_t* __restrict__ sink, int pipe) {
  ldgsts_body<STAGES, COPIES, false>(src, total_vec, total_tiles, passes, rotation, sink, nullptr, pipe);
}

template <int STAGES, int COPIES>
__global__ void __launch_bounds__(kLdgstsThreads, 1)
    ldgsts_validate_kernel(const uint4* __restrict__ src, int64_t total_vec, int64_t total_tiles,
                           uint32_t* __restrict__ sink, unsigned long long* __restrict__ mismatches) {
  ldgsts_body<STAGES, COPIES, true>(src, total_vec, total_tiles, 1, 0, sink, mismatches, 1);
}

// ------------------------------------------------------------------ TMA
template <int STAGES, bool VALIDATE>
__device__ __forceinline__ void tma_body(const CUtensorMap* tmap, int64_t total_vec, int64_t total_tiles,
                                         int stage_bytes, int tile_rows, int64_t passes, int64_t rotation,
                                         uint32_t* __restrict__ sink, unsigned long long* __restrict__ mismatches,
                                         int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[STAGES];
  __shared__ __align__(8) uint64_t empty[STAGES];
  __shared__ uint32_t red[4];
  const int tid = threadIdx.x;
  const int warp = tid / 32;
  const int lane = tid % 32;
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), kTmaConsumerThreads / 32);
    }
    fence_mbarrier_init_cluster();
  }
  __syncthreads();
  int64_t t0, n;
  cta_range(total_tiles, t0, n);
  const int vec_per_tile = stage_bytes / 16;
  const uint32_t zmask = static_cast<uint32_t>(total_vec >> 62);  // 0 for every real buffer
  uint32_t total = 0;
  unsigned long long bad = 0;

  if (warp == kTmaConsumerThreads / 32) {
    // ---------------------------------------------------------- producer
    if (lane == 0 && n > 0) {
      prefetch_tmap(tmap);
      bool ok = true;
      int stage = 0;
      uint32_t phase = 0;
      for (int64_t p = 0; p < passes && ok; ++p) {
        const int64_t rot = (rotation + p) % n;
        for (int64_t s = 0; s < n; ++s) {
          if (!bb_wait(smem_u32(&empty[stage]), phase ^ 1u, status, kDevTimeoutProducer)) {
            ok = false;
            break;
          }
          int64_t i = rot + s;
          if (i >= n) i -= n;
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_arrive_expect_tx(fb, static_cast<uint32_t>(stage_bytes));
          tma_load_2d(smem_u32(smem + stage * stage_bytes), tmap, fb, 0, static_cast<int32_t>((t0 + i) * tile_rows));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) bounded_sleep_ns(2000000);
    }
  } else {
    // ---------------------------------------------------------- consumers
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int64_t p = 0; p < passes && ok && n > 0; ++p) {
      const int64_t rot = (rotation + p) % n;
      uint4 acc = make_uint4(0, 0, 0, 0);
      for (int64_t s = 0; s < n; ++s) {
        if (!bb_wait(smem_u32(&full[stage]), phase, status, kDevTimeoutConsumer)) {
          ok = false;
          break;
        }
        int64_t i = rot + s;
        if (i >= n) i -= n;
        const int64_t vbase = (t0 + i) * vec_per_tile;
        const uint4* slot = reinterpret_cast<const uint4*>(smem + stage * stage_bytes);
        // This thread's vectors (at most kTmaMaxVecPerThread) into registers;
        // the slot is released as soon as they have arrived (the OR below
        // waits for every load), and the XOR runs after the release.
        uint4 x[kTmaMaxVecPerThread];
        uint32_t arrived = 0;
#pragma unroll
        for (int c = 0; c < kTmaMaxVecPerThread; ++c) {
          const int v = tid + c * kTmaConsumerThreads;
          x[c] = (v < vec_per_tile && vbase + v < total_vec) ? slot[v] : make_uint4(0, 0, 0, 0);
          arrived |= x[c].x;
        }
        // The mask carries a data dependence on every loaded value (OR-ed,
        // then AND-ed with a zero the compiler cannot see), so the warp
        // barrier, and the release after it, wait for all of the loads.
        __syncwarp(0xffffffffu | (arrived & zmask));
        if (lane == 0) mbar_arrive(smem_u32(&empty[stage]));
#pragma unroll
        for (int c = 0; c < kTmaMaxVecPerThread; ++c) {
          const int v = tid + c * kTmaConsumerThreads;
          acc.x ^= x[c].x;
          acc.y ^= x[c].y;
          acc.z ^= x[c].z;
          acc.w ^= x[c].w;
          if constexpr (VALIDATE) {
            if (v < vec_per_tile && vbase + v < total_vec) {
              const uint4 e = pattern_vector(static_cast<uint64_t>(vbase + v));
              bad += (x[c].x != e.x || x[c].y != e.y || x[c].z != e.z || x[c].w != e.w) ? 1 : 0;
            }
          }
        }
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      total ^= rotl32(acc.x ^ acc.y ^ acc.z ^ acc.w, static_cast<int>(p));
    }
  }
  const uint32_t cs = cta_xor<kTmaConsumerThreads>(warp < kTmaConsumerThreads / 32 ? total : 0u, red);
  if (tid == 0) sink[blockIdx.x] = cs;
  if constexpr (VALIDATE) {
    if (bad) atomicAdd(mismatches, bad);
  }
}

template <int STAGES>
__global__ void __launch_bounds__(kTmaThreads, 1)
    tma_benchmark_kernel(const __grid_constant__ CUtensorMap tmap, int64_t total_vec, int64_t total_tiles,
                         int stage_bytes, int tile_rows, int64_t passes, int64_t rotation,
                         uint32_t* __restrict__ sink, int* status) {
  tma_body<STAGES, false>(&tmap, total_vec, total_tiles, stage_bytes, tile_rows, passes, rotation, sink, nullptr,
                          status);
}

template <int STAGES>
__global__ void __launch_bounds__(kTmaThreads, 1)
    tma_validate_kernel(const __grid_constant__ CUtensorMap tmap, int64_t total_vec, int64_t total_tiles,
                        int stage_bytes, int tile_rows, uint32_t* __restrict__ sink,
                        unsigned long long* __restrict__ mismatches, int* status) {
  tma_body<STAGES, true>(&tmap, total_vec, total_tiles, stage_bytes, tile_rows, 1, 0, sink, mismatches, status);
}

// ------------------------------------------------------------------ fills
__global__ void fill_pattern_kernel(uint4* __restrict__ dst, int64_t nvec) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    dst[i] = pattern_vector(static_cast<uint64_t>(i));
  }
}

__global__ void fill_uniform_u32_kernel(uint32_t* __restrict__ dst, int64_t nwords, uint64_t seed) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const uint64_t base = seed * 0x9E3779B97F4A7C15ull;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nwords; i += stride) {
    dst[i] = static_cast<uint32_t>(mix64(base + static_cast<uint64_t>(i)));
  }
}

// ------------------------------------------------------------------ host
struct Geometry {
  int stages = 0;
  int stage_bytes = 0;
  int copies = 0;
  int row_bytes = 0;
  int tile_rows = 0;
  int threads = 0;
  int smem = 0;
  int grid = 0;
  int occupancy = 0;  // resident CTAs per SM of the benchmark kernel (0: not queried)
  int64_t total_tiles = 0;
};

static int geometry(int method, int stages, int bif_kib, int row_bytes, int64_t bytes, int sm_count, Geometry* g) {
  if (method != BB_COPY_LDGSTS && method != BB_COPY_TMA) {
    set_error("copy: unknown method %d", method);
    return BB_ERR_ARGUMENT;
  }
  if (stages != 2 && stages != 3 && stages != 4 && stages != 8) {
    set_error("copy: stages must be 2, 3, 4 or 8 (got %d)", stages);
    return BB_ERR_ARGUMENT;
  }
  if (bif_kib != 16 && bif_kib != 32 && bif_kib != 64) {
    set_error("copy: bytes in flight must be 16, 32 or 64 KiB (got %d)", bif_kib);
    return BB_ERR_ARGUMENT;
  }
  if (bytes <= 0 || bytes % 16 != 0) {
    set_error("copy: byte count %lld must be positive and a multiple of 16", (long long)bytes);
    return BB_ERR_ARGUMENT;
  }
  const int raw = bif_kib * 1024 / stages;
  g->stages = stages;
  if (method == BB_COPY_LDGSTS) {
    g->copies = raw / (kLdgstsThreads * 16);
    g->stage_bytes = g->copies * kLdgstsThreads * 16;
    g->row_bytes = 256;
    g->tile_rows = g->stage_bytes / 256;
    g->threads = kLdgstsThreads;
  } else {
    if (row_bytes != 128 && row_bytes != 256) {
      set_error("copy: TMA row width must be 128 or 256 bytes (got %d)", row_bytes);
      return BB_ERR_ARGUMENT;
    }
    if (bytes % row_bytes != 0) {
      set_error("copy: TMA byte count %lld must be a multiple of the %d-byte row", (long long)bytes, row_bytes);
      return BB_ERR_ARGUMENT;
    }
    g->row_bytes = row_bytes;
    g->tile_rows = raw / row_bytes;
    if (g->tile_rows > 256) g->tile_rows = 256;
    g->stage_bytes = g->tile_rows * row_bytes;
    g->copies = 0;
    g->threads = kTmaThreads;
  }
  g->total_tiles = (bytes + g->stage_bytes - 1) / g->stage_bytes;
  g->grid = sm_count;
  return BB_OK;
}

static int finish_geometry(Geometry* g, int* sm_count_out) {
  DeviceInfo dev;
  int rc = query_device(&dev);
  if (rc != BB_OK) return rc;
  if (g->grid <= 0) g->grid = dev.sm_count;
  // Strictly more than half an SM's shared memory: at most one CTA per SM.
  int half_plus = dev.smem_per_sm / 2 + 1;
  half_plus = (half_plus + 127) / 128 * 128;
  const int payload = g->stages * g->stage_bytes;
  g->smem = payload > half_plus ? payload : half_plus;
  if (g->smem > dev.smem_optin) {
    set_error("copy: shared-memory reservation %d exceeds the opt-in maximum %d", g->smem, dev.smem_optin);
    return BB_ERR_ARGUMENT;
  }
  if (sm_count_out) *sm_count_out = dev.sm_count;
  return BB_OK;
}

template <typename K>
static int occupancy_of(K kern, int threads, int smem, int* out) {
  int rc = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                      "cudaFuncSetAttribute(copy smem)");
  if (rc != BB_OK) return rc;
  return check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(out, kern, threads, smem),
                    "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
}

// Resident CTAs per SM of the benchmark kernel of this geometry (the
// reference checks it is exactly 1: ldgsts.cu:821-835).
static int query_occupancy(int method, Geometry* g);

template <typename K>
static int set_smem(K kern, int smem) {
  return check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                    "cudaFuncSetAttribute(copy smem)");
}

#define BB_LDGSTS_CASES(X) \
  X(2, 4) X(2, 8) X(2, 16) X(3, 2) X(3, 5) X(3, 10) X(4, 2) X(4, 4) X(4, 8) X(8, 1) X(8, 2) X(8, 4)

// LDGSTS pipeline form: the refill form (1) keeps every stage in flight
// while one is reduced and wins where stages are small (2-4 KiB: 8 x 16 KiB
// 2112 -> 3173 GB/s, 4 x 16 KiB 3449 -> 3536 on one box); with larger
// stages the classic form (0) streams faster (4 x 64 KiB 6990 against 5191).
// BB_COPY_PIPE=0|1 overrides.
static int ldgsts_pipe(const Geometry& g) {
  if (const char* e = std::getenv("BB_COPY_PIPE")) return std::atoi(e) != 0 ? 1 : 0;
  return g.stage_bytes <= 4096 ? 1 : 0;
}

static int launch_ldgsts(const Geometry& g, bool validate, const void* src, int64_t bytes, int64_t passes,
                         int64_t rotation, uint32_t* sink, unsigned long long* mism, cudaStream_t st) {
  const int64_t nvec = bytes / 16;
  const uint4* s = static_cast<const uint4*>(src);
#define X(S, C)                                                                                         \
  if (g.stages == S && g.copies == C) {                                                                 \
    if (validate) {                                                                                     \
      int rc = set_smem(ldgsts_validate_kernel<S, C>, g.smem);                                          \
      if (rc != BB_OK) return rc;                                                                       \
      ldgsts_validate_kernel<S, C><<<g.grid, kLdgstsThreads, g.smem, st>>>(s, nvec, g.total_tiles, sink, mism); \
    } else {                                                                                            \
      int rc = set_smem(ldgsts_benchmark_kernel<S, C>, g.smem);                                         \
      if (rc != BB_OK) return rc;                                                                       \
      ldgsts_benchmark_kernel<S, C><<<g.grid, kLdgstsThreads, g.smem, st>>>(s, nvec, g.total_tiles, passes, \
                                                                            rotation, sink, ldgsts_pipe(g)); \
    }                                                                                                   \
    return check_cuda(cudaGetLastError(), "ldgsts launch");                                             \
  }
  BB_LDGSTS_CASES(X)
#undef X
  set_error("copy: no LDGSTS specialisation for stages=%d copies=%d", g.stages, g.copies);
  return BB_ERR_INTERNAL;
}

static int launch_tma(const Geometry& g, bool validate, const void* src, int64_t bytes, int64_t passes,
                      int64_t rotation, uint32_t* sink, unsigned long long* mism, int* status, cudaStream_t st) {
  CUtensorMap tmap;
  const uint64_t dims[2] = {static_cast<uint64_t>(g.row_bytes / 4), static_cast<uint64_t>(bytes / g.row_bytes)};
  const uint64_t strides[1] = {static_cast<uint64_t>(g.row_bytes)};
  const uint32_t box[2] = {static_cast<uint32_t>(g.row_bytes / 4), static_cast<uint32_t>(g.tile_rows)};
  int rc = encode_tiled(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, 2, src, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE);
  if (rc != BB_OK) return rc;
  const int64_t nvec = bytes / 16;
#define X(S)                                                                                             \
  if (g.stages == S) {                                                                                   \
    if (validate) {                                                                                      \
      rc = set_smem(tma_validate_kernel<S>, g.smem);                                                     \
      if (rc != BB_OK) return rc;                                                                        \
      tma_validate_kernel<S><<<g.grid, kTmaThreads, g.smem, st>>>(tmap, nvec, g.total_tiles, g.stage_bytes, \
                                                                  g.tile_rows, sink, mism, status);      \
    } else {                                                                                             \
      rc = set_smem(tma_benchmark_kernel<S>, g.smem);                                                    \
      if (rc != BB_OK) return rc;                                                                        \
      tma_benchmark_kernel<S><<<g.grid, kTmaThreads, g.smem, st>>>(tmap, nvec, g.total_tiles, g.stage_bytes, \
                                                                   g.tile_rows, passes, rotation, sink, status); \
    }                                                                                                    \
    return check_cuda(cudaGetLastError(), "tma launch");                                                 \
  }
  X(2) X(3) X(4) X(8)
#undef X
  set_error("copy: no TMA specialisation for stages=%d", g.stages);
  return BB_ERR_INTERNAL;
}

static int query_occupancy(int method, Geometry* g) {
  if (method == BB_COPY_LDGSTS) {
#define X(S, C) \
  if (g->stages == S && g->copies == C) return occupancy_of(ldgsts_benchmark_kernel<S, C>, kLdgstsThreads, g->smem, &g->occupancy);
    BB_LDGSTS_CASES(X)
#undef X
  } else {
#define X(S) \
  if (g->stages == S) return occupancy_of(tma_benchmark_kernel<S>, kTmaThreads, g->smem, &g->occupancy);
    X(2) X(3) X(4) X(8)
#undef X
  }
  set_error("copy: no specialisation for stages=%d", g->stages);
  return BB_ERR_INTERNAL;
}

static int run(int method, int stages, int bif_kib, int row_bytes, const void* src, int64_t bytes, int64_t passes,
               int64_t rotation, bool validate, uint32_t* sink, unsigned long long* mism, int* status,
               void* stream) {
  Geometry g;
  int rc = geometry(method, stages, bif_kib, row_bytes, bytes, 0, &g);
  if (rc != BB_OK) return rc;
  rc = finish_geometry(&g, nullptr);
  if (rc != BB_OK) return rc;
  if (!src || !sink || (validate && !mism)) {
    set_error("copy: null device pointer");
    return BB_ERR_ARGUMENT;
  }
  if ((reinterpret_cast<uintptr_t>(src) & 15u) != 0) {
    set_error("copy: source pointer is not 16-byte aligned");
    return BB_ERR_ARGUMENT;
  }
  if (passes < 1 || rotation < 0) {
    set_error("copy: passes must be >= 1 and rotation >= 0");
    return BB_ERR_ARGUMENT;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = method == BB_COPY_LDGSTS ? launch_ldgsts(g, validate, src, bytes, passes, rotation, sink, mism, st)
                                : launch_tma(g, validate, src, bytes, passes, rotation, sink, mism, status, st);
  if (rc == BB_OK) g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return rc;
}

}  // namespace copy
}  // namespace bb

extern "C" {

BB_API size_t bb_copy_info_size(void) { return sizeof(bb_copy_info); }

BB_API int bb_copy_plan(int method, int stages, int bif_kib, int row_bytes, int64_t bytes, int sm_count,
                        bb_copy_info* info) {
  using namespace bb;
  try {
    clear_error();
    copy::Geometry g;
    int rc = copy::geometry(method, stages, bif_kib, row_bytes, bytes, sm_count, &g);
    if (rc != BB_OK) return rc;
    if (sm_count <= 0) {
      rc = copy::finish_geometry(&g, nullptr);
      if (rc != BB_OK) return rc;
      rc = copy::query_occupancy(method, &g);
      if (rc != BB_OK) return rc;
    } else {
      g.smem = g.stages * g.stage_bytes;  // host-only estimate; the launch reserves > half an SM
    }
    if (info) {
      info->method = method;
      info->stages = g.stages;
      info->bytes_in_flight_kib = bif_kib;
      info->stage_bytes = g.stage_bytes;
      info->bytes_in_flight = static_cast<int64_t>(g.stages) * g.stage_bytes;
      info->copies_per_thread = g.copies;
      info->row_bytes = g.row_bytes;
      info->tile_rows = g.tile_rows;
      info->threads_per_cta = g.threads;
      info->grid_ctas = g.grid;
      info->smem_bytes = g.smem;
      info->total_tiles = g.total_tiles;
      info->occupancy_ctas_per_sm = g.occupancy;
      for (int i = 0; i < 3; ++i) info->reserved[i] = 0;
    }
    return BB_OK;
  } catch (...) {
    bb::set_error("bb_copy_plan: unexpected C++ exception");
    return BB_ERR_INTERNAL;
  }
}

BB_API int bb_copy_run(int method, int stages, int bif_kib, int row_bytes, const void* src, int64_t bytes,
                       int64_t passes, int64_t rotation, uint32_t* sink, int* status, void* stream) {
  try {
    bb::clear_error();
    return bb::copy::run(method, stages, bif_kib, row_bytes, src, bytes, passes, rotation, false, sink, nullptr,
                         status, stream);
  } catch (...) {
    bb::set_error("bb_copy_run: unexpected C++ exception");
    return BB_ERR_INTERNAL;
  }
}

BB_API int bb_copy_validate(int method, int stages, int bif_kib, int row_bytes, const void* src, int64_t bytes,
                            uint32_t* sink, unsigned long long* mismatches, int* status, void* stream) {
  try {
    bb::clear_error();
    return bb::copy::run(method, stages, bif_kib, row_bytes, src, bytes, 1, 0, true, sink, mismatches, status,
                         stream);
  } catch (...) {
    bb::set_error("bb_copy_validate: unexpected C++ exception");
    return BB_ERR_INTERNAL;
  }
}

BB_API int bb_fill_pattern(void* dst, int64_t bytes, void* stream) {
  using namespace bb;
  clear_error();
  if (!dst || bytes <= 0 || bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(dst) & 15u)) {
    set_error("bb_fill_pattern: need a 16-byte aligned buffer and a positive multiple of 16 bytes");
    return BB_ERR_ARGUMENT;
  }
  DeviceInfo dev;
  int rc = query_device(&dev);
  if (rc != BB_OK) return rc;
  const int64_t nvec = bytes / 16;
  int64_t blocks = (nvec + 255) / 256;
  if (blocks > int64_t(dev.sm_count) * 8) blocks = int64_t(dev.sm_count) * 8;
  copy::fill_pattern_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(dst), nvec);
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return check_cuda(cudaGetLastError(), "fill_pattern_kernel");
}

BB_API int bb_fill_uniform_u32(void* dst, int64_t bytes, uint64_t seed, void* stream) {
  using namespace bb;
  clear_error();
  if (!dst || bytes <= 0 || bytes % 4 != 0 || (reinterpret_cast<uintptr_t>(dst) & 3u)) {
    set_error("bb_fill_uniform_u32: need a 4-byte aligned buffer and a positive multiple of 4 bytes");
    return BB_ERR_ARGUMENT;
  }
  DeviceInfo dev;
  int rc = query_device(&dev);
  if (rc != BB_OK) return rc;
  const int64_t n = bytes / 4;
  int64_t blocks = (n + 255) / 256;
  if (blocks > int64_t(dev.sm_count) * 8) blocks = int64_t(dev.sm_count) * 8;
  copy::fill_uniform_u32_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint32_t*>(dst), n, seed);
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return check_cuda(cudaGetLastError(), "fill_uniform_u32_kernel");
}

}  // extern "C"
