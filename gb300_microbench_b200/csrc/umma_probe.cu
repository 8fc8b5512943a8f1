// tcgen05 UMMA issue-throughput probes for sm_100a: the 1-SM (cta_group::1,
// M = 128) and 2-SM (cta_group::2, M = 256 over a CTA pair) BF16 probes of
// the reference (umma_throughput/umma_1sm.cu, umma_2sm.cu).
//
// Each CTA stages its operands from global memory into the canonical
// non-swizzled K-major core-matrix layout (8 rows x 16 bytes per core
// matrix; the two 8-element K halves LBO = 128 B apart, successive 8-row
// groups SBO = 256 B apart), so the same kernel serves the reference's
// integer patterns and the baseline-mode N(0,1) operands. One elected thread of
// CTA rank 0 issues DEPTH dependent MMAs per iteration (the first with
// enable_input_d = 0), commits to its own mbarrier and waits for it (bounded)
// before the next iteration; %clock64 brackets the loop.
//
// 2-SM probes have two loop forms. With the handshake (the reference's
// loop, umma_2sm.cu:617-659, and the default of the umma_2sm CLI), every
// iteration's commit arrives on both CTAs' mbarriers (two commits here, one
// per CTA, where the reference sends one to both), each CTA waits on its own,
// and all threads of both CTAs meet in a cluster barrier before the next
// iteration, inside the timed region. Without it, only the issuing CTA waits
// per iteration; the peer learns of the final MMA through one extra commit
// after the loop, so the timed loop carries no cluster handshake.
#include <atomic>

#include "common.cuh"
#include "ptx.cuh"

namespace bb {
extern std::atomic<int64_t> g_kernel_launches;

namespace umma {

constexpr int kThreads = 128;
constexpr int kK = 16;

// Element offset of (row, k) in the core-matrix layout described above.
__device__ __forceinline__ int core_index(int row, int k) {
  return (row >> 3) * 128 + (k >> 3) * 64 + (row & 7) * 8 + (k & 7);
}

template <int CG, int N, int DEPTH>
__device__ __forceinline__ void probe_body(int64_t iterations, int timed, const uint16_t* __restrict__ a_g,
                                           const uint16_t* __restrict__ b_g, float* __restrict__ d_out,
                                           unsigned long long* __restrict__ cycles, int* __restrict__ launch_ok,
                                           int* status, int handshake) {
  constexpr int kMLocal = 128;
  constexpr int kNLocal = N / CG;
  constexpr int kABytes = kMLocal * kK * 2;
  const int tid = threadIdx.x;
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
  const bool geometry_ok = gridDim.x == CG && gridDim.y == 1 && gridDim.z == 1 && blockDim.x == kThreads &&
                           blockDim.y == 1 && blockDim.z == 1 && (CG == 1 || cluster_nctarank() == 2);
  if (!geometry_ok) {
    if (tid == 0 && rank < 2) launch_ok[rank] = 0;
    if (tid == 0 && status) atomicCAS(status, 0, kDevBadLaunch);
    return;
  }
  if (tid == 0) launch_ok[rank] = 1;

  extern __shared__ __align__(1024) uint8_t smem[];
  uint16_t* sa = reinterpret_cast<uint16_t*>(smem);
  uint16_t* sb = reinterpret_cast<uint16_t*>(smem + kABytes);
  __shared__ __align__(8) uint64_t mbar;
  __shared__ __align__(8) uint64_t peer_done;
  __shared__ uint32_t tmem_slot;

  for (int i = tid; i < kMLocal * kK; i += kThreads) {
    const int r = i / kK, k = i % kK;
    sa[core_index(r, k)] = a_g[(rank * kMLocal + r) * kK + k];
  }
  for (int i = tid; i < kNLocal * kK; i += kThreads) {
    const int r = i / kK, k = i % kK;
    sb[core_index(r, k)] = b_g[(rank * kNLocal + r) * kK + k];
  }
  fence_proxy_async_smem();
  if (tid == 0) {
    mbar_init(smem_u32(&mbar), 1);
    mbar_init(smem_u32(&peer_done), 1);
    fence_mbarrier_init_cluster();
  }
  __syncthreads();
  if constexpr (CG == 2) {
    // Operand writes and barrier inits of both CTAs precede the first MMA.
    asm volatile("fence.proxy.async.shared::cluster;" ::: "memory");
    cluster_sync();
  }
  if (tid < 32) {
    tmem_alloc<CG>(smem_u32(&tmem_slot), N);
    tmem_relinquish<CG>();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();
  tc_fence_after();
  const uint32_t tmem_d = *reinterpret_cast<volatile uint32_t*>(&tmem_slot);

  const bool pair_handshake = CG == 2 && handshake != 0;
  if (pair_handshake) {
    // The reference's per-iteration handshake (see the header comment).
    constexpr uint32_t idesc = make_idesc_bf16_f32(kMLocal * CG, N);
    const uint64_t adesc = make_smem_desc(smem_u32(sa), 128, 256, kLayoutNone);
    const uint64_t bdesc = make_smem_desc(smem_u32(sb), 128, 256, kLayoutNone);
    const uint32_t mb = smem_u32(&mbar);
    uint32_t parity = 0;
    uint64_t c0 = 0;
    if (rank == 0 && tid == 0) c0 = clock64_now();
    for (int64_t it = 0; it < iterations; ++it) {
      if (rank == 0 && tid == 0) {
        umma_f16<CG>(tmem_d, adesc, bdesc, idesc, 0u);
#pragma unroll
        for (int d = 1; d < DEPTH; ++d) umma_f16<CG>(tmem_d, adesc, bdesc, idesc, 1u);
        umma_commit<CG>(mb);
        umma_commit<CG>(mapa_shared(mb, 1));
      }
      // Each CTA waits on its own barrier; after a timeout (status set) the
      // remaining waits return at once, so the loop still ends.
      if (tid == 0) bb_wait<true>(mb, parity, status, kDevTimeoutProbe, /*honor_abort=*/true);
      parity ^= 1u;
      __syncthreads();
      cluster_sync();
    }
    if (rank == 0 && tid == 0 && timed) cycles[0] = static_cast<unsigned long long>(clock64_now() - c0);
  }
  if (!pair_handshake && rank == 0 && tid == 0) {
    constexpr uint32_t idesc = make_idesc_bf16_f32(kMLocal * CG, N);
    const uint64_t adesc = make_smem_desc(smem_u32(sa), 128, 256, kLayoutNone);
    const uint64_t bdesc = make_smem_desc(smem_u32(sb), 128, 256, kLayoutNone);
    const uint32_t mb = smem_u32(&mbar);
    uint32_t parity = 0;
    const uint64_t c0 = clock64_now();
    for (int64_t it = 0; it < iterations; ++it) {
      umma_f16<CG>(tmem_d, adesc, bdesc, idesc, 0u);
#pragma unroll
      for (int d = 1; d < DEPTH; ++d) umma_f16<CG>(tmem_d, adesc, bdesc, idesc, 1u);
      umma_commit<CG>(mb);
      if (!bb_wait(mb, parity, status, kDevTimeoutProbe, /*honor_abort=*/false)) break;
      parity ^= 1u;
    }
    const uint64_t c1 = clock64_now();
    if (timed) cycles[0] = static_cast<unsigned long long>(c1 - c0);
    if constexpr (CG == 2) umma_commit<CG>(mapa_shared(smem_u32(&peer_done), 1));
  }
  if constexpr (CG == 2) {
    if (!pair_handshake && rank == 1 && tid == 0) {
      bb_wait<true>(smem_u32(&peer_done), 0, status, kDevTimeoutProbe, /*honor_abort=*/false);
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();
  tc_fence_after();

  // Untimed read-back: warp w reads TMEM lanes [32w, 32w + 32).
  const int warp = tid / 32, lane = tid % 32;
  const int row = static_cast<int>(rank) * kMLocal + warp * 32 + lane;
#pragma unroll 1
  for (int c = 0; c < N; c += 32) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(tmem_d + (static_cast<uint32_t>(warp * 32) << 16) + c, r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; ++j) d_out[static_cast<int64_t>(row) * N + c + j] = __uint_as_float(r[j]);
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();
  if (tid < 32) {
    tc_fence_after();
    tmem_dealloc<CG>(tmem_d, N);
  }
}

}  // namespace umma
}  // namespace bb

// Kernel names follow the reference's extern "C" symbols
// (umma_1sm.cu:509-527, umma_2sm.cu:715-731), extended with depths 32 and 128.
#define BB_UMMA_1SM(N, D)                                                                                   \
  extern "C" __global__ void __launch_bounds__(128, 1) umma_1sm_m128n##N##k16_d##D(                         \
      int64_t iterations, int timed, const uint16_t* a, const uint16_t* b, float* d, unsigned long long* cyc, \
      int* ok, int* st, int hs) {                                                                           \
    bb::umma::probe_body<1, N, D>(iterations, timed, a, b, d, cyc, ok, st, hs);                             \
  }
#define BB_UMMA_2SM(N, D)                                                                                   \
  extern "C" __global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128, 1) umma_2sm_m256n##N##k16_d##D( \
      int64_t iterations, int timed, const uint16_t* a, const uint16_t* b, float* d, unsigned long long* cyc, \
      int* ok, int* st, int hs) {                                                                           \
    bb::umma::probe_body<2, N, D>(iterations, timed, a, b, d, cyc, ok, st, hs);                             \
  }
#define BB_UMMA_ALL_DEPTHS(M, N) M(N, 4) M(N, 16) M(N, 32) M(N, 64) M(N, 128) M(N, 256)
BB_UMMA_ALL_DEPTHS(BB_UMMA_1SM, 64)
BB_UMMA_ALL_DEPTHS(BB_UMMA_1SM, 128)
BB_UMMA_ALL_DEPTHS(BB_UMMA_1SM, 256)
BB_UMMA_ALL_DEPTHS(BB_UMMA_2SM, 64)
BB_UMMA_ALL_DEPTHS(BB_UMMA_2SM, 128)
BB_UMMA_ALL_DEPTHS(BB_UMMA_2SM, 256)

namespace {

using ProbeFn = void (*)(int64_t, int, const uint16_t*, const uint16_t*, float*, unsigned long long*, int*, int*,
                         int);

struct ProbeEntry {
  int cg, n, depth;
  ProbeFn fn;
  const char* name;
};

#define E1(N, D) {1, N, D, &umma_1sm_m128n##N##k16_d##D, "umma_1sm_m128n" #N "k16_d" #D},
#define E2(N, D) {2, N, D, &umma_2sm_m256n##N##k16_d##D, "umma_2sm_m256n" #N "k16_d" #D},
const ProbeEntry kProbes[] = {BB_UMMA_ALL_DEPTHS(E1, 64) BB_UMMA_ALL_DEPTHS(E1, 128) BB_UMMA_ALL_DEPTHS(E1, 256)
                                  BB_UMMA_ALL_DEPTHS(E2, 64) BB_UMMA_ALL_DEPTHS(E2, 128)
                                      BB_UMMA_ALL_DEPTHS(E2, 256)};
#undef E1
#undef E2

const ProbeEntry* find_probe(int cg, int n, int depth) {
  for (const auto& e : kProbes) {
    if (e.cg == cg && e.n == n && e.depth == depth) return &e;
  }
  return nullptr;
}

__global__ void wait_timeout_kernel(int64_t budget_ns, int* status) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    bb::mbar_init(bb::smem_u32(&bar), 1);
    bb::fence_mbarrier_init_cluster();
  }
  __syncthreads();
  // Nothing ever arrives on `bar`: every wait form must give up after its
  // budget and record it. Status slots: [0] single-thread wait, [1] warp-wide
  // spinning wait, [2] warp-wide wait with the suspend hint.
  if (threadIdx.x == 0) {
    bb::bb_wait(bb::smem_u32(&bar), 0, status, bb::kDevTimeoutTest, false, static_cast<uint64_t>(budget_ns));
  }
  __syncwarp();
  bb::bb_wait_warp<false, false>(bb::smem_u32(&bar), 0, status + 1, bb::kDevTimeoutTest, false,
                                 static_cast<uint64_t>(budget_ns));
  bb::bb_wait_warp<false, true>(bb::smem_u32(&bar), 0, status + 2, bb::kDevTimeoutTest, false,
                                static_cast<uint64_t>(budget_ns));
  __syncthreads();
}

}  // namespace

extern "C" {

BB_API const char* bb_umma_kernel_name(int cta_group, int n, int depth) {
  const ProbeEntry* e = find_probe(cta_group, n, depth);
  return e ? e->name : nullptr;
}

BB_API int bb_umma_run_ex(int cta_group, int n, int depth, int64_t iterations, int timed, int handshake,
                          const void* a, const void* b, float* d_out, unsigned long long* cycles, int* launch_ok,
                          int* status, void* stream) {
  using namespace bb;
  try {
    clear_error();
    const ProbeEntry* e = find_probe(cta_group, n, depth);
    if (!e) {
      set_error("bb_umma_run: no probe for cta_group=%d n=%d depth=%d", cta_group, n, depth);
      return BB_ERR_ARGUMENT;
    }
    if (iterations < 1) {
      set_error("bb_umma_run: iterations must be >= 1");
      return BB_ERR_ARGUMENT;
    }
    if (!a || !b || !d_out || !cycles || !launch_ok) {
      set_error("bb_umma_run: null device pointer");
      return BB_ERR_ARGUMENT;
    }
    DeviceInfo dev;
    int rc = query_device(&dev);
    if (rc != BB_OK) return rc;
    const int smem = 1024 + (128 + n / cta_group) * 16 * 2;
    BB_CUDA_TRY(cudaFuncSetAttribute(e->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    e->fn<<<cta_group, 128, smem, static_cast<cudaStream_t>(stream)>>>(
        iterations, timed, static_cast<const uint16_t*>(a), static_cast<const uint16_t*>(b), d_out, cycles,
        launch_ok, status, handshake);
    BB_CUDA_TRY(cudaGetLastError());
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    return BB_OK;
  } catch (...) {
    bb::set_error("bb_umma_run: unexpected C++ exception");
    return BB_ERR_INTERNAL;
  }
}

BB_API int bb_umma_run(int cta_group, int n, int depth, int64_t iterations, int timed, const void* a, const void* b,
                       float* d_out, unsigned long long* cycles, int* launch_ok, int* status, void* stream) {
  return bb_umma_run_ex(cta_group, n, depth, iterations, timed, 0, a, b, d_out, cycles, launch_ok, status, stream);
}

BB_API int bb_test_wait_timeout(int64_t budget_ns, int* status, void* stream) {
  using namespace bb;
  clear_error();
  if (!status || budget_ns <= 0 || budget_ns > 10000000000ll) {
    set_error("bb_test_wait_timeout: need a status pointer and 0 < budget_ns <= 10 s");
    return BB_ERR_ARGUMENT;
  }
  wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(budget_ns, status);
  BB_CUDA_TRY(cudaGetLastError());
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  return BB_OK;
}

}  // extern "C"
