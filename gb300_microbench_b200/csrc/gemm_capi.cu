// C ABI of the sm_100a GEMM: plan create / execute / run_host / destroy.
// Mirrors the plan life cycle of the reference's cuBLASLt bridge
// (gemm_comparison/cublaslt_bridge.cu:563-1016) for our own kernel.
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <new>

#include "common.cuh"
#include "gemm_sm100.cuh"

namespace bb {
std::atomic<int64_t> g_kernel_launches{0};
}

// Host-buffer pipeline of bb_gemm_run_host: B first, then A in row chunks
// on an H2D stream; each chunk's GEMM on the plan's stream once its rows have
// landed; its C rows back on a D2H stream while later A chunks still arrive,
// so both copy directions and the compute overlap.
constexpr int kPipeChunks = 4;

struct HostPipe {
  static constexpr int kMaxChunks = 8;
  bool ready = false;
  int chunks = 0;
  int64_t row0[kMaxChunks] = {}, rows[kMaxChunks] = {};
  bb::gemm::Plan sub[kMaxChunks];
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t ev_b = nullptr, ev_a[kMaxChunks] = {}, ev_c[kMaxChunks] = {};
};

struct bb_gemm_plan {
  bb::gemm::Plan p;
  int* status_dev = nullptr;
  HostPipe pipe;
};

namespace bb {
namespace gemm {

int build_maps(Plan& pl) {
  using namespace bb;
  const uint64_t M = pl.m, N = pl.n, K = pl.k, L = pl.l;
  {
    const uint64_t dims[3] = {K, M, L};
    const uint64_t strides[2] = {K * 2, M * K * 2};
    const uint32_t box[3] = {64, 128, 1};
    int rc = encode_tiled(&pl.tm_a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3, pl.a, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (rc != BB_OK) return rc;
  }
  {
    const uint64_t dims[3] = {K, N, L};
    const uint64_t strides[2] = {K * 2, N * K * 2};
    const uint32_t box[3] = {64, static_cast<uint32_t>(pl.b_rows), 1};
    int rc = encode_tiled(&pl.tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3, pl.b, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
    if (rc != BB_OK) return rc;
    if (pl.narrow_tiles > 0) {
      // Half-height boxes of B for the narrow tail's half-width items.
      const uint32_t half_box[3] = {64, static_cast<uint32_t>(pl.b_rows / 2), 1};
      rc = encode_tiled(&pl.tm_b_half, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3, pl.b, dims, strides, half_box,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
      if (rc != BB_OK) return rc;
    }
  }
  {
    const bool f32 = pl.c_dtype == BB_DTYPE_F32;
    const uint64_t es = f32 ? 4 : 2;
    const uint64_t dims[3] = {N, M, L};
    const uint64_t strides[2] = {N * es, M * N * es};
    const uint32_t box[3] = {static_cast<uint32_t>(pl.epi_cols), 32, 1};
    int rc = encode_tiled(&pl.tm_c, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                          static_cast<int>(es), 3, pl.c, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_NONE);
    if (rc != BB_OK) return rc;
  }
  return BB_OK;
}

}  // namespace gemm
}  // namespace bb

namespace {

void fill_info(const bb::gemm::Plan& p, bb_gemm_info* info) {
  if (!info) return;
  info->mma_tiler_m = p.tile_m;
  info->mma_tiler_n = p.tile_n;
  info->cluster_m = p.cg;
  info->cluster_n = 1;
  info->use_2cta_instrs = p.cg == 2 ? 1 : 0;
  info->max_active_clusters = p.max_active_clusters;
  info->stages = p.stages;
  info->grid_ctas = p.grid;
  info->num_tiles = p.num_tiles;
  info->smem_bytes = p.smem_bytes;
  info->tmem_columns = p.tmem_cols;
  info->threads_per_cta = p.threads;
  info->persistent = p.persistent ? 1 : 0;
  info->raster_group_m = p.group_m;
  info->c_dtype = p.c_dtype;
  info->variant = p.variant;
}

void free_pipe(HostPipe& hp) {
  for (int i = 0; i < HostPipe::kMaxChunks; ++i) {
    if (hp.sub[i].partials) cudaFree(hp.sub[i].partials);
    if (hp.sub[i].counters) cudaFree(hp.sub[i].counters);
    hp.sub[i].partials = nullptr;
    hp.sub[i].counters = nullptr;
    if (hp.ev_a[i]) cudaEventDestroy(hp.ev_a[i]);
    if (hp.ev_c[i]) cudaEventDestroy(hp.ev_c[i]);
    hp.ev_a[i] = hp.ev_c[i] = nullptr;
  }
  if (hp.ev_b) cudaEventDestroy(hp.ev_b);
  if (hp.h2d) cudaStreamDestroy(hp.h2d);
  if (hp.d2h) cudaStreamDestroy(hp.d2h);
  hp.ev_b = nullptr;
  hp.h2d = hp.d2h = nullptr;
  hp.ready = false;
}

// Sub-plans over row chunks of a single-batch plan (chunk rows are multiples
// of 256, the CTA-pair tile height), their workspaces, streams and events.
int init_pipe(bb_gemm_plan* plan) {
  using namespace bb;
  HostPipe& hp = plan->pipe;
  const gemm::Plan& p = plan->p;
  DeviceInfo dev;
  int rc = query_device(&dev);
  if (rc != BB_OK) return rc;
  const int64_t units = p.m / 256;  // whole 256-row blocks
  // Four chunks measured best at 4096^3 (e2e 86.9 TFLOP/s; eight: 83.0, the
  // per-copy and per-launch costs outweigh the shorter tail).
  int want = kPipeChunks;
  bool taper = false;  // 1:3:3:1 row weights (four chunks)
  // BB_GEMM_PIPE=<chunks>[t] overrides (t: tapered four-chunk weights).
  if (const char* env = std::getenv("BB_GEMM_PIPE")) {
    const int c = std::atoi(env);
    if (c >= 1 && c <= HostPipe::kMaxChunks) want = c;
    taper = std::strchr(env, 't') != nullptr;
  }
  int chunks = static_cast<int>(units < want ? units : want);
  if (chunks < 2) return BB_ERR_UNSUPPORTED;
  hp.chunks = chunks;
  const size_t es = p.c_dtype == BB_DTYPE_F32 ? 4 : 2;
  int64_t r = 0;
  // Row weights 1:3:3:1 for four chunks: a small first chunk starts the
  // D2H stream early, a small last one shortens the tail after the final
  // H2D byte (its GEMM and C copy); the middle chunks carry the bulk.
  static const int kWeights4[4] = {1, 3, 3, 1};
  int64_t bounds[HostPipe::kMaxChunks + 1] = {0};
  for (int i = 0, acc = 0; i < chunks; ++i) {
    const bool tw = taper && chunks == 4 && units >= 8;
    acc += tw ? kWeights4[i] : 1;
    const int total = tw ? 8 : chunks;
    bounds[i + 1] = (units * acc) / total;
  }
  for (int i = 0; i < chunks; ++i) {
    const int64_t rows = (i == chunks - 1) ? p.m - r : (bounds[i + 1] - bounds[i]) * 256;
    hp.row0[i] = r;
    hp.rows[i] = rows;
    gemm::Plan& q = hp.sub[i];
    q = gemm::Plan{};
    q.m = rows;
    q.n = p.n;
    q.k = p.k;
    q.l = 1;
    q.a = static_cast<const uint8_t*>(p.a) + static_cast<size_t>(r) * p.k * 2;
    q.b = p.b;
    q.c = static_cast<uint8_t*>(p.c) + static_cast<size_t>(r) * p.n * es;
    q.c_dtype = p.c_dtype;
    q.stream = p.stream;
    q.alpha = p.alpha;
    q.beta = p.beta;
    q.epi_mode = p.epi_mode;
    q.c_src = p.c_src ? static_cast<const uint8_t*>(p.c_src) + static_cast<size_t>(r) * p.n * es : nullptr;
    rc = gemm::plan_init(q, p.variant, dev.sm_count);
    if (rc == BB_OK) rc = gemm::build_maps(q);
    if (rc == BB_OK && q.sk_tiles > 0) {
      rc = check_cuda(cudaMalloc(&q.partials, q.partial_floats * sizeof(float)), "cudaMalloc(pipe partials)");
      if (rc == BB_OK) rc = check_cuda(cudaMalloc(&q.counters, q.counter_ints * sizeof(int)), "cudaMalloc(pipe counters)");
      if (rc == BB_OK) rc = check_cuda(cudaMemset(q.counters, 0, q.counter_ints * sizeof(int)), "cudaMemset(pipe counters)");
    }
    q.status = plan->status_dev;
    if (rc == BB_OK) rc = check_cuda(cudaEventCreateWithFlags(&hp.ev_a[i], cudaEventDisableTiming), "cudaEventCreate");
    if (rc == BB_OK) rc = check_cuda(cudaEventCreateWithFlags(&hp.ev_c[i], cudaEventDisableTiming), "cudaEventCreate");
    if (rc != BB_OK) {
      free_pipe(hp);
      return rc;
    }
    r += rows;
  }
  rc = check_cuda(cudaEventCreateWithFlags(&hp.ev_b, cudaEventDisableTiming), "cudaEventCreate");
  if (rc == BB_OK) rc = check_cuda(cudaStreamCreateWithFlags(&hp.h2d, cudaStreamNonBlocking), "cudaStreamCreate");
  if (rc == BB_OK) rc = check_cuda(cudaStreamCreateWithFlags(&hp.d2h, cudaStreamNonBlocking), "cudaStreamCreate");
  if (rc != BB_OK) {
    free_pipe(hp);
    return rc;
  }
  hp.ready = true;
  return BB_OK;
}

// Queues the pipelined host-buffer run: B, then A chunk by chunk on the
// H2D stream; each chunk's GEMM on the plan's stream after its rows landed;
// its C rows on the D2H stream after its GEMM.
int enqueue_pipe(bb_gemm_plan* plan, const void* a_host, const void* b_host, void* c_host, size_t b_bytes,
                 size_t es) {
  using namespace bb;
  gemm::Plan& p = plan->p;
  HostPipe& hp = plan->pipe;
  BB_CUDA_TRY(cudaEventRecord(hp.ev_b, p.stream));
  BB_CUDA_TRY(cudaStreamWaitEvent(hp.h2d, hp.ev_b, 0));
  BB_CUDA_TRY(cudaMemcpyAsync(const_cast<void*>(p.b), b_host, b_bytes, cudaMemcpyHostToDevice, hp.h2d));
  BB_CUDA_TRY(cudaEventRecord(hp.ev_b, hp.h2d));
  for (int i = 0; i < hp.chunks; ++i) {
    const size_t off = static_cast<size_t>(hp.row0[i]) * p.k * 2;
    BB_CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(const_cast<void*>(p.a)) + off,
                                static_cast<const uint8_t*>(a_host) + off, static_cast<size_t>(hp.rows[i]) * p.k * 2,
                                cudaMemcpyHostToDevice, hp.h2d));
    BB_CUDA_TRY(cudaEventRecord(hp.ev_a[i], hp.h2d));
  }
  BB_CUDA_TRY(cudaStreamWaitEvent(p.stream, hp.ev_b, 0));
  for (int i = 0; i < hp.chunks; ++i) {
    BB_CUDA_TRY(cudaStreamWaitEvent(p.stream, hp.ev_a[i], 0));
    int rc = hp.sub[i].launch(hp.sub[i]);
    if (rc != BB_OK) return rc;
    ++p.launches;
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    BB_CUDA_TRY(cudaEventRecord(hp.ev_c[i], p.stream));
    BB_CUDA_TRY(cudaStreamWaitEvent(hp.d2h, hp.ev_c[i], 0));
    const size_t coff = static_cast<size_t>(hp.row0[i]) * p.n * es;
    BB_CUDA_TRY(cudaMemcpyAsync(static_cast<uint8_t*>(c_host) + coff, static_cast<const uint8_t*>(p.c) + coff,
                                static_cast<size_t>(hp.rows[i]) * p.n * es, cudaMemcpyDeviceToHost, hp.d2h));
  }
  return BB_OK;
}

}  // namespace

extern "C" {

BB_API size_t bb_gemm_info_size(void) { return sizeof(bb_gemm_info); }

BB_API int bb_gemm_plan_create(int64_t m, int64_t n, int64_t k, int64_t l, const void* a, const void* b, void* c,
                               int a_dtype, int b_dtype, int c_dtype, int variant, void* stream,
                               bb_gemm_plan** plan, bb_gemm_info* info) {
  using namespace bb;
  try {
    clear_error();
    if (!plan) {
      set_error("bb_gemm_plan_create: plan out-pointer is null");
      return BB_ERR_ARGUMENT;
    }
    *plan = nullptr;
    if (m <= 0 || n <= 0 || k <= 0 || l <= 0) {
      set_error("bb_gemm_plan_create: extents must be positive (m=%lld n=%lld k=%lld l=%lld)", (long long)m,
                (long long)n, (long long)k, (long long)l);
      return BB_ERR_ARGUMENT;
    }
    if (m * l > (int64_t(1) << 31) || n * l > (int64_t(1) << 31) || k > (int64_t(1) << 31)) {
      set_error("bb_gemm_plan_create: extents exceed the 32-bit tile coordinate range");
      return BB_ERR_ARGUMENT;
    }
    if (a_dtype != BB_DTYPE_BF16 || b_dtype != BB_DTYPE_BF16) {
      set_error("bb_gemm_plan_create: A and B must be BF16");
      return BB_ERR_UNSUPPORTED;
    }
    if (c_dtype != BB_DTYPE_BF16 && c_dtype != BB_DTYPE_F32) {
      set_error("bb_gemm_plan_create: C must be BF16 or FP32");
      return BB_ERR_UNSUPPORTED;
    }
    if (variant < BB_VARIANT_NONPERSISTENT_1CTA || variant > BB_VARIANT_TUNED) {
      set_error("bb_gemm_plan_create: unknown variant %d", variant);
      return BB_ERR_ARGUMENT;
    }
    if (k % 8 != 0) {
      set_error("bb_gemm_plan_create: K=%lld must be a multiple of 8 (16-byte TMA row stride)", (long long)k);
      return BB_ERR_ARGUMENT;
    }
    if ((c_dtype == BB_DTYPE_BF16 && n % 8 != 0) || (c_dtype == BB_DTYPE_F32 && n % 4 != 0)) {
      set_error("bb_gemm_plan_create: N=%lld breaks the 16-byte row stride of C", (long long)n);
      return BB_ERR_ARGUMENT;
    }
    DeviceInfo dev;
    int rc = query_device(&dev);
    if (rc != BB_OK) return rc;

    auto* h = new (std::nothrow) bb_gemm_plan();
    if (!h) {
      set_error("bb_gemm_plan_create: out of host memory");
      return BB_ERR_INTERNAL;
    }
    gemm::Plan& p = h->p;
    p.m = m;
    p.n = n;
    p.k = k;
    p.l = l;
    p.a = a;
    p.b = b;
    p.c = c;
    p.c_dtype = c_dtype;
    p.stream = static_cast<cudaStream_t>(stream);
    rc = gemm::plan_init(p, variant, dev.sm_count);
    if (rc == BB_OK) rc = gemm::build_maps(p);
    if (rc == BB_OK) rc = check_cuda(cudaMalloc(&h->status_dev, sizeof(int)), "cudaMalloc(status)");
    if (rc == BB_OK) rc = check_cuda(cudaMemset(h->status_dev, 0, sizeof(int)), "cudaMemset(status)");
    if (rc == BB_OK && p.sk_tiles > 0) {
      // Stream-K workspace, owned by the plan (as the reference bridge owns
      // its cuBLASLt workspace). Counters start at zero and are reset by the
      // kernel after each use.
      rc = check_cuda(cudaMalloc(&p.partials, p.partial_floats * sizeof(float)), "cudaMalloc(split-tail partials)");
      if (rc == BB_OK) rc = check_cuda(cudaMalloc(&p.counters, p.counter_ints * sizeof(int)), "cudaMalloc(counters)");
      if (rc == BB_OK) rc = check_cuda(cudaMemset(p.counters, 0, p.counter_ints * sizeof(int)), "cudaMemset(counters)");
    }
    if (rc != BB_OK) {
      if (h->status_dev) cudaFree(h->status_dev);
      if (p.partials) cudaFree(p.partials);
      if (p.counters) cudaFree(p.counters);
      delete h;
      return rc;
    }
    p.status = h->status_dev;
    fill_info(p, info);
    *plan = h;
    return BB_OK;
  } catch (...) {
    bb::set_error("bb_gemm_plan_create: unexpected C++ exception");
    return BB_ERR_INTERNAL;
  }
}

BB_API int bb_gemm_execute_n(bb_gemm_plan* plan, int iterations) {
  using namespace bb;
  try {
    if (!plan || !plan->p.launch) {
      set_error("bb_gemm_execute: null plan");
      return BB_ERR_ARGUMENT;
    }
    if (iterations < 0) {
      set_error("bb_gemm_execute: negative iteration count %d", iterations);
      return BB_ERR_ARGUMENT;
    }
    for (int i = 0; i < iterations; ++i) {
      int rc = plan->p.launch(plan->p);
      if (rc != BB_OK) return rc;
      ++plan->p.launches;
      g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    }
    return BB_OK;
  } catch (...) {
    bb::set_error("bb_gemm_execute: unexpected C++ exception");
    return BB_ERR_INTERNAL;
  }
}

BB_API int bb_gemm_execute(bb_gemm_plan* plan) { return bb_gemm_execute_n(plan, 1); }

BB_API int bb_gemm_synchronize(bb_gemm_plan* plan) {
  using namespace bb;
  try {
    if (!plan) {
      set_error("bb_gemm_synchronize: null plan");
      return BB_ERR_ARGUMENT;
    }
    BB_CUDA_TRY(cudaStreamSynchronize(plan->p.stream));
    int st = 0;
    BB_CUDA_TRY(cudaMemcpy(&st, plan->status_dev, sizeof(int), cudaMemcpyDeviceToHost));
    if (st != 0) {
      set_error("GEMM kernel reported device status 0x%x (%s)", st,
                st == 0x200 ? "launch contract violated" : "a bounded wait timed out");
      return st == 0x200 ? BB_ERR_INTERNAL : BB_ERR_TIMEOUT;
    }
    return BB_OK;
  } catch (...) {
    bb::set_error("bb_gemm_synchronize: unexpected C++ exception");
    return BB_ERR_INTERNAL;
  }
}

BB_API int bb_gemm_run_host(bb_gemm_plan* plan, const void* a_host, const void* b_host, void* c_host) {
  using namespace bb;
  try {
    if (!plan || !a_host || !b_host || !c_host) {
      set_error("bb_gemm_run_host: null argument");
      return BB_ERR_ARGUMENT;
    }
    gemm::Plan& p = plan->p;
    const size_t es = p.c_dtype == BB_DTYPE_F32 ? 4 : 2;
    const size_t a_bytes = static_cast<size_t>(p.m) * p.k * p.l * 2;
    const size_t b_bytes = static_cast<size_t>(p.n) * p.k * p.l * 2;
    const size_t c_bytes = static_cast<size_t>(p.m) * p.n * p.l * es;
    HostPipe& hp = plan->pipe;
    if (p.l == 1 && p.m >= 512 && !hp.ready) {
      const int rc = init_pipe(plan);
      if (rc != BB_OK && rc != BB_ERR_UNSUPPORTED) return rc;
    }
    if (!hp.ready || p.epi_mode != hp.sub[0].epi_mode || p.alpha != hp.sub[0].alpha || p.beta != hp.sub[0].beta) {
      // Serial path (batched problems, few rows, or an epilogue changed
      // since the pipeline was built).
      int rc = check_cuda(cudaMemcpyAsync(const_cast<void*>(p.a), a_host, a_bytes, cudaMemcpyHostToDevice, p.stream),
                          "cudaMemcpyAsync(A)");
      if (rc == BB_OK)
        rc = check_cuda(cudaMemcpyAsync(const_cast<void*>(p.b), b_host, b_bytes, cudaMemcpyHostToDevice, p.stream),
                        "cudaMemcpyAsync(B)");
      if (rc == BB_OK) rc = bb_gemm_execute_n(plan, 1);
      if (rc == BB_OK)
        rc = check_cuda(cudaMemcpyAsync(c_host, p.c, c_bytes, cudaMemcpyDeviceToHost, p.stream), "cudaMemcpyAsync(C)");
      if (rc != BB_OK) {
        cudaStreamSynchronize(p.stream);  // no copy may touch the host buffers after the call
        return rc;
      }
      return bb_gemm_synchronize(plan);
    }
    // Pipelined path. Work queued earlier on the plan's stream finishes
    // before the copies overwrite A and B. If queuing fails part-way, the
    // copy streams are drained before returning, so no copy still reads or
    // writes the caller's host buffers after the call.
    const int rc = enqueue_pipe(plan, a_host, b_host, c_host, b_bytes, es);
    if (rc != BB_OK) {
      cudaStreamSynchronize(hp.h2d);
      cudaStreamSynchronize(hp.d2h);
      cudaStreamSynchronize(p.stream);
      return rc;
    }
    BB_CUDA_TRY(cudaStreamSynchronize(hp.d2h));
    return bb_gemm_synchronize(plan);
  } catch (...) {
    bb::set_error("bb_gemm_run_host: unexpected C++ exception");
    return BB_ERR_INTERNAL;
  }
}

BB_API int bb_gemm_plan_set_epilogue(bb_gemm_plan* plan, float alpha, float beta, const void* c_src) {
  using namespace bb;
  try {
    clear_error();
    if (!plan) {
      set_error("bb_gemm_plan_set_epilogue: null plan");
      return BB_ERR_ARGUMENT;
    }
    gemm::Plan& p = plan->p;
    if (beta != 0.0f) {
      if (!c_src) {
        set_error("bb_gemm_plan_set_epilogue: beta != 0 needs a C source");
        return BB_ERR_ARGUMENT;
      }
      if (reinterpret_cast<uintptr_t>(c_src) % 16 != 0) {
        set_error("bb_gemm_plan_set_epilogue: the C source must be 16-byte aligned");
        return BB_ERR_ARGUMENT;
      }
    }
    p.alpha = alpha;
    p.beta = beta;
    p.c_src = beta != 0.0f ? c_src : nullptr;
    p.epi_mode = beta != 0.0f ? 2 : (alpha != 1.0f ? 1 : 0);
    // The host-buffer pipeline's row-chunk plans follow.
    HostPipe& hp = plan->pipe;
    const size_t es = p.c_dtype == BB_DTYPE_F32 ? 4 : 2;
    for (int i = 0; hp.ready && i < hp.chunks; ++i) {
      hp.sub[i].alpha = p.alpha;
      hp.sub[i].beta = p.beta;
      hp.sub[i].epi_mode = p.epi_mode;
      hp.sub[i].c_src =
          p.c_src ? static_cast<const uint8_t*>(p.c_src) + static_cast<size_t>(hp.row0[i]) * p.n * es : nullptr;
    }
    return BB_OK;
  } catch (...) {
    bb::set_error("bb_gemm_plan_set_epilogue: unexpected C++ exception");
    return BB_ERR_INTERNAL;
  }
}

BB_API int64_t bb_gemm_launches(const bb_gemm_plan* plan) { return plan ? plan->p.launches : -1; }

BB_API int bb_gemm_destroy(bb_gemm_plan* plan) {
  using namespace bb;
  if (!plan) return BB_OK;
  int rc = BB_OK;
  free_pipe(plan->pipe);
  for (void* ptr : {static_cast<void*>(plan->status_dev), static_cast<void*>(plan->p.partials),
                    static_cast<void*>(plan->p.counters)}) {
    if (!ptr) continue;
    cudaError_t e = cudaFree(ptr);
    if (e != cudaSuccess && rc == BB_OK) rc = check_cuda(e, "cudaFree(plan buffer)");
  }
  delete plan;
  return rc;
}

BB_API int64_t bb_kernel_launches(void) { return bb::g_kernel_launches.load(); }

}  // extern "C"
