// bb_gemm_run_noalloc: the tuned GEMM for callers that cannot allocate
// device memory, e.g. code running where cudaMalloc is off limits (inside a
// custom allocator's own callbacks, a plugin host that owns the whole device
// heap, or a CUDA-graph-building framework that forbids allocation while it
// records). It runs the kernel of bb_gemm_plan_create/bb_gemm_execute with
// the tuned variant; only where its scratch lives differs.
//
// Scratch: the GEMM's stream-K workspace (partial tiles, k-block counters)
// and its device status word live in one file-scope __device__ array of
// kScratchBytes (37 MiB + 64 KiB). Every GPU that loads this library holds
// that array until the process exits. The partial tiles take two slots per
// cluster: 2 x 74 pairs x 2 CTAs x 128 x 256 FP32 = 37 MiB on a 148-SM B200,
// the most any tuned plan needs there (only tiles up to 256 wide get a
// stream-K region; 148 single CTAs with 128-wide tiles need half of it). A
// problem whose workspace would not fit (a device with more SMs) is refused
// with BB_ERR_ARGUMENT.
//
// Host code cannot use the array's name as a device address (in host code
// it names a host-side stand-in), so the first call in each CUDA context
// (normally a device's primary context), with that context current,
// resolves the address with cudaGetSymbolAddress and caches it per context.
// That first call should therefore come before any stream capture. Every
// call then clears the status word and the counters with cudaMemsetAsync on
// the caller's stream and launches the kernel; no call allocates or frees
// device memory. With wait != 0 the call also synchronises the stream and
// returns BB_ERR_TIMEOUT when a device-side wait gave up; with wait == 0 it
// returns as soon as the work is queued and gives up that report (the next
// call clears the status word). All calls share the one array, which keeps
// the last call's contents: calls that overlap on the GPU (different streams
// without ordering between them) race on it.
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "gemm_sm100.cuh"

namespace bb {
extern std::atomic<int64_t> g_kernel_launches;

namespace gemm_noalloc {

constexpr size_t kStatusBytes = 256;
constexpr size_t kCounterBytes = 64 * 1024 - kStatusBytes;
constexpr size_t kPartialBytes = 37u << 20;
constexpr size_t kScratchBytes = kStatusBytes + kCounterBytes + kPartialBytes;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

// Device addresses of g_scratch, one per CUDA context (each context that
// loads the module has its own copy of the array).
constexpr int kMaxContexts = 64;
std::mutex g_mutex;
void* g_ctx_key[kMaxContexts] = {};
void* g_scratch_addr[kMaxContexts] = {};

using CtxGetCurrentFn = int (*)(void**);

// The current driver context (CUcontext) as an opaque key; null if none.
void* current_context() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
    }
  });
  void* ctx = nullptr;
  if (fn && fn(&ctx) != 0) ctx = nullptr;
  return ctx;
}

// Resolves the device address of g_scratch in the current context, once.
int scratch_address(int device, unsigned char** out) {
  // The context current to this thread is the one the launch will use. If
  // none is current yet, bind the device's primary context (since CUDA 12
  // cudaSetDevice initialises it).
  void* ctx = current_context();
  if (!ctx) {
    BB_CUDA_TRY(cudaSetDevice(device));
    ctx = current_context();
  }
  if (!ctx) {
    set_error("bb_gemm_run_noalloc: no current CUDA context");
    return BB_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_mutex);
  int slot = -1;
  for (int i = 0; i < kMaxContexts; ++i) {
    if (g_ctx_key[i] == ctx) {
      *out = static_cast<unsigned char*>(g_scratch_addr[i]);
      return BB_OK;
    }
    if (slot < 0 && g_ctx_key[i] == nullptr) slot = i;
  }
  if (slot < 0) {
    set_error("bb_gemm_run_noalloc: more than %d CUDA contexts", kMaxContexts);
    return BB_ERR_UNSUPPORTED;
  }
  void* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ptr, g_scratch);
  if (e != cudaSuccess || ptr == nullptr) {
    return check_cuda(e == cudaSuccess ? cudaErrorInvalidSymbol : e, "cudaGetSymbolAddress(noalloc scratch)");
  }
  g_ctx_key[slot] = ctx;
  g_scratch_addr[slot] = ptr;
  *out = static_cast<unsigned char*>(ptr);
  return BB_OK;
}

}  // namespace gemm_noalloc
}  // namespace bb

extern "C" BB_API int bb_gemm_run_noalloc(int64_t m, int64_t n, int64_t k, int64_t l, const void* a, const void* b,
                                          void* c, int c_dtype, void* stream, int wait) {
  using namespace bb;
  namespace na = bb::gemm_noalloc;
  try {
    clear_error();
    if (m <= 0 || n <= 0 || k <= 0 || l <= 0 || !a || !b || !c) {
      set_error("bb_gemm_run_noalloc: extents must be positive and pointers non-null");
      return BB_ERR_ARGUMENT;
    }
    if (m * l > (int64_t(1) << 31) || n * l > (int64_t(1) << 31) || k > (int64_t(1) << 31)) {
      set_error("bb_gemm_run_noalloc: extents exceed the 32-bit tile coordinate range");
      return BB_ERR_ARGUMENT;
    }
    if (c_dtype != BB_DTYPE_BF16 && c_dtype != BB_DTYPE_F32) {
      set_error("bb_gemm_run_noalloc: C must be BF16 or FP32");
      return BB_ERR_UNSUPPORTED;
    }
    if (k % 8 != 0) {
      set_error("bb_gemm_run_noalloc: K=%lld must be a multiple of 8 (16-byte TMA row stride)", (long long)k);
      return BB_ERR_ARGUMENT;
    }
    if ((c_dtype == BB_DTYPE_BF16 && n % 8 != 0) || (c_dtype == BB_DTYPE_F32 && n % 4 != 0)) {
      set_error("bb_gemm_run_noalloc: N=%lld breaks the 16-byte row stride of C", (long long)n);
      return BB_ERR_ARGUMENT;
    }
    DeviceInfo dev;
    int rc = query_device(&dev);
    if (rc != BB_OK) return rc;
    unsigned char* scratch = nullptr;
    rc = na::scratch_address(dev.device, &scratch);
    if (rc != BB_OK) return rc;

    gemm::Plan p;
    p.m = m;
    p.n = n;
    p.k = k;
    p.l = l;
    p.a = a;
    p.b = b;
    p.c = c;
    p.c_dtype = c_dtype;
    p.stream = static_cast<cudaStream_t>(stream);
    rc = gemm::plan_init(p, BB_VARIANT_TUNED, dev.sm_count);
    if (rc != BB_OK) return rc;
    const size_t partial_bytes = static_cast<size_t>(p.partial_floats) * sizeof(float);
    const size_t counter_bytes = static_cast<size_t>(p.counter_ints) * sizeof(int);
    if (partial_bytes > na::kPartialBytes || counter_bytes > na::kCounterBytes) {
      set_error(
          "bb_gemm_run_noalloc: this problem's stream-K workspace needs %zu bytes of partial tiles and %zu bytes "
          "of counters on this device (%d SMs); the static scratch holds at most %zu and %zu",
          partial_bytes, counter_bytes, dev.sm_count, na::kPartialBytes, na::kCounterBytes);
      return BB_ERR_ARGUMENT;
    }
    rc = gemm::build_maps(p);
    if (rc != BB_OK) return rc;
    p.status = reinterpret_cast<int*>(scratch);
    p.counters = p.counter_ints > 0 ? reinterpret_cast<int*>(scratch + na::kStatusBytes) : nullptr;
    p.partials = p.partial_floats > 0
                     ? reinterpret_cast<float*>(scratch + na::kStatusBytes + na::kCounterBytes)
                     : nullptr;
    // The status word and the counters must start at zero; the partial
    // tiles are always written before they are read.
    BB_CUDA_TRY(cudaMemsetAsync(scratch, 0, na::kStatusBytes + counter_bytes, p.stream));
    // Ordered after the memset by plain stream order.
    p.pdl = false;
    rc = p.launch(p);
    if (rc != BB_OK) return rc;
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
    if (wait) {
      // Synchronous form: wait for the stream and report a device-side wait
      // that gave up (the status word is 4 bytes of the static scratch).
      BB_CUDA_TRY(cudaStreamSynchronize(p.stream));
      int st = 0;
      BB_CUDA_TRY(cudaMemcpy(&st, p.status, sizeof(int), cudaMemcpyDeviceToHost));
      if (st != 0) {
        set_error("bb_gemm_run_noalloc: kernel reported device status 0x%x", st);
        return st == 0x200 ? BB_ERR_INTERNAL : BB_ERR_TIMEOUT;
      }
    }
    return BB_OK;
  } catch (...) {
    bb::set_error("bb_gemm_run_noalloc: unexpected C++ exception");
    return BB_ERR_INTERNAL;
  }
}
