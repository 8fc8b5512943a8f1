// bb_gemm_run_noalloc: the tuned GEMM for callers that cannot allocate
// device memory, e.g. code running where cudaMalloc is off limits (inside a
// custom allocator's own callbacks, a plugin host that owns the whole device
// heap, or a CUDA-graph-building framework that forbids allocation while it
// records). It is the same kernel as bb_gemm_plan_create/bb_gemm_execute
// with the tuned variant; only where its scratch lives differs.
//
// Scratch: the GEMM's split-tail workspace (partial slices, arrival
// counters) and its device status word live in one file-scope __device__
// array of kScratchBytes (16 MiB + 64 KiB). Every GPU that loads this
// library holds that array until the process exits. The tuned split tail
// needs at most rem * (s - 1) * 256 KiB of partials with rem * s <= 74
// clusters and s in {2, 4} (13.5 MiB at most), so it always fits; a problem
// that would need more is rejected with BB_ERR_ARGUMENT all the same.
// Problems without a split tail need only the status word.
//
// Host code cannot use the array's name as a device address (in host code
// it names a host-side stand-in), so the first call on each device, with
// that device current, resolves the address with cudaGetSymbolAddress and
// caches it. That first call should therefore come before any stream
// capture. Every call then clears the status word and the counters with
// cudaMemsetAsync on the caller's stream and launches the kernel; no call
// allocates or frees device memory. With wait != 0 the call also
// synchronises the stream and returns BB_ERR_TIMEOUT when a device-side wait
// gave up; with wait == 0 it returns as soon as the work is queued. All calls share the one array, which
// keeps the last call's contents: calls that overlap on the GPU (different
// streams without ordering between them) race on it.
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "gemm_sm100.cuh"

namespace bb {
extern std::atomic<int64_t> g_kernel_launches;

namespace gemm_noalloc {

constexpr size_t kStatusBytes = 256;
constexpr size_t kCounterBytes = 64 * 1024 - kStatusBytes;
constexpr size_t kPartialBytes = 16u << 20;
constexpr size_t kScratchBytes = kStatusBytes + kCounterBytes + kPartialBytes;

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
void* g_scratch_addr[kMaxDevices] = {};

// Resolves the device address of g_scratch for the current device, once.
int scratch_address(int device, unsigned char** out) {
  if (device < 0 || device >= kMaxDevices) {
    set_error("bb_gemm_run_noalloc: device index %d out of range", device);
    return BB_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_scratch_addr[device]) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      return check_cuda(e == cudaSuccess ? cudaErrorInvalidSymbol : e, "cudaGetSymbolAddress(noalloc scratch)");
    }
    g_scratch_addr[device] = ptr;
  }
  *out = static_cast<unsigned char*>(g_scratch_addr[device]);
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
    if (k % 8 != 0 || (c_dtype == BB_DTYPE_BF16 && n % 8 != 0) || (c_dtype == BB_DTYPE_F32 && n % 4 != 0)) {
      set_error("bb_gemm_run_noalloc: K must be a multiple of 8 and N keep C rows 16-byte aligned");
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
          "bb_gemm_run_noalloc: this problem's split tail needs %zu bytes of partial storage and %zu bytes of "
          "counters; the static scratch holds at most %zu and %zu",
          partial_bytes, counter_bytes, na::kPartialBytes, na::kCounterBytes);
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
    // slices are always written before they are read.
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
