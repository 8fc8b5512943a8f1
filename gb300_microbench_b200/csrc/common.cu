#include "common.cuh"

#include <cstring>
#include <mutex>

namespace bb {

namespace {
thread_local char g_last_error[1024] = {0};
}

void set_error(const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  std::vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
  va_end(args);
}

void clear_error() { g_last_error[0] = '\0'; }

const char* last_error() { return g_last_error; }

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return BB_OK;
  set_error("%s failed: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
  return BB_ERR_CUDA;
}

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  if (!fn) set_error("cuTensorMapEncodeTiled is not available from the CUDA driver");
  return fn;
}

int encode_tiled(CUtensorMap* out, CUtensorMapDataType dtype, int elem_bytes, int rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo) {
  if (base == nullptr) {
    set_error("tensor map: null base pointer");
    return BB_ERR_ARGUMENT;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) {
    set_error("tensor map: base pointer %p is not 16-byte aligned", base);
    return BB_ERR_ARGUMENT;
  }
  for (int i = 0; i + 1 < rank; ++i) {
    if (strides_bytes[i] % 16 != 0) {
      set_error("tensor map: stride %d (%llu bytes) is not a multiple of 16", i,
                (unsigned long long)strides_bytes[i]);
      return BB_ERR_ARGUMENT;
    }
  }
  if ((static_cast<uint64_t>(box[0]) * elem_bytes) % 16 != 0) {
    set_error("tensor map: box inner extent %u x %d bytes is not a multiple of 16", box[0], elem_bytes);
    return BB_ERR_ARGUMENT;
  }
  for (int i = 0; i < rank; ++i) {
    if (dims[i] == 0 || box[i] == 0 || box[i] > 256) {
      set_error("tensor map: dim %d = %llu with box %u is invalid", i, (unsigned long long)dims[i], box[i]);
      return BB_ERR_ARGUMENT;
    }
  }
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return BB_ERR_UNSUPPORTED;
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  std::memset(out, 0, sizeof(*out));
  CUresult r = fn(out, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult %d", static_cast<int>(r));
    return BB_ERR_CUDA;
  }
  return BB_OK;
}

int query_device(DeviceInfo* info) {
  // cudaGetDeviceProperties costs milliseconds; properties are cached per
  // device after the first query.
  static std::mutex mu;
  static DeviceInfo cache[64];
  static bool valid[64] = {};
  int dev = 0;
  BB_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64) {
    std::lock_guard<std::mutex> lock(mu);
    if (valid[dev]) {
      *info = cache[dev];
      return BB_OK;
    }
  }
  cudaDeviceProp prop{};
  BB_CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
  DeviceInfo d;
  d.device = dev;
  d.sm_count = prop.multiProcessorCount;
  d.major = prop.major;
  d.minor = prop.minor;
  d.smem_per_sm = static_cast<int>(prop.sharedMemPerMultiprocessor);
  d.l2_bytes = prop.l2CacheSize;
  int optin = 0;
  BB_CUDA_TRY(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  d.smem_optin = optin;
  if (prop.major != 10 || prop.minor != 0) {
    set_error("device %d is compute capability %d.%d; this library is built for sm_100a (10.0) only", dev,
              prop.major, prop.minor);
    return BB_ERR_UNSUPPORTED;
  }
  if (dev >= 0 && dev < 64) {
    std::lock_guard<std::mutex> lock(mu);
    cache[dev] = d;
    valid[dev] = true;
  }
  *info = d;
  return BB_OK;
}

}  // namespace bb

extern "C" {

BB_API int bb_abi_version(void) { return BB_ABI_VERSION; }

BB_API const char* bb_last_error(void) { return bb::last_error(); }

BB_API const char* bb_status_name(int status) {
  switch (status) {
    case BB_OK: return "OK";
    case BB_ERR_ARGUMENT: return "BAD_ARGUMENT";
    case BB_ERR_CUDA: return "CUDA_ERROR";
    case BB_ERR_MISMATCH: return "MISMATCH";
    case BB_ERR_TIMEOUT: return "TIMEOUT";
    case BB_ERR_UNSUPPORTED: return "UNSUPPORTED";
    case BB_ERR_INTERNAL: return "INTERNAL";
    default: return "UNKNOWN";
  }
}

}  // extern "C"
