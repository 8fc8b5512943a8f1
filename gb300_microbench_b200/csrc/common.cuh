// Host-side helpers shared by every translation unit of libb200bench.so:
// thread-local last-error text, CUDA status checks that never throw across
// the C ABI, and a lazily resolved cuTensorMapEncodeTiled (obtained through
// cudaGetDriverEntryPoint, so the library links only against cudart).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "../../include/b200bench.h"

namespace bb {

void set_error(const char* fmt, ...);
void clear_error();
const char* last_error();

// Records the CUDA error and returns BB_ERR_CUDA when `e` is not cudaSuccess.
int check_cuda(cudaError_t e, const char* what);

#define BB_CUDA_TRY(call)                                  \
  do {                                                     \
    int rc__ = ::bb::check_cuda((call), #call);            \
    if (rc__ != BB_OK) return rc__;                        \
  } while (0)

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

// Returns nullptr (with the error recorded) when the driver entry point is
// unavailable.
EncodeTiledFn encode_tiled_fn();

// Encodes a tiled tensor map, validating the alignment rules TMA imposes
// (16-byte base, strides multiple of 16 bytes, box inner extent multiple of
// 16 bytes) before calling the driver, so a bad argument becomes
// BB_ERR_ARGUMENT instead of a device fault.
int encode_tiled(CUtensorMap* out, CUtensorMapDataType dtype, int elem_bytes, int rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo);

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int major = 0, minor = 0;
  int smem_optin = 0;
  int smem_per_sm = 0;
  int64_t l2_bytes = 0;
};
int query_device(DeviceInfo* info);

}  // namespace bb
