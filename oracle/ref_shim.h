// Supplies cuda::ptx::elect_sync, which the reference's sources use and CUDA
// 12.9's <cuda/ptx> does not declare. Forced-included before the reference
// translation unit by oracle/Makefile; test infrastructure only.
#pragma once
#include <cuda/ptx>
#include <cstdint>
namespace cuda { namespace ptx {
__device__ inline bool elect_sync(const uint32_t& membermask) {
  uint32_t is_elected = 0;
  asm volatile("{\n\t.reg .pred P;\n\telect.sync _|P, %1;\n\tselp.b32 %0, 1, 0, P;\n\t}"
               : "=r"(is_elected) : "r"(membermask));
  return is_elected != 0;
}
}}  // namespace cuda::ptx
