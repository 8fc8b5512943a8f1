// Internal plan of the sm_100a GEMM (see gemm_sm100.cu); the C ABI in
// gemm_capi.cu wraps it as the opaque bb_gemm_plan.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace bb {
namespace gemm {

struct Plan {
  int64_t m = 0, n = 0, k = 0, l = 0;
  const void* a = nullptr;
  const void* b = nullptr;
  void* c = nullptr;
  int c_dtype = 0;
  int variant = 0;
  cudaStream_t stream = nullptr;
  CUtensorMap tm_a{}, tm_b{}, tm_c{};
  CUtensorMap tm_b_half{};  // B with half-height boxes (narrow tail items)
  int threads = 0;
  int cg = 1, tile_m = 0, tile_n = 0, stages = 0, smem_bytes = 0, tmem_cols = 0, b_rows = 0, epi_cols = 0;
  int tiles_m = 0, tiles_n = 0, num_tiles = 0, k_blocks = 0, group_m = 8, max_active_clusters = 0, grid = 0;
  bool persistent = true;
  bool stream_k = false;
  bool pdl = true;           // launch with programmatic stream serialisation
  int dp_tiles = 0;          // tiles computed whole (data-parallel)
  int narrow_tiles = 0;      // tail tiles computed as two half-width items
  int sk_tiles = 0;          // tiles of the stream-K region (0: none)
  int sk_snap = 0;           // k-blocks within which a range end snaps to a tile edge
  int64_t partial_floats = 0;  // workspace the stream-K fix-up needs
  int64_t counter_ints = 0;
  float* partials = nullptr;
  int* counters = nullptr;
  int* status = nullptr;  // device word: 0, or the code of a timed-out wait
  // Epilogue D = alpha * acc + beta * c_src (bb_gemm_plan_set_epilogue).
  int epi_mode = 0;
  int spin = 0;  // ring waits that spin (bit 0 producer, bit 1 MMA warp)
  float alpha = 1.0f, beta = 0.0f;
  const void* c_src = nullptr;
  int64_t launches = 0;
  int (*launch)(const Plan&) = nullptr;
};

// Picks the kernel for `variant` and fills the launch geometry (needs m, n,
// k, l, c_dtype set). Returns a BB_* status.
int plan_init(Plan& pl, int variant, int sm_count);

// Encodes the A, B and C tensor maps of a plan whose geometry is set.
int build_maps(Plan& pl);

}  // namespace gemm
}  // namespace bb
