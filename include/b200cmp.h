/*
 * b200cmp.h - C ABI of libb200cmp.so, the cuBLASLt comparator used beside
 * libb200bench.so's GEMM. It is a library call, not part of the product
 * path; it plays the role of the reference's cuBLASLt bridge
 * (gemm_comparison/cublaslt_bridge.cu) for BF16 A/B with either FP32 D (the
 * reference's frozen descriptor, cublaslt_bridge.cu:75-128) or BF16 D.
 *
 * Problem: D = A * B^T, A (M,K) row-major BF16, B (N,K) row-major BF16,
 * D (M,N) row-major, FP32 compute and scale, alpha = 1, beta = 0.
 * Two descriptor layouts give the same result:
 *   BB_CMP_LAYOUT_REFERENCE  the reference's descriptor: CUBLASLT_ORDER_ROW
 *                            on all four matrices, TRANSA = N, TRANSB = T
 *                            (cublaslt_bridge.cu:75-128);
 *   BB_CMP_LAYOUT_COLUMN     the column-major view D^T = B * A^T
 *                            (TRANSA = T, TRANSB = N, default order).
 * Algorithm policy as in the reference (cublaslt_bridge.cu:40-53): 32
 * heuristic results requested with a 64 MiB workspace limit, best-fit
 * search, the first supported one used, unless autotune is asked for (every
 * supported result timed once, the fastest kept).
 */
#ifndef B200CMP_H_
#define B200CMP_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BB_CMP_API __attribute__((visibility("default")))

enum { BB_CMP_LAYOUT_COLUMN = 0, BB_CMP_LAYOUT_REFERENCE = 1 };

/* Plan metadata, 8-byte fields (the cuBLASLt columns of the reference's
 * CSV, gemm_comparison.py:344-381, and P35PlanInfo, cublaslt_bridge.cu:
 * 156-220). Enum-valued fields hold the cuBLASLt enum values. */
typedef struct bb_cmp_info {
  int64_t layout;
  int64_t cublaslt_version;
  int64_t lda, ldb, ldc, ldd;
  int64_t transa, transb;
  int64_t order_a, order_b, order_c, order_d;
  int64_t type_ab, type_d, compute_type, scale_type, pointer_mode, epilogue, search_mode;
  int64_t workspace_limit_bytes, workspace_bytes;
  int64_t heuristic_requested, heuristic_returned, heuristic_index;
  int64_t alignment_a_bytes, alignment_b_bytes, alignment_c_bytes, alignment_d_bytes;
  int64_t algo_id, tile_id, stages_id, split_k, reduction_scheme, cta_swizzling, custom_option,
      inner_shape_id, cluster_shape_id;
  double waves_count;
  double alpha, beta;
} bb_cmp_info;

typedef struct bb_cmp_plan bb_cmp_plan;

BB_CMP_API int bb_cmp_abi_version(void);
BB_CMP_API size_t bb_cmp_info_size(void);
BB_CMP_API const char* bb_cmp_last_error(void);
/* d_dtype: 1 = BF16, 2 = FP32 (BB_DTYPE_* of b200bench.h). */
BB_CMP_API int bb_cmp_plan_create(int64_t m, int64_t n, int64_t k, const void* a, const void* b, void* d,
                                  int d_dtype, int layout, int autotune, void* stream, bb_cmp_plan** plan,
                                  bb_cmp_info* info);
/* Block-scaled comparator for libb200bench.so's bb_lowp_* GEMM, same
 * operands and D: kind 1 NVFP4 (E2M1 data, VEC16_UE4M3 scales in the
 * 512-byte atom layout, alpha = global_scale), kind 2 FP8 E4M3 with
 * BLK128x128_32F scales, kind 3 plain FP8 E4M3 (no scale tensors, sfa /
 * sfb ignored: a throughput reference for kind 2, not the same function).
 * Returns 5 (unsupported) when this cuBLASLt offers no algorithm for the
 * combination. */
BB_CMP_API int bb_cmp_lowp_plan_create(int kind, int64_t m, int64_t n, int64_t k, const void* a, const void* b,
                                       const void* sfa, const void* sfb, float global_scale, void* d, int autotune,
                                       void* stream, bb_cmp_plan** plan, bb_cmp_info* info);
/* D = alpha * A * B^T + beta * Csrc for later executions (Csrc: D's dtype
 * and layout, may be D; read only when beta != 0). */
BB_CMP_API int bb_cmp_plan_set_epilogue(bb_cmp_plan* plan, float alpha, float beta, const void* c_src);
BB_CMP_API int bb_cmp_execute_n(bb_cmp_plan* plan, int iterations);
BB_CMP_API int bb_cmp_destroy(bb_cmp_plan* plan);

#ifdef __cplusplus
}
#endif

#endif /* B200CMP_H_ */
