/*
 * b200cmp.h - C ABI of libb200cmp.so, the cuBLASLt comparator used beside
 * libb200bench.so's GEMM. It is a library call, not part of the product
 * path; it plays the role of the reference's cuBLASLt bridge
 * (gemm_comparison/cublaslt_bridge.cu) for BF16 A/B with either FP32 D (the
 * reference's frozen descriptor, cublaslt_bridge.cu:75-128) or BF16 D.
 *
 * Layout contract: A (M,K) row-major BF16, B (N,K) row-major BF16,
 * D (M,N) row-major; D = A * B^T, FP32 compute, alpha = 1, beta = 0.
 * Algorithm policy as in the reference (cublaslt_bridge.cu:40-53): up to
 * 32 heuristic results with a 64 MiB workspace limit, the first supported
 * one is used unless bb_cmp_plan_create is asked to autotune.
 */
#ifndef B200CMP_H_
#define B200CMP_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BB_CMP_API __attribute__((visibility("default")))

typedef struct bb_cmp_plan bb_cmp_plan;

BB_CMP_API int bb_cmp_abi_version(void);
BB_CMP_API const char* bb_cmp_last_error(void);
/* d_dtype: 1 = BF16, 2 = FP32 (same codes as BB_DTYPE_*). autotune != 0
 * times every returned heuristic once and keeps the fastest. */
BB_CMP_API int bb_cmp_plan_create(int64_t m, int64_t n, int64_t k, const void* a, const void* b, void* d,
                                  int d_dtype, int autotune, void* stream, bb_cmp_plan** plan);
BB_CMP_API int bb_cmp_execute_n(bb_cmp_plan* plan, int iterations);
/* Index of the heuristic result in use and the number returned. */
BB_CMP_API int bb_cmp_algo_index(const bb_cmp_plan* plan);
BB_CMP_API int bb_cmp_algo_count(const bb_cmp_plan* plan);
BB_CMP_API int64_t bb_cmp_workspace_bytes(const bb_cmp_plan* plan);
BB_CMP_API int bb_cmp_destroy(bb_cmp_plan* plan);

#ifdef __cplusplus
}
#endif

#endif /* B200CMP_H_ */
