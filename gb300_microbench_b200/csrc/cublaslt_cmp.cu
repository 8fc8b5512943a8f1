// cuBLASLt comparator (library GEMM) for the sm_100a GEMM of
// libb200bench.so. Row-major D = A * B^T is expressed in cuBLASLt's
// column-major terms as D^T (N x M) = B (N x K, col-major view K x N
// transposed) * A^T: op(A_lt) = T on the K x N buffer of B, op(B_lt) = N on
// the K x M buffer of A.
#include <cublasLt.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <new>
#include <vector>

#include "../../include/b200cmp.h"

namespace {
thread_local char g_err[512];
void set_err(const char* what, int code) { std::snprintf(g_err, sizeof(g_err), "%s failed (status %d)", what, code); }
constexpr size_t kWorkspaceLimit = 64ull << 20;
constexpr int kHeuristics = 32;
}  // namespace

struct bb_cmp_plan {
  cublasLtHandle_t handle = nullptr;
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t la = nullptr, lb = nullptr, ld = nullptr;
  cublasLtMatmulAlgo_t algo{};
  int algo_index = -1, algo_count = 0;
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
  const void* a = nullptr;
  const void* b = nullptr;
  void* d = nullptr;
  cudaStream_t stream = nullptr;
  float alpha = 1.0f, beta = 0.0f;
};

#define LT(call)                              \
  do {                                        \
    cublasStatus_t s__ = (call);              \
    if (s__ != CUBLAS_STATUS_SUCCESS) {       \
      set_err(#call, static_cast<int>(s__));  \
      bb_cmp_destroy(p);                      \
      return 2;                               \
    }                                         \
  } while (0)
#define CU(call)                              \
  do {                                        \
    cudaError_t e__ = (call);                 \
    if (e__ != cudaSuccess) {                 \
      set_err(#call, static_cast<int>(e__));  \
      bb_cmp_destroy(p);                      \
      return 2;                               \
    }                                         \
  } while (0)

extern "C" {

BB_CMP_API int bb_cmp_abi_version(void) { return 1; }
BB_CMP_API const char* bb_cmp_last_error(void) { return g_err; }

BB_CMP_API int bb_cmp_destroy(bb_cmp_plan* p) {
  if (!p) return 0;
  if (p->workspace) cudaFree(p->workspace);
  if (p->ld) cublasLtMatrixLayoutDestroy(p->ld);
  if (p->lb) cublasLtMatrixLayoutDestroy(p->lb);
  if (p->la) cublasLtMatrixLayoutDestroy(p->la);
  if (p->op) cublasLtMatmulDescDestroy(p->op);
  if (p->handle) cublasLtDestroy(p->handle);
  delete p;
  return 0;
}

BB_CMP_API int bb_cmp_plan_create(int64_t m, int64_t n, int64_t k, const void* a, const void* b, void* d,
                                  int d_dtype, int autotune, void* stream, bb_cmp_plan** out) {
  try {
    g_err[0] = 0;
    if (!out || m <= 0 || n <= 0 || k <= 0 || (d_dtype != 1 && d_dtype != 2)) {
      std::snprintf(g_err, sizeof(g_err), "bb_cmp_plan_create: bad argument");
      return 1;
    }
    *out = nullptr;
    bb_cmp_plan* p = new (std::nothrow) bb_cmp_plan();
    if (!p) return 6;
    p->a = a;
    p->b = b;
    p->d = d;
    p->stream = static_cast<cudaStream_t>(stream);
    const cudaDataType_t dt = d_dtype == 1 ? CUDA_R_16BF : CUDA_R_32F;
    LT(cublasLtCreate(&p->handle));
    LT(cublasLtMatmulDescCreate(&p->op, CUBLAS_COMPUTE_32F, CUDA_R_32F));
    const cublasOperation_t tA = CUBLAS_OP_T, tB = CUBLAS_OP_N;
    LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_TRANSA, &tA, sizeof(tA)));
    LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_TRANSB, &tB, sizeof(tB)));
    // "A" of cuBLASLt = our B buffer (K x N col-major, ld K), transposed.
    LT(cublasLtMatrixLayoutCreate(&p->la, CUDA_R_16BF, k, n, k));
    // "B" of cuBLASLt = our A buffer (K x M col-major, ld K).
    LT(cublasLtMatrixLayoutCreate(&p->lb, CUDA_R_16BF, k, m, k));
    // D^T: N x M col-major, ld N == our row-major M x N.
    LT(cublasLtMatrixLayoutCreate(&p->ld, dt, n, m, n));
    cublasLtMatmulPreference_t pref = nullptr;
    LT(cublasLtMatmulPreferenceCreate(&pref));
    size_t ws = kWorkspaceLimit;
    cublasStatus_t s = cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &ws, sizeof(ws));
    std::vector<cublasLtMatmulHeuristicResult_t> res(kHeuristics);
    int found = 0;
    if (s == CUBLAS_STATUS_SUCCESS) {
      s = cublasLtMatmulAlgoGetHeuristic(p->handle, p->op, p->la, p->lb, p->ld, p->ld, pref, kHeuristics, res.data(),
                                         &found);
    }
    cublasLtMatmulPreferenceDestroy(pref);
    if (s != CUBLAS_STATUS_SUCCESS || found == 0) {
      set_err("cublasLtMatmulAlgoGetHeuristic", static_cast<int>(s));
      bb_cmp_destroy(p);
      return 2;
    }
    p->algo_count = found;
    size_t max_ws = 0;
    for (int i = 0; i < found; ++i)
      if (res[i].state == CUBLAS_STATUS_SUCCESS && res[i].workspaceSize > max_ws) max_ws = res[i].workspaceSize;
    if (max_ws > 0) CU(cudaMalloc(&p->workspace, max_ws));
    p->workspace_bytes = max_ws;
    int chosen = -1;
    if (!autotune) {
      for (int i = 0; i < found; ++i)
        if (res[i].state == CUBLAS_STATUS_SUCCESS) {
          chosen = i;
          break;
        }
    } else {
      cudaEvent_t e0, e1;
      CU(cudaEventCreate(&e0));
      CU(cudaEventCreate(&e1));
      float best = 1e30f;
      for (int i = 0; i < found; ++i) {
        if (res[i].state != CUBLAS_STATUS_SUCCESS) continue;
        bool ok = true;
        for (int rep = 0; rep < 3 && ok; ++rep)
          ok = cublasLtMatmul(p->handle, p->op, &p->alpha, p->b, p->la, p->a, p->lb, &p->beta, p->d, p->ld, p->d,
                              p->ld, &res[i].algo, p->workspace, max_ws, p->stream) == CUBLAS_STATUS_SUCCESS;
        if (!ok) continue;
        cudaEventRecord(e0, p->stream);
        for (int rep = 0; rep < 5; ++rep)
          cublasLtMatmul(p->handle, p->op, &p->alpha, p->b, p->la, p->a, p->lb, &p->beta, p->d, p->ld, p->d, p->ld,
                         &res[i].algo, p->workspace, max_ws, p->stream);
        cudaEventRecord(e1, p->stream);
        cudaEventSynchronize(e1);
        float ms = 0;
        cudaEventElapsedTime(&ms, e0, e1);
        if (ms < best) {
          best = ms;
          chosen = i;
        }
      }
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
    }
    if (chosen < 0) {
      std::snprintf(g_err, sizeof(g_err), "no supported cuBLASLt algorithm");
      bb_cmp_destroy(p);
      return 5;
    }
    p->algo = res[chosen].algo;
    p->algo_index = chosen;
    *out = p;
    return 0;
  } catch (...) {
    std::snprintf(g_err, sizeof(g_err), "bb_cmp_plan_create: exception");
    return 6;
  }
}

BB_CMP_API int bb_cmp_execute_n(bb_cmp_plan* p, int iterations) {
  if (!p) return 1;
  for (int i = 0; i < iterations; ++i) {
    cublasStatus_t s = cublasLtMatmul(p->handle, p->op, &p->alpha, p->b, p->la, p->a, p->lb, &p->beta, p->d, p->ld,
                                      p->d, p->ld, &p->algo, p->workspace, p->workspace_bytes, p->stream);
    if (s != CUBLAS_STATUS_SUCCESS) {
      set_err("cublasLtMatmul", static_cast<int>(s));
      return 2;
    }
  }
  return 0;
}

BB_CMP_API int bb_cmp_algo_index(const bb_cmp_plan* p) { return p ? p->algo_index : -1; }
BB_CMP_API int bb_cmp_algo_count(const bb_cmp_plan* p) { return p ? p->algo_count : -1; }
BB_CMP_API int64_t bb_cmp_workspace_bytes(const bb_cmp_plan* p) { return p ? static_cast<int64_t>(p->workspace_bytes) : -1; }

}  // extern "C"
