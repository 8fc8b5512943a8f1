// cuBLASLt comparator (library GEMM) for the sm_100a GEMM of
// libb200bench.so; see include/b200cmp.h for the contract.
#include <cublasLt.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "../../include/b200cmp.h"

namespace {
thread_local char g_err[512];
void set_err(const char* what, int code) { std::snprintf(g_err, sizeof(g_err), "%s failed (status %d)", what, code); }
constexpr size_t kWorkspaceLimit = 64ull << 20;
constexpr int kHeuristics = 32;

uint32_t alignment_of(const void* p) {
  const uintptr_t v = reinterpret_cast<uintptr_t>(p);
  uint32_t a = 256;
  while (a > 1 && (v % a) != 0) a >>= 1;
  return a;
}

template <typename T>
int64_t algo_attr(const cublasLtMatmulAlgo_t& algo, cublasLtMatmulAlgoConfigAttributes_t attr) {
  T v{};
  size_t written = 0;
  if (cublasLtMatmulAlgoConfigGetAttribute(&algo, attr, &v, sizeof(v), &written) != CUBLAS_STATUS_SUCCESS) return -1;
  return static_cast<int64_t>(v);
}
}  // namespace

struct bb_cmp_plan {
  cublasLtHandle_t handle = nullptr;
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t la = nullptr, lb = nullptr, ld = nullptr;
  cublasLtMatmulAlgo_t algo{};
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
  const void* first = nullptr;   // cuBLASLt's "A" operand
  const void* second = nullptr;  // cuBLASLt's "B" operand
  void* d = nullptr;
  const void* c = nullptr;  // C source of beta * C (nullptr: D itself)
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

BB_CMP_API int bb_cmp_abi_version(void) { return 2; }
BB_CMP_API size_t bb_cmp_info_size(void) { return sizeof(bb_cmp_info); }
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
                                  int d_dtype, int layout, int autotune, void* stream, bb_cmp_plan** out,
                                  bb_cmp_info* info) {
  try {
    g_err[0] = 0;
    if (!out || m <= 0 || n <= 0 || k <= 0 || (d_dtype != 1 && d_dtype != 2) ||
        (layout != BB_CMP_LAYOUT_COLUMN && layout != BB_CMP_LAYOUT_REFERENCE)) {
      std::snprintf(g_err, sizeof(g_err), "bb_cmp_plan_create: bad argument");
      return 1;
    }
    *out = nullptr;
    bb_cmp_plan* p = new (std::nothrow) bb_cmp_plan();
    if (!p) return 6;
    p->d = d;
    p->stream = static_cast<cudaStream_t>(stream);
    const cudaDataType_t dt = d_dtype == 1 ? CUDA_R_16BF : CUDA_R_32F;
    LT(cublasLtCreate(&p->handle));
    LT(cublasLtMatmulDescCreate(&p->op, CUBLAS_COMPUTE_32F, CUDA_R_32F));
    cublasOperation_t tA, tB;
    int64_t lda, ldb, ldd;
    cublasLtOrder_t order = CUBLASLT_ORDER_COL;
    if (layout == BB_CMP_LAYOUT_REFERENCE) {
      // Row-major A (M x K), op N; row-major B (N x K), op T; row-major D.
      tA = CUBLAS_OP_N;
      tB = CUBLAS_OP_T;
      p->first = a;
      p->second = b;
      lda = k;
      ldb = k;
      ldd = n;
      order = CUBLASLT_ORDER_ROW;
      LT(cublasLtMatrixLayoutCreate(&p->la, CUDA_R_16BF, m, k, lda));
      LT(cublasLtMatrixLayoutCreate(&p->lb, CUDA_R_16BF, n, k, ldb));
      LT(cublasLtMatrixLayoutCreate(&p->ld, dt, m, n, ldd));
      for (cublasLtMatrixLayout_t l : {p->la, p->lb, p->ld}) {
        LT(cublasLtMatrixLayoutSetAttribute(l, CUBLASLT_MATRIX_LAYOUT_ORDER, &order, sizeof(order)));
      }
    } else {
      // D^T (N x M, col-major, ld N) = B (K x N col-major, ld K)^T * A^T (K x M col-major, ld K).
      tA = CUBLAS_OP_T;
      tB = CUBLAS_OP_N;
      p->first = b;
      p->second = a;
      lda = k;
      ldb = k;
      ldd = n;
      LT(cublasLtMatrixLayoutCreate(&p->la, CUDA_R_16BF, k, n, lda));
      LT(cublasLtMatrixLayoutCreate(&p->lb, CUDA_R_16BF, k, m, ldb));
      LT(cublasLtMatrixLayoutCreate(&p->ld, dt, n, m, ldd));
    }
    LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_TRANSA, &tA, sizeof(tA)));
    LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_TRANSB, &tB, sizeof(tB)));
    cublasLtMatmulPreference_t pref = nullptr;
    LT(cublasLtMatmulPreferenceCreate(&pref));
    size_t ws = kWorkspaceLimit;
    cublasStatus_t s =
        cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &ws, sizeof(ws));
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
          ok = cublasLtMatmul(p->handle, p->op, &p->alpha, p->first, p->la, p->second, p->lb, &p->beta, p->d, p->ld,
                              p->d, p->ld, &res[i].algo, p->workspace, max_ws, p->stream) == CUBLAS_STATUS_SUCCESS;
        if (!ok) continue;
        cudaEventRecord(e0, p->stream);
        for (int rep = 0; rep < 5; ++rep)
          cublasLtMatmul(p->handle, p->op, &p->alpha, p->first, p->la, p->second, p->lb, &p->beta, p->d, p->ld, p->d,
                         p->ld, &res[i].algo, p->workspace, max_ws, p->stream);
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
    if (info) {
      std::memset(info, 0, sizeof(*info));
      info->layout = layout;
      info->cublaslt_version = static_cast<int64_t>(cublasLtGetVersion());
      info->lda = lda;
      info->ldb = ldb;
      info->ldc = ldd;
      info->ldd = ldd;
      info->transa = tA;
      info->transb = tB;
      info->order_a = info->order_b = info->order_c = info->order_d = order;
      info->type_ab = CUDA_R_16BF;
      info->type_d = dt;
      info->compute_type = CUBLAS_COMPUTE_32F;
      info->scale_type = CUDA_R_32F;
      info->pointer_mode = CUBLASLT_POINTER_MODE_HOST;
      info->epilogue = CUBLASLT_EPILOGUE_DEFAULT;
      info->search_mode = CUBLASLT_SEARCH_BEST_FIT;
      info->workspace_limit_bytes = static_cast<int64_t>(kWorkspaceLimit);
      info->workspace_bytes = static_cast<int64_t>(max_ws);
      info->heuristic_requested = kHeuristics;
      info->heuristic_returned = found;
      info->heuristic_index = chosen;
      info->alignment_a_bytes = alignment_of(a);
      info->alignment_b_bytes = alignment_of(b);
      info->alignment_c_bytes = alignment_of(d);
      info->alignment_d_bytes = alignment_of(d);
      info->algo_id = algo_attr<int32_t>(p->algo, CUBLASLT_ALGO_CONFIG_ID);
      info->tile_id = algo_attr<uint32_t>(p->algo, CUBLASLT_ALGO_CONFIG_TILE_ID);
      info->stages_id = algo_attr<uint32_t>(p->algo, CUBLASLT_ALGO_CONFIG_STAGES_ID);
      info->split_k = algo_attr<int32_t>(p->algo, CUBLASLT_ALGO_CONFIG_SPLITK_NUM);
      info->reduction_scheme = algo_attr<uint32_t>(p->algo, CUBLASLT_ALGO_CONFIG_REDUCTION_SCHEME);
      info->cta_swizzling = algo_attr<uint32_t>(p->algo, CUBLASLT_ALGO_CONFIG_CTA_SWIZZLING);
      info->custom_option = algo_attr<uint32_t>(p->algo, CUBLASLT_ALGO_CONFIG_CUSTOM_OPTION);
      info->inner_shape_id = algo_attr<uint16_t>(p->algo, CUBLASLT_ALGO_CONFIG_INNER_SHAPE_ID);
      info->cluster_shape_id = algo_attr<uint16_t>(p->algo, CUBLASLT_ALGO_CONFIG_CLUSTER_SHAPE_ID);
      info->waves_count = res[chosen].wavesCount;
      info->alpha = 1.0;
      info->beta = 0.0;
    }
    *out = p;
    return 0;
  } catch (...) {
    std::snprintf(g_err, sizeof(g_err), "bb_cmp_plan_create: exception");
    return 6;
  }
}

BB_CMP_API int bb_cmp_lowp_plan_create(int kind, int64_t m, int64_t n, int64_t k, const void* a, const void* b,
                                       const void* sfa, const void* sfb, float global_scale, void* d, int autotune,
                                       void* stream, bb_cmp_plan** out, bb_cmp_info* info) {
  try {
    g_err[0] = 0;
    if (!out || m <= 0 || n <= 0 || k <= 0 || kind < 1 || kind > 3 || !a || !b || !d ||
        (kind != 3 && (!sfa || !sfb))) {
      std::snprintf(g_err, sizeof(g_err), "bb_cmp_lowp_plan_create: bad argument");
      return 1;
    }
    *out = nullptr;
    bb_cmp_plan* p = new (std::nothrow) bb_cmp_plan();
    if (!p) return 6;
    p->d = d;
    p->stream = static_cast<cudaStream_t>(stream);
    p->alpha = global_scale;
    const cudaDataType_t tab = kind == 1 ? CUDA_R_4F_E2M1 : CUDA_R_8F_E4M3;
    const cublasLtMatmulMatrixScale_t mode =
        kind == 1 ? CUBLASLT_MATMUL_MATRIX_SCALE_VEC16_UE4M3 : CUBLASLT_MATMUL_MATRIX_SCALE_BLK128x128_32F;
    const bool block_scaled = kind != 3;  // kind 3: plain FP8, no scale tensors
    LT(cublasLtCreate(&p->handle));
    LT(cublasLtMatmulDescCreate(&p->op, CUBLAS_COMPUTE_32F, CUDA_R_32F));
    // Column-major view (the only one the narrow types allow, "TN"):
    // D^T (N x M, ld N) = B (K x N, ld K)^T * A (K x M, ld K); cuBLASLt's A is
    // our B with B's scales, its B is our A with A's scales.
    const cublasOperation_t tA = CUBLAS_OP_T, tB = CUBLAS_OP_N;
    p->first = b;
    p->second = a;
    LT(cublasLtMatrixLayoutCreate(&p->la, tab, k, n, k));
    LT(cublasLtMatrixLayoutCreate(&p->lb, tab, k, m, k));
    LT(cublasLtMatrixLayoutCreate(&p->ld, CUDA_R_16BF, n, m, n));
    LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_TRANSA, &tA, sizeof(tA)));
    LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_TRANSB, &tB, sizeof(tB)));
    if (block_scaled) {
      LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_A_SCALE_MODE, &mode, sizeof(mode)));
      LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_B_SCALE_MODE, &mode, sizeof(mode)));
      LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_A_SCALE_POINTER, &sfb, sizeof(sfb)));
      LT(cublasLtMatmulDescSetAttribute(p->op, CUBLASLT_MATMUL_DESC_B_SCALE_POINTER, &sfa, sizeof(sfa)));
    }
    cublasLtMatmulPreference_t pref = nullptr;
    LT(cublasLtMatmulPreferenceCreate(&pref));
    size_t ws = kWorkspaceLimit;
    cublasStatus_t s =
        cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &ws, sizeof(ws));
    std::vector<cublasLtMatmulHeuristicResult_t> res(kHeuristics);
    int found = 0;
    if (s == CUBLAS_STATUS_SUCCESS) {
      s = cublasLtMatmulAlgoGetHeuristic(p->handle, p->op, p->la, p->lb, p->ld, p->ld, pref, kHeuristics, res.data(),
                                         &found);
    }
    cublasLtMatmulPreferenceDestroy(pref);
    if (s != CUBLAS_STATUS_SUCCESS || found == 0) {
      std::snprintf(g_err, sizeof(g_err), "cuBLASLt %d offers no algorithm for this block-scaled GEMM (status %d)",
                    static_cast<int>(cublasLtGetVersion()), static_cast<int>(s));
      bb_cmp_destroy(p);
      return 5;
    }
    size_t max_ws = 0;
    for (int i = 0; i < found; ++i)
      if (res[i].state == CUBLAS_STATUS_SUCCESS && res[i].workspaceSize > max_ws) max_ws = res[i].workspaceSize;
    if (max_ws > 0) CU(cudaMalloc(&p->workspace, max_ws));
    p->workspace_bytes = max_ws;
    int chosen = -1;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (autotune) {
      CU(cudaEventCreate(&e0));
      CU(cudaEventCreate(&e1));
    }
    float best = 1e30f;
    for (int i = 0; i < found; ++i) {
      if (res[i].state != CUBLAS_STATUS_SUCCESS) continue;
      if (!autotune) {
        chosen = i;
        break;
      }
      bool ok = true;
      for (int rep = 0; rep < 3 && ok; ++rep)
        ok = cublasLtMatmul(p->handle, p->op, &p->alpha, p->first, p->la, p->second, p->lb, &p->beta, p->d, p->ld,
                            p->d, p->ld, &res[i].algo, p->workspace, max_ws, p->stream) == CUBLAS_STATUS_SUCCESS;
      if (!ok) continue;
      cudaEventRecord(e0, p->stream);
      for (int rep = 0; rep < 5; ++rep)
        cublasLtMatmul(p->handle, p->op, &p->alpha, p->first, p->la, p->second, p->lb, &p->beta, p->d, p->ld, p->d,
                       p->ld, &res[i].algo, p->workspace, max_ws, p->stream);
      cudaEventRecord(e1, p->stream);
      cudaEventSynchronize(e1);
      float ms = 0;
      cudaEventElapsedTime(&ms, e0, e1);
      if (ms < best) {
        best = ms;
        chosen = i;
      }
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (chosen < 0) {
      std::snprintf(g_err, sizeof(g_err), "no supported cuBLASLt algorithm");
      bb_cmp_destroy(p);
      return 5;
    }
    p->algo = res[chosen].algo;
    if (info) {
      std::memset(info, 0, sizeof(*info));
      info->layout = BB_CMP_LAYOUT_COLUMN;
      info->cublaslt_version = static_cast<int64_t>(cublasLtGetVersion());
      info->lda = k;
      info->ldb = k;
      info->ldc = n;
      info->ldd = n;
      info->transa = tA;
      info->transb = tB;
      info->order_a = info->order_b = info->order_c = info->order_d = CUBLASLT_ORDER_COL;
      info->type_ab = tab;
      info->type_d = CUDA_R_16BF;
      info->compute_type = CUBLAS_COMPUTE_32F;
      info->scale_type = CUDA_R_32F;
      info->pointer_mode = CUBLASLT_POINTER_MODE_HOST;
      info->epilogue = CUBLASLT_EPILOGUE_DEFAULT;
      info->search_mode = CUBLASLT_SEARCH_BEST_FIT;
      info->workspace_limit_bytes = static_cast<int64_t>(kWorkspaceLimit);
      info->workspace_bytes = static_cast<int64_t>(max_ws);
      info->heuristic_requested = kHeuristics;
      info->heuristic_returned = found;
      info->heuristic_index = chosen;
      info->alignment_a_bytes = alignment_of(b);
      info->alignment_b_bytes = alignment_of(a);
      info->alignment_c_bytes = alignment_of(d);
      info->alignment_d_bytes = alignment_of(d);
      info->algo_id = algo_attr<int32_t>(p->algo, CUBLASLT_ALGO_CONFIG_ID);
      info->tile_id = algo_attr<uint32_t>(p->algo, CUBLASLT_ALGO_CONFIG_TILE_ID);
      info->stages_id = algo_attr<uint32_t>(p->algo, CUBLASLT_ALGO_CONFIG_STAGES_ID);
      info->split_k = algo_attr<int32_t>(p->algo, CUBLASLT_ALGO_CONFIG_SPLITK_NUM);
      info->reduction_scheme = algo_attr<uint32_t>(p->algo, CUBLASLT_ALGO_CONFIG_REDUCTION_SCHEME);
      info->cta_swizzling = algo_attr<uint32_t>(p->algo, CUBLASLT_ALGO_CONFIG_CTA_SWIZZLING);
      info->custom_option = algo_attr<uint32_t>(p->algo, CUBLASLT_ALGO_CONFIG_CUSTOM_OPTION);
      info->inner_shape_id = algo_attr<uint16_t>(p->algo, CUBLASLT_ALGO_CONFIG_INNER_SHAPE_ID);
      info->cluster_shape_id = algo_attr<uint16_t>(p->algo, CUBLASLT_ALGO_CONFIG_CLUSTER_SHAPE_ID);
      info->waves_count = res[chosen].wavesCount;
      info->alpha = global_scale;
      info->beta = 0.0;
    }
    *out = p;
    return 0;
  } catch (...) {
    std::snprintf(g_err, sizeof(g_err), "bb_cmp_lowp_plan_create: exception");
    return 6;
  }
}

BB_CMP_API int bb_cmp_plan_set_epilogue(bb_cmp_plan* p, float alpha, float beta, const void* c_src) {
  if (!p || (beta != 0.0f && !c_src)) {
    std::snprintf(g_err, sizeof(g_err), "bb_cmp_plan_set_epilogue: bad argument");
    return 1;
  }
  p->alpha = alpha;
  p->beta = beta;
  p->c = beta != 0.0f ? c_src : nullptr;
  return 0;
}

BB_CMP_API int bb_cmp_execute_n(bb_cmp_plan* p, int iterations) {
  if (!p) return 1;
  const void* c = p->c ? p->c : p->d;
  for (int i = 0; i < iterations; ++i) {
    cublasStatus_t s = cublasLtMatmul(p->handle, p->op, &p->alpha, p->first, p->la, p->second, p->lb, &p->beta, c,
                                      p->ld, p->d, p->ld, &p->algo, p->workspace, p->workspace_bytes, p->stream);
    if (s != CUBLAS_STATUS_SUCCESS) {
      set_err("cublasLtMatmul", static_cast<int>(s));
      return 2;
    }
  }
  return 0;
}

}  // extern "C"
