/*
 * b200bench.h - C ABI of libb200bench.so, the sm_100a (B200) kernels of the
 * gb300-microbench hot path: the dense BF16 GEMM, the HBM->SMEM streaming
 * kernels (LDGSTS and 2D TMA) and the tcgen05 UMMA throughput probes.
 *
 * Conventions (the same ones the reference's native bridge follows,
 * gemm_comparison/cublaslt_bridge.cu:30-38):
 *   - every entry point is extern "C", returns int (BB_OK == 0 on success)
 *     or a plain size / pointer, and lets no C++ exception escape;
 *   - nothing is printed; the reason for a failure is in bb_last_error()
 *     (thread-local);
 *   - an ABI-version and struct-size handshake (bb_abi_version,
 *     bb_gemm_info_size, bb_copy_info_size) lets a ctypes caller refuse a
 *     mismatched library (mirrors p35_bridge_abi_version / p35_plan_info_size,
 *     cublaslt_bridge.cu:525-527);
 *   - device pointers and the CUDA stream are passed as void*; the caller
 *     keeps ownership of every buffer it passes;
 *   - opaque plan handles have create / execute / destroy (mirrors
 *     p35_plan_create / p35_plan_execute / p35_plan_destroy,
 *     cublaslt_bridge.cu:563, 949, 1008).
 */
#ifndef B200BENCH_H_
#define B200BENCH_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BB_API __attribute__((visibility("default")))

#define BB_ABI_VERSION 1

/* Status codes. TIMEOUT means a device-side wait ran out of its budget (the
 * kernel recorded it and returned; the context stays usable). */
enum {
  BB_OK = 0,
  BB_ERR_ARGUMENT = 1,
  BB_ERR_CUDA = 2,
  BB_ERR_MISMATCH = 3,
  BB_ERR_TIMEOUT = 4,
  BB_ERR_UNSUPPORTED = 5,
  BB_ERR_INTERNAL = 6
};

/* ABI handshake; replaces p35_bridge_abi_version (cublaslt_bridge.cu:525). */
BB_API int bb_abi_version(void);
/* Last failure text of the calling thread; replaces p35_last_error. */
BB_API const char* bb_last_error(void);
BB_API const char* bb_status_name(int status);

/* ===================================================================== GEMM
 * C[l] = A[l] * B[l]^T with A (M,K,L) K-major BF16, B (N,K,L) K-major BF16,
 * FP32 accumulation in TMEM, C (M,N,L) N-major in BF16 or FP32.
 * Replaces the CuTe DSL DenseGemmKernel / PersistentDenseGemmKernel the
 * reference configures at gemm_comparison/gemm_comparison.py:209-260 and
 * launches at gemm_comparison.py:2850-2867.
 */
enum { BB_DTYPE_BF16 = 1, BB_DTYPE_F32 = 2 };

/* The three reference candidate slots (gemm_comparison.py:209-245) plus the
 * tuned configuration of this library. */
enum {
  BB_VARIANT_NONPERSISTENT_1CTA = 0, /* 128x128 tiles, 1 CTA, one tile per CTA */
  BB_VARIANT_PERSISTENT_1CTA = 1,    /* 128x128 tiles, 1 CTA, persistent      */
  BB_VARIANT_PERSISTENT_2CTA = 2,    /* 256x128 tiles, CTA pair, persistent   */
  BB_VARIANT_TUNED = 3               /* shape-dependent best configuration    */
};

/* Plan metadata, 16 x 8-byte fields (mirrors the CuTe DSL CSV columns the
 * reference records: gemm_comparison.py:319-429). */
typedef struct bb_gemm_info {
  int64_t mma_tiler_m;         /* rows of one cluster tile (128 or 256)   */
  int64_t mma_tiler_n;         /* columns of one tile                    */
  int64_t cluster_m;           /* CTAs per cluster along M (1 or 2)      */
  int64_t cluster_n;           /* always 1                               */
  int64_t use_2cta_instrs;     /* 1 when tcgen05.mma.cta_group::2        */
  int64_t max_active_clusters; /* clusters resident at once              */
  int64_t stages;              /* shared-memory ring depth               */
  int64_t grid_ctas;           /* CTAs launched                          */
  int64_t num_tiles;           /* output tiles of the problem            */
  int64_t smem_bytes;          /* dynamic shared memory per CTA          */
  int64_t tmem_columns;        /* TMEM columns allocated per CTA         */
  int64_t threads_per_cta;
  int64_t persistent;          /* 1 when CTAs loop over tiles            */
  int64_t raster_group_m;      /* tile-rows per rasterisation group      */
  int64_t c_dtype;             /* BB_DTYPE_*                             */
  int64_t variant;             /* BB_VARIANT_* actually used             */
} bb_gemm_info;

typedef struct bb_gemm_plan bb_gemm_plan;

BB_API size_t bb_gemm_info_size(void);

/* Builds the tensor maps and launch configuration for one problem. `a`, `b`
 * and `c` are device pointers (16-byte aligned; K a multiple of 8 and N a
 * multiple of 8 (BF16 C) or 4 (FP32 C)). `stream` is a cudaStream_t or NULL.
 * Replaces p35_plan_create (cublaslt_bridge.cu:563). */
BB_API int bb_gemm_plan_create(int64_t m, int64_t n, int64_t k, int64_t l, const void* a, const void* b,
                               void* c, int a_dtype, int b_dtype, int c_dtype, int variant, void* stream,
                               bb_gemm_plan** plan, bb_gemm_info* info);
/* One launch on the plan's stream (asynchronous). Replaces p35_plan_execute
 * (cublaslt_bridge.cu:949). */
BB_API int bb_gemm_execute(bb_gemm_plan* plan);
/* `iterations` back-to-back launches (asynchronous); 0 queues nothing,
 * a negative count is BB_ERR_ARGUMENT. */
BB_API int bb_gemm_execute_n(bb_gemm_plan* plan, int iterations);
/* End-to-end call with HOST buffers: copies a_host/b_host into the plan's
 * device A/B, runs the GEMM and copies C back into c_host, then waits for
 * the stream. Host buffers should be pinned for full PCIe bandwidth. */
BB_API int bb_gemm_run_host(bb_gemm_plan* plan, const void* a_host, const void* b_host, void* c_host);
/* Synchronises the plan's stream and reports a device-side wait timeout
 * recorded by any launch so far (BB_ERR_TIMEOUT) or a CUDA error. Replaces
 * the synchronize step of the reference bridge (cublaslt_bridge.cu:987). */
BB_API int bb_gemm_synchronize(bb_gemm_plan* plan);
/* Epilogue of later launches: C = alpha * A * B^T + beta * Csrc, where
 * Csrc (device pointer) has C's dtype and (L, M, N) row-major layout, is
 * 16-byte aligned and may be the plan's own C (in-place accumulate). Csrc is
 * read only when beta != 0 (then it must not be NULL). Defaults: alpha 1,
 * beta 0. The reference bridge exposes alpha / beta through its cuBLASLt
 * descriptor (gemm_comparison/cublaslt_bridge.cu:101-128, fixed to 1 / 0
 * there); this is the same epilogue for the sm_100a kernel. */
BB_API int bb_gemm_plan_set_epilogue(bb_gemm_plan* plan, float alpha, float beta, const void* c_src);
/* Number of kernel launches made through this plan so far. */
BB_API int64_t bb_gemm_launches(const bb_gemm_plan* plan);
/* Replaces p35_plan_destroy (cublaslt_bridge.cu:1008). */
BB_API int bb_gemm_destroy(bb_gemm_plan* plan);

/* GEMM for callers that cannot allocate device memory (code that runs where
 * cudaMalloc is not allowed, such as inside an allocator's callbacks or a
 * host that owns the whole device heap). No counterpart in the reference.
 * The tuned variant's kernel of bb_gemm_plan_create / bb_gemm_execute, but no
 * plan and no allocation: its scratch (the stream-K partial tiles and
 * counters, and the status word) is a static 37 MiB + 64 KiB device array
 * that every GPU loading this library keeps until exit: the most a tuned plan
 * needs on a 148-SM B200. A problem whose workspace would not fit (a device
 * with more SMs) is refused with BB_ERR_ARGUMENT. The first call in a CUDA context resolves the
 * array's address (cudaGetSymbolAddress), so make it before any stream
 * capture. Calls share the array: calls that overlap on the GPU race. With
 * wait != 0 the call synchronises `stream` and reports a device-side wait
 * timeout as BB_ERR_TIMEOUT; with wait == 0 it only queues the work and
 * gives up that report. */
BB_API int bb_gemm_run_noalloc(int64_t m, int64_t n, int64_t k, int64_t l, const void* a, const void* b, void* c,
                               int c_dtype, void* stream, int wait);

/* ============================================================ copy kernels
 * HBM->SMEM streaming read of `bytes` from `src`, 1 CTA per SM. Replaces
 * ldgsts_validate_kernel / ldgsts_benchmark_kernel (memory_paths/ldgsts.cu:
 * 266-373) and tma_validate_kernel / tma_benchmark_kernel
 * (memory_paths/tma.cu:447-602) together with their run_specialization
 * drivers (ldgsts.cu:774-941).
 *
 * The work is cut into tiles of `stage_bytes` (the last one may be short).
 * CTA i owns the contiguous tile range [i*T/G, (i+1)*T/G) and writes into
 * sink[i] the XOR of every 32-bit word it read in the first pass, XORed
 * with each later pass's checksum rotated left by (pass % 32).
 */
enum { BB_COPY_LDGSTS = 0, BB_COPY_TMA = 1 };

typedef struct bb_copy_info {
  int64_t method;
  int64_t stages;
  int64_t bytes_in_flight_kib;   /* requested bytes in flight per SM      */
  int64_t stage_bytes;           /* actual bytes per stage                 */
  int64_t bytes_in_flight;       /* actual: stages * stage_bytes           */
  int64_t copies_per_thread;     /* LDGSTS: 16-byte copies per thread/stage */
  int64_t row_bytes;             /* TMA: box row width in bytes            */
  int64_t tile_rows;             /* TMA: box rows per stage                */
  int64_t threads_per_cta;
  int64_t grid_ctas;
  int64_t smem_bytes;            /* dynamic shared memory reserved per CTA */
  int64_t total_tiles;
  int64_t occupancy_ctas_per_sm; /* benchmark kernel, 0 when not queried   */
  int64_t reserved[3];
} bb_copy_info;

BB_API size_t bb_copy_info_size(void);

/* Host-only geometry: stage_bytes = bif/stages rounded down to the copy
 * granularity (2 KiB for LDGSTS, one `row_bytes` row for TMA); row_bytes
 * is 128 or 256 (TMA only; ignored by LDGSTS). Needs a current device only
 * for grid_ctas (pass sm_count > 0 to skip the query). Replaces make_spec
 * (ldgsts.cu:186-195, tma.cu:252-262). */
BB_API int bb_copy_plan(int method, int stages, int bif_kib, int row_bytes, int64_t bytes, int sm_count,
                        bb_copy_info* info);

/* One timed-path launch (asynchronous). `sink` holds grid_ctas uint32
 * checksums; `status` (may be NULL) receives a device wait timeout code.
 * `rotation` rotates each CTA's starting tile (ldgsts.cu:342). */
BB_API int bb_copy_run(int method, int stages, int bif_kib, int row_bytes, const void* src, int64_t bytes,
                       int64_t passes, int64_t rotation, uint32_t* sink, int* status, void* stream);

/* Validation launch: compares every 16-byte vector against the SplitMix64
 * pattern (ldgsts.cu:220-232) and adds mismatches to *mismatches (device
 * pointer); also writes the one-pass checksums to sink. */
BB_API int bb_copy_validate(int method, int stages, int bif_kib, int row_bytes, const void* src,
                            int64_t bytes, uint32_t* sink, unsigned long long* mismatches, int* status,
                            void* stream);

/* Fills dst with the SplitMix64 pattern: vector i = {lo32(mix(i)),
 * hi32(mix(i)), lo32(mix(i^salt)), hi32(mix(i^salt))}. Replaces
 * init_pattern_kernel (ldgsts.cu:234-240). bytes % 16 == 0. */
BB_API int bb_fill_pattern(void* dst, int64_t bytes, void* stream);
/* Fills dst with uniform 32-bit words: word i = lo32(mix64(seed *
 * 0x9E3779B97F4A7C15 + i)) (the seeded uniform-u32 buffer of the streaming
 * benchmark). bytes % 4 == 0. */
BB_API int bb_fill_uniform_u32(void* dst, int64_t bytes, uint64_t seed, void* stream);

/* ============================================================ UMMA probes
 * DEPTH dependent tcgen05.mma (kind::f16, BF16 in, FP32 TMEM accumulator,
 * shared-memory operands, K = 16) per iteration, `iterations` times; each
 * iteration starts from enable_input_d = 0, so D = depth * A * B^T.
 * cta_group 1: M = 128, one CTA. cta_group 2: M = 256 over a CTA pair.
 * a: M x 16 BF16 row-major, b: N x 16 BF16 row-major (device pointers),
 * d_out: M x N FP32. cycles[0] = %clock64 cycles of the issuing thread
 * around the loop (when timed != 0). launch_ok[0..cta_group-1] = 1 per CTA
 * that accepted its launch geometry. Replaces umma_1sm_body / umma_2sm_body
 * and their extern "C" kernels (umma_throughput/umma_1sm.cu:354-527,
 * umma_2sm.cu:441-731). n in {64,128,256}; depth in {4,16,32,64,128,256}.
 */
BB_API int bb_umma_run(int cta_group, int n, int depth, int64_t iterations, int timed, const void* a,
                       const void* b, float* d_out, unsigned long long* cycles, int* launch_ok, int* status,
                       void* stream);
/* bb_umma_run with the 2-SM loop form chosen: handshake != 0 (cta_group 2
 * only) runs the reference's per-iteration handshake inside the timed loop
 * (each commit arrives on both CTAs' mbarriers, each CTA waits on its own,
 * then a cluster barrier of all threads: umma_2sm.cu:617-659); handshake = 0
 * is bb_umma_run's loop (only the issuing CTA waits per iteration). */
BB_API int bb_umma_run_ex(int cta_group, int n, int depth, int64_t iterations, int timed, int handshake,
                          const void* a, const void* b, float* d_out, unsigned long long* cycles, int* launch_ok,
                          int* status, void* stream);
/* Kernel symbol name of one probe specialisation (e.g.
 * "umma_1sm_m128n256k16_d256"), or NULL. */
BB_API const char* bb_umma_kernel_name(int cta_group, int n, int depth);

/* ======================================================== fault injection
 * Launches a one-warp kernel that waits on an mbarrier nothing will complete,
 * with a wait budget of `budget_ns` per wait, in three forms: one thread
 * (status[0]), the whole warp spinning (status[1]) and the whole warp with
 * the suspend hint (status[2]); each records the BB timeout code in its
 * status int (`status` points at three ints) and the kernel returns after
 * about 3 x budget_ns. Exercises the bounded-wait paths without faulting or
 * hanging the GPU. No counterpart in the reference (its waits are unbounded:
 * memory_paths/tma.cu:399-403). */
BB_API int bb_test_wait_timeout(int64_t budget_ns, int* status, void* stream);

/* Library-wide count of kernels launched through this ABI. */
BB_API int64_t bb_kernel_launches(void);

/* ====================================================== block-scaled GEMM
 * D (M x N, BF16, row-major) = dequant(A) * dequant(B)^T, FP32 accumulate.
 * The reference has no low-precision GEMM; this is its dense GEMM plan
 * interface (bb_gemm_plan_create above, after cublaslt_bridge.cu:563)
 * extended with the two scale operands.
 *
 * BB_LOWP_NVFP4: A (M x K/2 bytes) and B (N x K/2 bytes) hold E2M1 values,
 *   two per byte, element 2i in the low nibble. sfa / sfb hold one UE4M3
 *   scale per 16 K elements as 512-byte atoms: for 128-row block rb and
 *   64-wide K group kg, atom (rb * K/64 + kg); scale j of row r inside it at
 *   byte (r % 32) * 16 + (r / 32) * 4 + j (rows past M / N are padding).
 *   global_scale is the product of the two per-tensor FP32 scales.
 *   K must be a multiple of 256.
 * BB_LOWP_FP8_BLOCK128: A (M x K) and B (N x K) hold E4M3 bytes. sfa is
 *   FP32 [ceil(M/128)][K/128] and sfb FP32 [ceil(N/128)][K/128], one scale
 *   per 128 x 128 block; global_scale multiplies the result (1 for none).
 *   K must be a multiple of 128.
 * N must be a multiple of 8 and every buffer 16-byte aligned. */
enum { BB_LOWP_NVFP4 = 1, BB_LOWP_FP8_BLOCK128 = 2 };

typedef struct bb_lowp_info {
  int64_t kind;
  int64_t tile_m, tile_n, tile_k; /* output tile (of a CTA or CTA pair), K elements per stage */
  int64_t stages;
  int64_t grid_ctas;
  int64_t num_tiles;
  int64_t smem_bytes;
  int64_t tmem_columns;
  int64_t threads_per_cta;
  int64_t cta_group; /* 1: one CTA per tile, 2: CTA pair (cta_group::2) */
  int64_t reserved[5];
} bb_lowp_info;

typedef struct bb_lowp_plan bb_lowp_plan;

BB_API size_t bb_lowp_info_size(void);
/* Bytes of one scale operand (sfa with rows = M, sfb with rows = N), or -1
 * when K does not fit the kind. */
BB_API int64_t bb_lowp_scale_bytes(int kind, int64_t rows, int64_t k);
BB_API int bb_lowp_plan_create(int kind, int64_t m, int64_t n, int64_t k, const void* a, const void* b,
                               const void* sfa, const void* sfb, float global_scale, void* d, void* stream,
                               bb_lowp_plan** plan, bb_lowp_info* info);
BB_API int bb_lowp_execute_n(bb_lowp_plan* plan, int iterations);
/* Waits for the plan's stream; BB_ERR_TIMEOUT if a device wait ran out. */
BB_API int bb_lowp_synchronize(bb_lowp_plan* plan);
BB_API int64_t bb_lowp_launches(const bb_lowp_plan* plan);
BB_API int bb_lowp_destroy(bb_lowp_plan* plan);

#ifdef __cplusplus
}
#endif

#endif /* B200BENCH_H_ */
