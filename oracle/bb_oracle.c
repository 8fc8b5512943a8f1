/*
 * bb_oracle.c - CPU restatement of the reference's known-answer algorithms
 * for the gb300-microbench hot path. TEST INFRASTRUCTURE ONLY: the parity
 * tests, __graft_entry__.smoke() and bench.py's CPU-baseline leg call it as
 * the checker; no product code path links or calls it.
 *
 * Parity pinning: the SplitMix64 mixer is checked against SplitMix64's
 * published first output for seed 0 (0xE220A8397B1DCDAF); the UMMA
 * known answer is checked against the reference's own reference_d compiled
 * from umma_throughput/umma_1sm.cu where it lies (oracle/ref_harness.cu);
 * the GEMM input draw against the reference's input helper
 * (tests/golden/make_golden.py).
 */
#include <stdint.h>
#include <string.h>
#include <math.h>

#define BBO_SALT 0xD1B54A32D192ED03ull

/* SplitMix64 finaliser; memory_paths/ldgsts.cu:220-225. */
uint64_t bbo_mix64(uint64_t x) {
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

/* 16-byte pattern vectors vec0 .. vec0+nvec-1 as 4 words each;
 * memory_paths/ldgsts.cu:227-232 (expected_vector). */
void bbo_pattern(uint32_t* out, int64_t vec0, int64_t nvec) {
  for (int64_t i = 0; i < nvec; ++i) {
    const uint64_t idx = (uint64_t)(vec0 + i);
    const uint64_t lo = bbo_mix64(idx);
    const uint64_t hi = bbo_mix64(idx ^ BBO_SALT);
    out[4 * i + 0] = (uint32_t)lo;
    out[4 * i + 1] = (uint32_t)(lo >> 32);
    out[4 * i + 2] = (uint32_t)hi;
    out[4 * i + 3] = (uint32_t)(hi >> 32);
  }
}

/* Seeded uniform words: word i = lo32(mix64(seed * golden + i)). */
void bbo_uniform_u32(uint32_t* out, int64_t word0, int64_t n, uint64_t seed) {
  const uint64_t base = seed * 0x9E3779B97F4A7C15ull;
  for (int64_t i = 0; i < n; ++i) out[i] = (uint32_t)bbo_mix64(base + (uint64_t)(word0 + i));
}

static uint32_t rotl32(uint32_t x, int r) {
  r &= 31;
  return r == 0 ? x : ((x << r) | (x >> (32 - r)));
}

/* Per-CTA checksums of the streaming kernels: CTA g of `grid` owns tiles
 * [g*T/G, (g+1)*T/G) of stage_bytes each (T = ceil(nbytes/stage_bytes)); its
 * checksum is the XOR of its 32-bit words, and pass p (p >= 1) contributes
 * that XOR rotated left by p % 32. (The reference's sink is the XOR of one
 * word per thread per tile, memory_paths/ldgsts.cu:341-369; the checksum
 * here covers every word read.) */
void bbo_copy_checksums(const uint32_t* words, int64_t nbytes, int64_t stage_bytes, int grid, int64_t passes,
                        uint32_t* sink) {
  const int64_t tiles = (nbytes + stage_bytes - 1) / stage_bytes;
  const int64_t nwords = nbytes / 4;
  for (int g = 0; g < grid; ++g) {
    const int64_t t0 = ((int64_t)g * tiles) / grid;
    const int64_t t1 = ((int64_t)(g + 1) * tiles) / grid;
    int64_t w0 = t0 * stage_bytes / 4;
    int64_t w1 = t1 * stage_bytes / 4;
    if (w1 > nwords) w1 = nwords;
    uint32_t x = 0;
    for (int64_t w = w0; w < w1; ++w) x ^= words[w];
    uint32_t total = 0;
    for (int64_t p = 0; p < passes; ++p) total ^= rotl32(x, (int)p);
    sink[g] = total;
  }
}

/* XOR of every word of the buffer (checksum of checksums for one pass). */
uint32_t bbo_xor_all(const uint32_t* words, int64_t nwords) {
  uint32_t x = 0;
  for (int64_t i = 0; i < nwords; ++i) x ^= words[i];
  return x;
}

/* UMMA known answer, pattern mode: umma_1sm.cu:566-575 (reference_a/b/d),
 * with the global row for the 2-SM probe (umma_2sm.cu:778). */
static int32_t ref_a(int row, int k) { return ((row + 3 * k) % 7) - 3; }
static int32_t ref_b(int k, int col) { return ((2 * k + col) % 5) - 2; }
double bbo_umma_reference_d(int row, int col, int depth) {
  int64_t sum = 0;
  for (int k = 0; k < 16; ++k) sum += (int64_t)ref_a(row, k) * (int64_t)ref_b(k, col);
  return (double)depth * (double)sum;
}

static float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* D[r, c] = depth * sum_k A[r, k] * B[c, k] in double, for BF16 operands
 * A (m x 16) and B (n x 16) stored row-major. */
void bbo_umma_expected(const uint16_t* a, const uint16_t* b, int m, int n, int depth, double* d) {
  for (int r = 0; r < m; ++r)
    for (int c = 0; c < n; ++c) {
      double s = 0.0;
      for (int k = 0; k < 16; ++k) s += (double)bf16_to_f32(a[r * 16 + k]) * (double)bf16_to_f32(b[c * 16 + k]);
      d[(int64_t)r * n + c] = (double)depth * s;
    }
}

/* C = A * B^T for BF16 A (m x k) and B (n x k), accumulated in double and
 * rounded to float: the reference's FP32 oracle (gemm_comparison.py:
 * 2698-2715) with a more accurate accumulation, for small shapes. */
void bbo_gemm_ref(const uint16_t* a, const uint16_t* b, float* c, int64_t m, int64_t n, int64_t k) {
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) {
      double s = 0.0;
      const uint16_t* ar = a + i * k;
      const uint16_t* br = b + j * k;
      for (int64_t t = 0; t < k; ++t) s += (double)bf16_to_f32(ar[t]) * (double)bf16_to_f32(br[t]);
      c[i * n + j] = (float)s;
    }
}

/* Elementwise check of gemm_comparison.py:2718-2755: |c - ref| <= atol +
 * rtol * |ref| for every element, all finite; max abs error and max relative
 * error with a denominator floor of `floor`. Returns the mismatch count, or
 * -1 when c holds a non-finite value. */
int64_t bbo_validate_elementwise(const float* c, const float* ref, int64_t n, double atol, double rtol, double floor,
                                 double* max_abs, double* max_rel) {
  int64_t bad = 0;
  double ma = 0.0, mr = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    if (!isfinite(c[i])) return -1;
    const double d = fabs((double)c[i] - (double)ref[i]);
    const double r = fabs((double)ref[i]);
    if (d > atol + rtol * r) ++bad;
    if (d > ma) ma = d;
    const double den = r > floor ? r : floor;
    if (d / den > mr) mr = d / den;
  }
  *max_abs = ma;
  *max_rel = mr;
  return bad;
}
