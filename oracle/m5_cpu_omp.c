/*
 * m5_cpu_omp.c — multi-threaded CPU restatement of the online W8A8 projection.
 *
 * TEST INFRASTRUCTURE / CPU BASELINE ONLY.  bench.py times it as the second
 * CPU baseline of the headline workload (beside the float64 NumPy port of the
 * reference's own CPU path), and tests/ check it against the single-threaded
 * restatement in m5_oracle.c.  No product code path links, loads or calls it.
 *
 * What it computes (reference file:line, 9Tempest/m5-max-kernels):
 *   per-token INT8 codes     src/m5kernels/numerics.py:29-46 (quantize_reference):
 *                            scale = amax / 127 (1 for an all-zero row),
 *                            q = clip(rint(x / scale), -127, 127), IEEE binary32
 *   W8A8 GEMM + epilogue     src/m5kernels/metal.py:89-98 (row-scaled epilogue):
 *                            acc = exact INT32 sum_k q_a * q_w,
 *                            out = bf16((float(acc) * sa[m]) * sw[n])
 *
 * Rows of the quantizer and output blocks of the GEMM are split over OpenMP
 * threads.  The GEMM keeps 64 x 64 output blocks in a local INT32 buffer and
 * walks K in chunks of 1024, so a chunk of A rows and W rows (64 KB each)
 * stays in the core's caches while its 4 x 4 register blocks run; the inner
 * products use AVX-512 VNNI (vpdpwssd on sign-extended 16-bit lanes) or AVX2
 * (vpmaddwd) when the CPU has them, chosen at run time, else plain C.  Every
 * path produces the exact INT32 sums, so the outputs are identical.
 */
#include <immintrin.h>
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) { /* round to nearest even; finite inputs */
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

int m5c_threads(void) { return omp_get_max_threads(); }

/* Which inner-product kernel m5c_gemm_i8_bf16 uses: 2 AVX-512 VNNI, 1 AVX2, 0 plain C
 * (M5C_SIMD=<level> caps it, so the tests can check every path on one CPU). */
int m5c_simd_level(void) {
  __builtin_cpu_init();
  int level = 0;
  if (__builtin_cpu_supports("avx512bw") && __builtin_cpu_supports("avx512vnni"))
    level = 2;
  else if (__builtin_cpu_supports("avx2"))
    level = 1;
  const char* cap = getenv("M5C_SIMD");
  if (cap && *cap >= '0' && *cap <= '2' && *cap - '0' < level) level = *cap - '0';
  return level;
}

/* Per-token symmetric INT8 codes of bf16 rows x[rows, k]. */
void m5c_quantize_bf16(const uint16_t* x, int64_t rows, int64_t k, int8_t* q, float* s) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const uint16_t* xr = x + r * k;
    float peak = 0.0f;
    for (int64_t i = 0; i < k; ++i) {
      const float v = fabsf(bf16_to_f32(xr[i]));
      if (v > peak) peak = v;
    }
    const float scale = peak == 0.0f ? 1.0f : peak / 127.0f;
    s[r] = scale;
    int8_t* qr = q + r * k;
    for (int64_t i = 0; i < k; ++i) {
      float z = rintf(bf16_to_f32(xr[i]) / scale);
      if (z > 127.0f) z = 127.0f;
      if (z < -127.0f) z = -127.0f;
      qr[i] = (int8_t)(int)z;
    }
  }
}

#define BM 64
#define BN 64
#define KC 1024

/* acc[4][4] += a[4 rows] . b[4 rows] over kn elements (kn % 32 == 0). */
__attribute__((target("avx512bw,avx512vnni"))) static void dot4x4_vnni(
    const int8_t* a, const int8_t* b, int64_t lda, int64_t kn, int32_t acc[4][4]) {
  __m512i c[4][4];
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 4; ++j) c[i][j] = _mm512_setzero_si512();
  for (int64_t k = 0; k < kn; k += 32) {
    __m512i av[4], bv[4];
    for (int i = 0; i < 4; ++i)
      av[i] = _mm512_cvtepi8_epi16(_mm256_loadu_si256((const __m256i*)(a + i * lda + k)));
    for (int j = 0; j < 4; ++j)
      bv[j] = _mm512_cvtepi8_epi16(_mm256_loadu_si256((const __m256i*)(b + j * lda + k)));
    for (int i = 0; i < 4; ++i)
      for (int j = 0; j < 4; ++j) c[i][j] = _mm512_dpwssd_epi32(c[i][j], av[i], bv[j]);
  }
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 4; ++j) acc[i][j] += _mm512_reduce_add_epi32(c[i][j]);
}

static inline int32_t hsum256(__m256i v) __attribute__((target("avx2")));
static inline int32_t hsum256(__m256i v) {
  __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
  s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4E));
  s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xB1));
  return _mm_cvtsi128_si32(s);
}

/* acc[4][4] += over kn elements (kn % 16 == 0), as two 4 x 2 halves (AVX2 has 16 registers). */
__attribute__((target("avx2"))) static void dot4x4_avx2(const int8_t* a, const int8_t* b,
                                                         int64_t lda, int64_t kn,
                                                         int32_t acc[4][4]) {
  for (int jh = 0; jh < 4; jh += 2) {
    __m256i c[4][2];
    for (int i = 0; i < 4; ++i) c[i][0] = c[i][1] = _mm256_setzero_si256();
    for (int64_t k = 0; k < kn; k += 16) {
      __m256i av[4], bv[2];
      for (int i = 0; i < 4; ++i)
        av[i] = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(a + i * lda + k)));
      for (int j = 0; j < 2; ++j)
        bv[j] = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i*)(b + (jh + j) * lda + k)));
      for (int i = 0; i < 4; ++i)
        for (int j = 0; j < 2; ++j)
          c[i][j] = _mm256_add_epi32(c[i][j], _mm256_madd_epi16(av[i], bv[j]));
    }
    for (int i = 0; i < 4; ++i)
      for (int j = 0; j < 2; ++j) acc[i][jh + j] += hsum256(c[i][j]);
  }
}

static void dot4x4_c(const int8_t* a, const int8_t* b, int64_t lda, int64_t kn,
                     int32_t acc[4][4]) {
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 4; ++j) {
      int32_t t = 0;
      for (int64_t k = 0; k < kn; ++k) t += (int32_t)a[i * lda + k] * (int32_t)b[j * lda + k];
      acc[i][j] += t;
    }
}

/*
 * out[m, n] = bf16((float(sum_k a[m, k] * w[n, k]) * sa[m]) * sw[n]) for
 * a [M, K] and w [N, K] INT8 codes (K-major, row stride K).  Requires M, N
 * multiples of 4 (the bench's shapes); any K.
 */
void m5c_gemm_i8_bf16(const int8_t* a, const int8_t* w, int64_t M, int64_t N, int64_t K,
                      const float* sa, const float* sw, uint16_t* out) {
  const int level = m5c_simd_level();
  const int64_t mb = (M + BM - 1) / BM, nb = (N + BN - 1) / BN;
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t blk = 0; blk < mb * nb; ++blk) {
    const int64_t m0 = (blk / nb) * BM, n0 = (blk % nb) * BN;
    const int64_t m1 = m0 + BM < M ? m0 + BM : M, n1 = n0 + BN < N ? n0 + BN : N;
    int32_t acc[BM][BN];
    memset(acc, 0, sizeof(acc));
    for (int64_t k0 = 0; k0 < K; k0 += KC) {
      const int64_t kn = K - k0 < KC ? K - k0 : KC;
      const int64_t kv = level == 2 ? kn & ~(int64_t)31 : level == 1 ? kn & ~(int64_t)15 : 0;
      for (int64_t m = m0; m < m1; m += 4)
        for (int64_t n = n0; n < n1; n += 4) {
          int32_t t[4][4] = {{0}};
          const int8_t* ap = a + m * K + k0;
          const int8_t* bp = w + n * K + k0;
          if (level == 2 && kv)
            dot4x4_vnni(ap, bp, K, kv, t);
          else if (level == 1 && kv)
            dot4x4_avx2(ap, bp, K, kv, t);
          if (kv < kn) dot4x4_c(ap + kv, bp + kv, K, kn - kv, t);
          for (int i = 0; i < 4; ++i)
            for (int j = 0; j < 4; ++j) acc[m - m0 + i][n - n0 + j] += t[i][j];
        }
    }
    for (int64_t m = m0; m < m1; ++m)
      for (int64_t n = n0; n < n1; ++n)
        out[m * N + n] = f32_to_bf16(((float)acc[m - m0][n - n0] * sa[m]) * sw[n]);
  }
}
