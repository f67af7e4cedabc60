/*
 * m5_oracle.c — CPU restatement of the quantized-projection hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: tests/, the smoke()
 * entry point and bench.py's CPU-baseline leg are the only callers.  No
 * product code path links, loads or calls it.
 *
 * What it restates (reference file:line, 9Tempest/m5-max-kernels):
 *   per-token INT8 / E4M3 quantization   src/m5kernels/numerics.py:29-46 (quantize_reference),
 *                                          numerics.py:17-26 (fp8_encode)
 *   signed block Hadamard X D H          src/m5kernels/hadamard_reference.py:26-68,
 *                                          shaders/hadamard.metal:1-26
 *   norm + AdaLN modulation              src/m5kernels/norm_hadamard_reference.py:24-64,
 *                                          shaders/norm_hadamard.metal:1-121
 *   gated residual update                src/m5kernels/gated_residual_reference.py:21-60,
 *                                          norm_hadamard.py:62-70
 *   W8A8 GEMM + scale/bias/gate epilogue src/m5kernels/metal.py:89-128
 *   Q/K RMSNorm + split-half RoPE        src/m5kernels/qk_rope_reference.py:45-134,
 *                                          shaders/qk_rope_body.metal:1-20
 *   RMS scale-folding INT8 preparation   src/m5kernels/rms_quant_reference.py:24-89,
 *                                          rms_quant.py:41-117, shaders/rms_quant.metal:1-97
 *
 * The reference's own references are float64; its GPU kernels round in FP32
 * with an unspecified reduction order, which is why the reference accepts a
 * one-code difference.  This restatement instead fixes the FP32 order so it is
 * bit-comparable with the CUDA kernels:
 *   - row reductions: the row is cut into 16-element chunks [16 c, 16 c + 16)
 *     (elements past K count as zero).  A chunk is eight pairs
 *     p_k = (x_2k, x_2k+1); pairs combine as L1_j = p_2j (+) p_2j+1 -- for
 *     squares fmaf(u_2j, u_2j, u_2j+1 * u_2j+1) with u = x or x - mean --
 *     then (L1_0 + L1_1) + (L1_2 + L1_3), each step on both halves of the
 *     pair, and the chunk is the pair's even half + odd half.  The chunk sums
 *     of a row combine as a pairwise tree over chunk index (c0 + c1, c2 + c3,
 *     ..., then pairs of pairs), padded with zero chunks to a power of two,
 *     and the total is added to +0 (kernels may pad the tree further);
 *     The tree does not depend on how a kernel splits the row among threads
 *     and warps, so every schedule (16 or 64 elements per thread) forms it;
 *     the centered LayerNorm pass uses u = x - mean, rounded once;
 *   - Hadamard butterflies in natural Sylvester order with increasing stride,
 *     then one multiply by fp32(1/sqrt(B));
 *   - every other operation is a single IEEE-754 binary32 operation in the
 *     order written (compile with -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define O_F32 0
#define O_F16 1
#define O_BF16 2

#define NORM_NONE 0
#define NORM_RMS 1
#define NORM_LAYER 2

#define OUT_INT8 0
#define OUT_E4M3 1
#define OUT_F32 2


/* ------------------------------------------------------------------ dtypes */
static float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static uint16_t f32_to_bf16(float f) { /* round to nearest even; inputs are finite */
  uint32_t u;
  memcpy(&u, &f, 4);
  uint32_t rounding = 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)((u + rounding) >> 16);
}

static float f16_to_f32(uint16_t h) {
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}

static uint16_t f32_to_f16(float f) {
  _Float16 v = (_Float16)f; /* IEEE round to nearest even */
  uint16_t h;
  memcpy(&h, &v, 2);
  return h;
}

static float load_elem(const void* base, int dtype, int64_t i) {
  switch (dtype) {
    case O_BF16: return bf16_to_f32(((const uint16_t*)base)[i]);
    case O_F16: return f16_to_f32(((const uint16_t*)base)[i]);
    default: return ((const float*)base)[i];
  }
}

static void store_elem(void* base, int dtype, int64_t i, float v) {
  switch (dtype) {
    case O_BF16: ((uint16_t*)base)[i] = f32_to_bf16(v); break;
    case O_F16: ((uint16_t*)base)[i] = f32_to_f16(v); break;
    default: ((float*)base)[i] = v; break;
  }
}

static float round_through(float v, int dtype) {
  switch (dtype) {
    case O_BF16: return bf16_to_f32(f32_to_bf16(v));
    case O_F16: return f16_to_f32(f32_to_f16(v));
    default: return v;
  }
}

/* ------------------------------------------------------------------ codes */
static int8_t int8_code(float v, float scale) {
  float z = rintf(v / scale);
  if (z > 127.0f) z = 127.0f;
  if (z < -127.0f) z = -127.0f;
  return (int8_t)(int)z;
}

/* OCP E4M3 (finite-only "fn" variant): RNE, saturate to 448 (code 0x7E). */
uint8_t m5o_e4m3_encode(float z) {
  const uint8_t sign = signbit(z) ? 0x80 : 0x00;
  const float a = fabsf(z);
  if (!(a < 448.0f)) return sign | 0x7E;
  if (a < 0.015625f) { /* subnormal range: step 2^-9; code 8 is the first normal */
    const float m = rintf(a * 512.0f);
    return sign | (uint8_t)(int)m;
  }
  int e2;
  const float f = frexpf(a, &e2); /* a = f * 2^e2, f in [0.5, 1) */
  int exp = e2 - 1;              /* a = (2f) * 2^exp, 2f in [1, 2) */
  float t = rintf(ldexpf(f, 4)); /* mantissa in eighths: [8, 16] */
  if (t == 16.0f) {
    t = 8.0f;
    exp += 1;
  }
  int code = ((exp + 7) << 3) | ((int)t - 8);
  if (code > 0x7E) code = 0x7E;
  return sign | (uint8_t)code;
}

static uint8_t e4m3_code(float v, float scale) { return m5o_e4m3_encode(v / scale); }

/* ------------------------------------------------------------------ layout */
/* Sum of f(v[j]) over one row in the canonical order.  kind 0: sum of v,
 * kind 1: sum of v*v, kind 2: sum of (v-mean)^2; squares of a pair of
 * elements as fmaf(u0, u0, u1 * u1). */
#define RCHUNK 16
static float chunk16(const float* v, int64_t j0, int64_t K, int kind, float mean) {
  float u[RCHUNK];
  for (int i = 0; i < RCHUNK; ++i) {
    const int64_t j = j0 + i;
    float x = j < K ? v[j] : 0.0f;
    if (kind == 2) x = j < K ? x - mean : 0.0f;
    u[i] = x;
  }
  float l1[4][2];
  for (int jj = 0; jj < 4; ++jj)
    for (int h = 0; h < 2; ++h) {
      const float a = u[4 * jj + h], b = u[4 * jj + 2 + h];
      if (kind == 0) {
        l1[jj][h] = a + b;
      } else {
        const float bb = b * b;
        l1[jj][h] = fmaf(a, a, bb);
      }
    }
  float pe = (l1[0][0] + l1[1][0]) + (l1[2][0] + l1[3][0]);
  float po = (l1[0][1] + l1[1][1]) + (l1[2][1] + l1[3][1]);
  return pe + po;
}

static float row_reduce(const float* v, int64_t K, int kind, float mean) {
  const int64_t n = (K + RCHUNK - 1) / RCHUNK;
  int64_t np2 = 1;
  while (np2 < n) np2 <<= 1;
  float* s = (float*)malloc((size_t)np2 * sizeof(float));
  for (int64_t c = 0; c < np2; ++c) s[c] = c < n ? chunk16(v, c * RCHUNK, K, kind, mean) : 0.0f;
  for (int64_t len = np2; len > 1; len >>= 1)
    for (int64_t c = 0; c < len / 2; ++c) s[c] = s[2 * c] + s[2 * c + 1];
  const float total = s[0] + 0.0f; /* -0 -> +0: kernels may pad the tree further */
  free(s);
  return total;
}

static void fwht_block(float* v, int B) {
  for (int h = 1; h < B; h <<= 1)
    for (int i = 0; i < B; ++i)
      if ((i & h) == 0) {
        const float lo = v[i], hi = v[i + h];
        v[i] = lo + hi;
        v[i + h] = lo - hi;
      }
}

/*
 * One call = the row-preparation kernel over all rows.  Pointers are host
 * arrays with the same meaning as RowPrepArgs in the CUDA library.  `block`
 * 0 means no rotation; `norm` NORM_NONE skips normalization/modulation.
 */
void m5o_row_prep(const void* x, int x_dtype, const void* branch, const void* gate,
                  int gate_dtype, const int32_t* gate_row_map, const void* gamma,
                  int gamma_dtype, const void* scale, int scale_dtype, const void* shift,
                  int shift_dtype, const int32_t* row_map, const int8_t* signs, int64_t rows,
                  int64_t K, int norm, float eps, int round_output, int block, int out, void* q,
                  float* s, float* y, void* r_out) {
  float* v = (float*)malloc(sizeof(float) * (size_t)K);
  const float inv_sqrt_block = block > 0 ? (float)(1.0 / sqrt((double)block)) : 1.0f;
  for (int64_t r = 0; r < rows; ++r) {
    /* load, gated residual update */
    const int64_t goff = (gate && gate_row_map) ? (int64_t)gate_row_map[r] * K : 0;
    for (int64_t j = 0; j < K; ++j) {
      float xv = load_elem(x, x_dtype, r * K + j);
      if (branch) {
        const float b = load_elem(branch, x_dtype, r * K + j);
        const float g = load_elem(gate, gate_dtype, goff + j);
        xv = round_through(fmaf(b, g, xv), x_dtype);
        store_elem(r_out, x_dtype, r * K + j, xv);
      }
      v[j] = xv;
    }
    /* statistics */
    float mean = 0.0f, inv = 1.0f;
    if (norm != NORM_NONE) {
      const float kf = (float)K;
      const float first =
          row_reduce(v, K, norm == NORM_LAYER ? 0 : 1, 0.0f) / kf;
      float moment = first;
      if (norm == NORM_LAYER) {
        mean = first;
        moment = row_reduce(v, K, 2, mean) / kf;
      }
      inv = 1.0f / sqrtf(moment + eps);
    }
    /* modulation, rounding, signs */
    const int64_t moff = row_map ? (int64_t)row_map[r] * K : 0;
    for (int64_t j = 0; j < K; ++j) {
      float t = v[j];
      if (norm != NORM_NONE) {
        const float g = load_elem(gamma, gamma_dtype, j);
        const float sc = load_elem(scale, scale_dtype, moff + j);
        const float sh = load_elem(shift, shift_dtype, moff + j);
        const float n = ((t - mean) * inv) * g;
        t = fmaf(n, 1.0f + sc, sh);
        if (round_output) t = round_through(t, x_dtype);
      }
      if (signs && signs[j] < 0) t = -t;
      v[j] = t;
    }
    /* rotation */
    if (block > 0) {
      for (int64_t b0 = 0; b0 < K; b0 += block) fwht_block(v + b0, block);
      for (int64_t j = 0; j < K; ++j) v[j] = v[j] * inv_sqrt_block;
    }
    if (out == OUT_F32) {
      memcpy(y + r * K, v, sizeof(float) * (size_t)K);
      continue;
    }
    float peak = 0.0f;
    for (int64_t j = 0; j < K; ++j) peak = fmaxf(peak, fabsf(v[j]));
    const float qmax = out == OUT_E4M3 ? 448.0f : 127.0f;
    const float sc = peak == 0.0f ? 1.0f : peak / qmax;
    s[r] = sc;
    uint8_t* qrow = (uint8_t*)q + r * K;
    for (int64_t j = 0; j < K; ++j)
      qrow[j] = out == OUT_E4M3 ? e4m3_code(v[j], sc) : (uint8_t)int8_code(v[j], sc);
  }
  free(v);
}

/*
 * RMS preparation with the inverse RMS folded into the row scale (fold != 0)
 * or applied before gamma (fold == 0), INT8 codes only.  gamma is fp32[K],
 * signs int8[K] (+-1), block 0 = no rotation.  Per row:
 *   r = 1 / sqrt(sum(x^2) / K + eps), sum in the canonical order;
 *   u_j = (x_j * gamma_j) * sign_j          (fold)
 *   u_j = ((x_j * r) * gamma_j) * sign_j    (direct)
 *   u = blockwise Hadamard butterflies, then * fp32(1/sqrt(block));
 *   peak = max |u|; scale = peak == 0 ? 1 : (peak * r) / 127 (fold) or
 *   peak / 127 (direct); q_j = peak == 0 ? 0 : clip(rint((u_j / peak) * 127)).
 */
void m5o_rms_quantize(const void* x, int x_dtype, const float* gamma, const int8_t* signs,
                      int64_t rows, int64_t K, int block, int fold, float eps, int8_t* q,
                      float* s) {
  float* v = (float*)malloc(sizeof(float) * (size_t)K);
  const float inv_sqrt_block = block > 0 ? (float)(1.0 / sqrt((double)block)) : 1.0f;
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t j = 0; j < K; ++j) v[j] = load_elem(x, x_dtype, r * K + j);
    const float moment = row_reduce(v, K, 1, 0.0f) / (float)K;
    const float inv = 1.0f / sqrtf(moment + eps);
    for (int64_t j = 0; j < K; ++j) {
      float t = fold ? v[j] : v[j] * inv;
      t = t * gamma[j];
      if (signs && signs[j] < 0) t = -t;
      v[j] = t;
    }
    if (block > 0) {
      for (int64_t b0 = 0; b0 < K; b0 += block) fwht_block(v + b0, block);
      for (int64_t j = 0; j < K; ++j) v[j] = v[j] * inv_sqrt_block;
    }
    float peak = 0.0f;
    for (int64_t j = 0; j < K; ++j) peak = fmaxf(peak, fabsf(v[j]));
    s[r] = peak == 0.0f ? 1.0f : (peak * (fold ? inv : 1.0f)) / 127.0f;
    for (int64_t j = 0; j < K; ++j) {
      float c = 0.0f;
      if (peak != 0.0f) c = rintf((v[j] / peak) * 127.0f);
      if (c > 127.0f) c = 127.0f;
      if (c < -127.0f) c = -127.0f;
      q[r * K + j] = (int8_t)(int)c;
    }
  }
  free(v);
}

/* ------------------------------------------------------------------ MXINT8 */
/* 32-element blocks of each row (k % 32 == 0): e = clip(floor(log2(peak)) - 6,
 * -127, 127) (0 for an all-zero block), q = clip(rint(x / 2^e), +-127),
 * byte = e + 127 (numerics.py:32-40).  floor(log2(peak)) is the exact binary
 * exponent of the fp32 peak (frexpf), and x / 2^e an exact power-of-two
 * scaling (ldexpf). */
void m5o_quantize_mxint8(const void* x, int x_dtype, int64_t rows, int64_t k, int8_t* q,
                         uint8_t* ebytes) {
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t b = 0; b < k / 32; ++b) {
      const int64_t base = r * k + b * 32;
      float peak = 0.0f;
      for (int i = 0; i < 32; ++i) {
        const float v = fabsf(load_elem(x, x_dtype, base + i));
        if (v > peak) peak = v;
      }
      int e = 0;
      if (peak > 0.0f) {
        int ex = 0;
        (void)frexpf(peak, &ex); /* peak = m * 2^ex, m in [0.5, 1) */
        e = (ex - 1) - 6;
        if (e < -127) e = -127;
        if (e > 127) e = 127;
      }
      ebytes[r * (k / 32) + b] = (uint8_t)(e + 127);
      for (int i = 0; i < 32; ++i) {
        float z = rintf(ldexpf(load_elem(x, x_dtype, base + i), -e));
        if (z > 127.0f) z = 127.0f;
        if (z < -127.0f) z = -127.0f;
        q[base + i] = (int8_t)(int)z;
      }
    }
  }
}

/* ------------------------------------------------------------------ GEMM */
/* Exact INT32 accumulators acc[m, n] = sum_k a[m, k] * b[n, k]. */
void m5o_gemm_i8_acc(const int8_t* a, const int8_t* b, int64_t M, int64_t N, int64_t K,
                     int32_t* acc) {
  for (int64_t m = 0; m < M; ++m) {
    const int8_t* ar = a + m * K;
    for (int64_t n = 0; n < N; ++n) {
      const int8_t* br = b + n * K;
      int32_t t = 0;
      for (int64_t k = 0; k < K; ++k) t += (int32_t)ar[k] * (int32_t)br[k];
      acc[m * N + n] = t;
    }
  }
}

#define EPI_PLAIN 0
#define EPI_BIAS_VEC 1
#define EPI_BIAS_TABLE 2
#define EPI_GATE_VEC 3
#define EPI_GATE_TABLE 4

/*
 * Epilogue of the quantized GEMM given exact accumulators (INT32 as float
 * source for INT8: float(acc) with round-to-nearest-even):
 *   v = (float(acc) * sa[m]) * sb[n]
 *   bias: v = v + bias[...]; gate: out = fmaf(bf16(v), gate[...], R[m, n])
 *   out rounded to out_dtype (bf16 / f16 / f32).
 */
void m5o_gemm_epilogue_i32(const int32_t* acc, int64_t M, int64_t N, const float* sa,
                           const float* sb, int epi, const float* bias,
                           const int32_t* bias_row_map, const uint16_t* residual,
                           const uint16_t* gate, const int32_t* gate_row_map, void* out,
                           int out_dtype) {
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t n = 0; n < N; ++n) {
      float v = (float)acc[m * N + n];
      if (sa) v = (v * sa[m]) * sb[n];
      if (epi == EPI_BIAS_VEC) v = v + bias[n];
      if (epi == EPI_BIAS_TABLE) v = v + bias[(int64_t)bias_row_map[m] * N + n];
      if (epi == EPI_GATE_VEC || epi == EPI_GATE_TABLE) {
        const int64_t go = epi == EPI_GATE_TABLE ? (int64_t)gate_row_map[m] * N : 0;
        const float br = bf16_to_f32(f32_to_bf16(v));
        v = fmaf(br, bf16_to_f32(gate[go + n]), bf16_to_f32(residual[m * N + n]));
      }
      store_elem(out, out_dtype, m * N + n, v);
    }
  }
}

/*
 * Q/K epilogue for one projection given exact accumulators acc[M, N]
 * (N = heads * 128): z = bf16((float(acc) * sa) * sb) (or bf16(acc) when sa
 * is NULL), per (row, head) sumsq = sequential fmaf over the 128 channels,
 * inv = 1 / sqrt(sumsq / 128 + eps), u_j = (z_j * inv) * gamma_j,
 * split-half RoPE on j < 2R, bf16 head-major out [heads, M, 128].
 */
void m5o_qk_rope_from_acc(const float* accf, int64_t M, int64_t N, const float* sa,
                          const float* sb, const uint16_t* gamma, const uint16_t* cosb,
                          const uint16_t* sinb, int R, float eps, uint16_t* out) {
  const int64_t heads = N / 128;
  float z[128], u[128];
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t h = 0; h < heads; ++h) {
      float sumsq = 0.0f;
      for (int j = 0; j < 128; ++j) {
        const int64_t col = h * 128 + j;
        float v = accf[m * N + col];
        if (sa) v = (v * sa[m]) * sb[col];
        z[j] = bf16_to_f32(f32_to_bf16(v));
        sumsq = fmaf(z[j], z[j], sumsq);
      }
      const float inv = 1.0f / sqrtf(sumsq / 128.0f + eps);
      for (int j = 0; j < 128; ++j) u[j] = (z[j] * inv) * bf16_to_f32(gamma[j]);
      for (int j = 0; j < 128; ++j) {
        float o = u[j];
        if (j < 2 * R) {
          const int p = j < R ? j + R : j - R;
          const int ang = j < R ? j : j - R;
          const float c = bf16_to_f32(cosb[m * R + ang]);
          const float s = bf16_to_f32(sinb[m * R + ang]);
          o = j < R ? (u[j] * c) - (u[p] * s) : (u[j] * c) + (u[p] * s);
        }
        out[(h * M + m) * 128 + j] = f32_to_bf16(o);
      }
    }
  }
}

/* ------------------------------------------------------------------------
 * The kernels' division-free INT8 code (csrc/common.cuh, i8_pair_div),
 * restated to check its claim here: with y = RN(1/s), q = RN(x y),
 * r = fma(-q, s, x) and c = fma(r, y, q) (Markstein's correction step),
 * rint(c) == rint(RN(x / s)) for every s >= 2^-90 and |x| <= 127.0001 s.
 * m5o_check_i8_div_free counts, over the given scales and every finite bf16
 * value x in that domain, the x whose two codes differ (0 expected);
 * m5o_check_i8_div_free_f32 does the same for `samples` fp32 pairs (x, s)
 * drawn by a fixed generator, half of them next to (k + 1/2) s.  *tested
 * receives the number of pairs compared. */
static float f32_of_bits(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static uint32_t bits_of_f32(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

static float i8_div_free_code(float x, float s, float y) {
  const float q = x * y;
  const float r = fmaf(-q, s, x);
  return rintf(fmaf(r, y, q));
}

int64_t m5o_check_i8_div_free(const float* scales, int64_t n, int64_t* tested) {
  int64_t bad = 0, count = 0;
  for (int64_t i = 0; i < n; ++i) {
    const float s = scales[i];
    if (!(s >= 0x1p-90f) || !isfinite(s)) continue;
    const float y = 1.0f / s;
    for (uint32_t h = 0; h < 65536u; ++h) {
      const float x = bf16_to_f32((uint16_t)h);
      if (!isfinite(x) || fabsf(x) > 127.0001f * s) continue;
      ++count;
      if (i8_div_free_code(x, s, y) != rintf(x / s)) ++bad;
    }
  }
  if (tested) *tested = count;
  return bad;
}

int64_t m5o_check_i8_div_free_f32(int64_t samples, uint64_t seed, int64_t* tested) {
  uint64_t st = seed ? seed : 0x9E3779B97F4A7C15ull;
  int64_t bad = 0, count = 0;
  for (int64_t t = 0; t < samples; ++t) {
    st ^= st << 13; st ^= st >> 7; st ^= st << 17;
    const uint32_t e = (uint32_t)(37 + st % 190);  /* scales 2^-90 .. 2^99 */
    st ^= st << 13; st ^= st >> 7; st ^= st << 17;
    const float s = f32_of_bits((e << 23) | (uint32_t)(st & 0x7FFFFFu));
    st ^= st << 13; st ^= st >> 7; st ^= st << 17;
    float x;
    if (t & 1) {  /* within 4 ulps of (k + 1/2) s */
      x = ((float)(int64_t)(st % 254) - 127.0f + 0.5f) * s;
      x = f32_of_bits(bits_of_f32(x) + (uint32_t)((int)((st >> 20) % 9) - 4));
    } else {
      x = ((float)(st % 2000001u) / 1000000.0f - 1.0f) * 127.0f * s;
    }
    if (!isfinite(x) || fabsf(x) > 127.0001f * s) continue;
    ++count;
    if (i8_div_free_code(x, s, 1.0f / s) != rintf(x / s)) ++bad;
  }
  if (tested) *tested = count;
  return bad;
}

/* The corrected quotient itself, for the RMS folding's
 * rint(RN(RN(v / peak) * 127)): c == RN(x / s) whenever s >= 2^-90 and
 * min_ratio <= |RN(x / s)| <= max_ratio.  Counts the finite bf16 values x
 * (over the given scales) and the `samples` random fp32 values for which c
 * and the IEEE quotient differ; *tested receives the number compared. */
int64_t m5o_check_div_free_quotient(const float* scales, int64_t n, float min_ratio,
                                    float max_ratio, int64_t samples, uint64_t seed,
                                    int64_t* tested) {
  int64_t bad = 0, count = 0;
  for (int64_t i = 0; i < n; ++i) {
    const float s = scales[i];
    if (!(s >= 0x1p-90f) || !isfinite(s)) continue;
    const float y = 1.0f / s;
    for (uint32_t h = 0; h < 65536u; ++h) {
      const float x = bf16_to_f32((uint16_t)h);
      if (!isfinite(x)) continue;
      const float ref = x / s;
      if (!(fabsf(ref) >= min_ratio && fabsf(ref) <= max_ratio)) continue;
      ++count;
      const float q = x * y, r = fmaf(-q, s, x), c = fmaf(r, y, q);
      if (bits_of_f32(c) != bits_of_f32(ref)) ++bad;
    }
  }
  uint64_t st = seed ? seed : 0x2545F4914F6CDD1Dull;
  for (int64_t t = 0; t < samples; ++t) {
    st ^= st << 13; st ^= st >> 7; st ^= st << 17;
    const uint32_t e = (uint32_t)(37 + st % 190);
    st ^= st << 13; st ^= st >> 7; st ^= st << 17;
    const float s = f32_of_bits((e << 23) | (uint32_t)(st & 0x7FFFFFu));
    st ^= st << 13; st ^= st >> 7; st ^= st << 17;
    /* a ratio log-uniform in [min_ratio, max_ratio], random sign */
    const double u = (double)(st >> 11) / 9007199254740992.0;
    const double ratio = exp(log((double)min_ratio) + u * (log((double)max_ratio) - log((double)min_ratio)));
    const float x = (float)((st & 1) ? -ratio : ratio) * s;
    const float ref = x / s;
    if (!isfinite(x) || !(fabsf(ref) >= min_ratio && fabsf(ref) <= max_ratio)) continue;
    ++count;
    const float y = 1.0f / s, q = x * y, r = fmaf(-q, s, x), c = fmaf(r, y, q);
    if (bits_of_f32(c) != bits_of_f32(ref)) ++bad;
  }
  if (tested) *tested = count;
  return bad;
}
