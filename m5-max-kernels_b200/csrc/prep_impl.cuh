// Row-preparation kernels (template shared by prep_{bf16,f16,f32}.cu).
//
// One kernel template covers every memory-bound stage of the online activation
// path (reference operator contracts in parentheses):
//   * per-token symmetric INT8 / E4M3 quantization
//       (src/m5kernels/metal.py:27-44, numerics.py:29-46)
//   * signed block Hadamard rotation X D H, FP32 output
//       (src/m5kernels/hadamard.py:33-77, hadamard_reference.py:26-68)
//   * Hadamard + quantization in one pass (hadamard_gemm.py:65-66)
//   * fused RMS / LayerNorm + AdaLN modulation + rotation + quantization
//       (src/m5kernels/norm_hadamard.py:122-176, norm_hadamard_reference.py:67-94)
//   * the gated-residual extension R' = cast_R(R + branch * gate), written once
//       (src/m5kernels/norm_hadamard.py:198-265, gated_residual_reference.py:21-60)
//   * RMS scale folding: codes of (X gamma) D H, inverse RMS folded into the
//       row scale, or the direct form that normalizes first
//       (src/m5kernels/rms_quant.py:41-117, rms_quant_reference.py:24-89)
//
// Data layout in HBM: row-major [rows, K] activations; codes [rows, K] int8 /
// uint8 (E4M3 bits); scales fp32 [rows].  Each row is read once and its codes
// are written once: 3K + 4 bytes per row for bf16 in / int8 out (7K + 4 for the
// gated form, which also reads the branch and writes R').
//
// Execution: persistent CTAs of W warps (W = ceil(K / 2048)), one row at a
// time per CTA.  A ring of STAGES row buffers in shared memory is filled by
// TMA tile loads (one thread issues, completion on an mbarrier), so the next
// rows stream in while the current one is transformed.  Rows that are not
// whole 64-element chunks or not 16-byte aligned are read with plain loads.
//
// Ownership: thread t of the CTA owns the contiguous chunk of kChunk = 64
// elements [64 t, 64 t + 64) of the row, held in registers.  Hence Hadamard
// strides 1..32 are register butterflies and strides 64..B/2 are warp
// shuffles (lane xor 1 .. B/128).  Row reductions have one canonical order,
// mirrored by the C oracle and independent of the schedule: the row is cut
// into 16-element chunks, each summed by chunk16_sum (eight pairs, combined
// pairwise), and the chunk sums combine as a pairwise tree over chunk index
// (zero chunks pad the tree), the total finally added to +0.  Here a thread
// sums its four chunks pairwise, lanes continue the tree with a xor butterfly
// of increasing offset (1, 2, 4, 8, 16) and warps pairwise in index order.
#pragma once
#include "common.cuh"
#include "m5b_internal.h"

namespace m5b {

constexpr int kChunk = 64;  // elements per thread

// ---------------------------------------------------------------- quantization
// rint(v / scale) clipped to +-127 with the exact semantics of an IEEE divide
// followed by rint.  t = v * (1/scale) is within 2^-15.6 of the correctly
// rounded quotient when |v| <= peak; unless t lies within 2^-14 of a
// half-integer both round to the same integer, and in that case the code is
// decided exactly by int8_code_near_tie.
__device__ __forceinline__ int quant_i8(float v, float scale, float inv, bool fast) {
  if (!fast) return static_cast<int>(fminf(fmaxf(rintf(__fdiv_rn(v, scale)), -127.0f), 127.0f));
  const float t = __fmul_rn(v, inv);
  const float r = __fsub_rn(__fadd_rn(t, 12582912.0f), 12582912.0f);
  if (fabsf(__fsub_rn(t, r)) > 0.5f - 0x1p-14f) return static_cast<int>(int8_code_near_tie(v, scale, t, r));
  return static_cast<int>(fminf(fmaxf(r, -127.0f), 127.0f));
}

// E4M3 code of RN(v / scale) (RNE, saturating).  The conversion is monotonic,
// so when t(1 - 2^-18) and t(1 + 2^-18), which bracket the correctly rounded
// quotient, share one code, that is the code; otherwise divide exactly.
__device__ __forceinline__ uint32_t quant_e4m3(float v, float scale, float inv, bool fast) {
  if (fast) {
    const float t = __fmul_rn(v, inv);
    if ((__float_as_uint(scale) & 0x007FFFFFu) == 0u)  // exact reciprocal: t == v / scale
      return static_cast<uint32_t>(__nv_cvt_float_to_fp8(t, __NV_SATFINITE, __NV_E4M3));
    const __nv_fp8x2_storage_t two = __nv_cvt_float2_to_fp8x2(
        make_float2(__fmul_rn(t, 1.0f - 0x1p-18f), __fmul_rn(t, 1.0f + 0x1p-18f)), __NV_SATFINITE,
        __NV_E4M3);
    if ((two & 0xFFu) == (two >> 8)) return two & 0xFFu;
  }
  return static_cast<uint32_t>(
      __nv_cvt_float_to_fp8(__fdiv_rn(v, scale), __NV_SATFINITE, __NV_E4M3));
}

// Round-to-nearest-even of |t| < 2^22 by the 1.5 * 2^23 magic constant: the
// low byte of the sum's bit pattern is the two's-complement int8 of rint(t).
constexpr float kRoundMagic = 12582912.0f;

__device__ __forceinline__ void quant_i8_fast16(const float* v, float scale, float inv,
                                                uint32_t* words) {
  if (scale >= kI8DivMinScale) {
    const I8Div d = i8_div(inv, scale);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float2 m0 = i8_pair_div(make_float2(v[4 * w], v[4 * w + 1]), d);
      const float2 m1 = i8_pair_div(make_float2(v[4 * w + 2], v[4 * w + 3]), d);
      words[w] = pack4_low_bytes(m0.x, m0.y, m1.x, m1.y);
    }
  } else {  // scale below 2^-90: divide exactly
#pragma unroll
    for (int w = 0; w < 4; ++w)
      words[w] = (quant_i8(v[4 * w], scale, inv, false) & 0xFF) |
                 ((quant_i8(v[4 * w + 1], scale, inv, false) & 0xFF) << 8) |
                 ((quant_i8(v[4 * w + 2], scale, inv, false) & 0xFF) << 16) |
                 ((quant_i8(v[4 * w + 3], scale, inv, false) & 0xFF) << 24);
  }
}

// Codes of the RMS preparation, rint(RN(RN(v / peak) * 127)) clipped to
// +-127 (the reference's order: divide by the row peak, then scale by 127),
// for 16 values: the correctly rounded quotients of packed pairs
// (quot_pair_div, exact wherever a code can be nonzero), times 127, rounded
// to integers by the magic constant.  |v| <= peak keeps the codes inside
// +-127.  Peaks below kI8DivMinScale divide each value exactly.
__device__ __forceinline__ void rel_i8_fast16(const float* v, float peak, uint32_t* words) {
  if (peak < kI8DivMinScale) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t x = 0u;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float c = rintf(__fmul_rn(__fdiv_rn(v[4 * w + e], peak), 127.0f));
        const int code = static_cast<int>(fminf(fmaxf(c, -127.0f), 127.0f));
        x |= (static_cast<uint32_t>(code) & 0xFFu) << (8 * e);
      }
      words[w] = x;
    }
    return;
  }
  const I8Div d = i8_div(__frcp_rn(peak), peak);
  // RN(q * 127), then rint by the magic add: two separately rounded scalar
  // operations (__fmul_rn / __fadd_rn are never merged into a multiply-add;
  // a merged form, RN(q * 127 + magic), rounds products next to a
  // half-integer differently -- observed with the packed forms).
  auto code2 = [&](float2 x) -> float2 {
    const float2 q = quot_pair_div(x, d);
    return make_float2(__fadd_rn(__fmul_rn(q.x, 127.0f), kRoundMagic),
                       __fadd_rn(__fmul_rn(q.y, 127.0f), kRoundMagic));
  };
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const float2 m0 = code2(make_float2(v[4 * w], v[4 * w + 1]));
    const float2 m1 = code2(make_float2(v[4 * w + 2], v[4 * w + 3]));
    words[w] = pack4_low_bytes(m0.x, m0.y, m1.x, m1.y);
  }
}

// One RMS-preparation code, exactly (ragged tails, tiny peaks).
__device__ __forceinline__ int rel_i8_code(float v, float peak) {
  if (peak == 0.0f) return 0;
  const float c = rintf(__fmul_rn(__fdiv_rn(v, peak), 127.0f));
  return static_cast<int>(fminf(fmaxf(c, -127.0f), 127.0f));
}

// ---------------------------------------------------------------- loads
template <typename T>
__device__ __forceinline__ void cvt8(const uint4& raw, float* out) {
  if constexpr (sizeof(T) == 2) {
    const T* h = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] = to_f32(h[e]);
  }
}

// Eight parameter values starting at element j of a bf16 / fp16 / fp32 table.
__device__ __forceinline__ void param8(const void* base, int dtype, int64_t j, bool vec,
                                       float* out) {
  if (vec) {
    if (dtype == DT_F32) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(base) + (j >> 2));
      const float4 b = __ldg(reinterpret_cast<const float4*>(base) + (j >> 2) + 1);
      out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
      out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
    } else {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(
          reinterpret_cast<const uint16_t*>(base) + j));
      if (dtype == DT_BF16)
        cvt8<__nv_bfloat16>(raw, out);
      else
        cvt8<__half>(raw, out);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] = load_param(base, dtype, j + e);
  }
}

// ---------------------------------------------------------------- reductions
// Canonical sum of one 16-element chunk given as eight pairs p_k = (u_2k,
// u_2k+1): SQUARE false sums u, true sums u*u.  Pairs combine as
// p_2j + p_2j+1 (squares: fma(p_2j, p_2j, p_2j+1 * p_2j+1)), then
// (l_0 + l_1) + (l_2 + l_3), on both halves at once; the chunk is the even
// half plus the odd half.
template <bool SQUARE>
__device__ __forceinline__ float chunk16_sum(const float2* p) {
  float2 l[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if constexpr (SQUARE)
      l[j] = __ffma2_rn(p[2 * j], p[2 * j], __fmul2_rn(p[2 * j + 1], p[2 * j + 1]));
    else
      l[j] = __fadd2_rn(p[2 * j], p[2 * j + 1]);
  }
  const float2 t = __fadd2_rn(__fadd2_rn(l[0], l[1]), __fadd2_rn(l[2], l[3]));
  return __fadd_rn(t.x, t.y);
}

// Canonical sum over a thread's 64-element chunk: its four 16-element chunks
// (elements past cnt count as zero) combined pairwise.  KIND 0: sum v,
// 1: sum v*v, 2: sum (v-mean)^2.
template <int KIND>  // 0: sum v, 1: sum v*v, 2: sum (v-mean)^2
__device__ __forceinline__ float chunk_sum(const float* v, int cnt, float mean) {
  float c[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 p[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int e = 16 * i + 2 * k;
      float x0 = e < cnt ? v[e] : 0.0f, x1 = e + 1 < cnt ? v[e + 1] : 0.0f;
      if constexpr (KIND == 2) {
        x0 = e < cnt ? __fsub_rn(x0, mean) : 0.0f;
        x1 = e + 1 < cnt ? __fsub_rn(x1, mean) : 0.0f;
      }
      p[k] = make_float2(x0, x1);
    }
    c[i] = chunk16_sum<KIND != 0>(p);
  }
  return __fadd_rn(__fadd_rn(c[0], c[1]), __fadd_rn(c[2], c[3]));
}

// max |v| over a chunk as a balanced tree (exact in any order)
__device__ __forceinline__ float chunk_absmax(const float* v, int cnt) {
  float m[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) m[e] = 0.0f;
#pragma unroll
  for (int i = 0; i < 64; i += 8)
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (i + e < cnt) m[e] = fmaxf(m[e], fabsf(v[i + e]));
  return fmaxf(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])),
               fmaxf(fmaxf(m[4], m[5]), fmaxf(m[6], m[7])));
}
__device__ __forceinline__ float warp_sum_tree(float v) {
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// Canonical sum over the CTA: lanes pairwise (xor 1..16), warps pairwise.
__device__ __forceinline__ float cta_sum(float v, float* red, int W) {
  v = warp_sum_tree(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float part[16];
#pragma unroll
  for (int w = 0; w < 16; ++w) part[w] = (w < W) ? red[w] : 0.0f;
#pragma unroll
  for (int step = 1; step < 16; step <<= 1)
#pragma unroll
    for (int w = 0; w + step < 16; w += 2 * step) part[w] = __fadd_rn(part[w], part[w + step]);
  __syncthreads();
  return __fadd_rn(part[0], 0.0f);
}

__device__ __forceinline__ float cta_max(float v, float* red, int W) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = red[0];
  for (int w = 1; w < W; ++w) t = fmaxf(t, red[w]);
  __syncthreads();
  return t;
}

// Sum (canonical order, as cta_sum) and max over the CTA with one pair of
// barriers: the RMS scale-folding kernel reduces the squared norm of the
// input and the peak of the rotated row together.
__device__ __forceinline__ float2 cta_sum_max(float v, float m, float* red, float* red_max,
                                              int W) {
  v = warp_sum_tree(v);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((threadIdx.x & 31) == 0) {
    red[threadIdx.x >> 5] = v;
    red_max[threadIdx.x >> 5] = m;
  }
  __syncthreads();
  float part[16];
#pragma unroll
  for (int w = 0; w < 16; ++w) part[w] = (w < W) ? red[w] : 0.0f;
#pragma unroll
  for (int step = 1; step < 16; step <<= 1)
#pragma unroll
    for (int w = 0; w + step < 16; w += 2 * step) part[w] = __fadd_rn(part[w], part[w + step]);
  float t = red_max[0];
  for (int w = 1; w < W; ++w) t = fmaxf(t, red_max[w]);
  __syncthreads();
  return make_float2(__fadd_rn(part[0], 0.0f), t);
}

// ---------------------------------------------------------------- TMA row tiles
// A row of K elements is viewed as [K / E] box rows of E = 128 / sizeof(T)
// elements (128 bytes); the 3D tensor map {E, K/E, rows} loads whole rows
// with the 128-byte swizzle, so 16-byte slot i of box row r sits at physical
// slot i ^ (r & 7): threads that read their own chunk slot by slot hit eight
// different bank groups.

// 16-byte slot `slot` (0..7 within the chunk's 128-byte box row `br`) of a
// swizzled row buffer.
__device__ __forceinline__ const uint4* swz_slot(const uint8_t* base, int br, int slot) {
  return reinterpret_cast<const uint4*>(base + br * 128 + ((slot ^ (br & 7)) << 4));
}

// FULL: every chunk that exists is complete (K % 64 == 0), so per-element
// bounds checks vanish; always the case for rotations with B >= 64.
template <typename T, int B, int OUT, bool FULL>
__global__ void __launch_bounds__(512)
    row_prep_kernel(const __grid_constant__ CUtensorMap map_x,
                    const __grid_constant__ CUtensorMap map_b, const RowPrepArgs a,
                    const int stages, const int box_rows) {
  constexpr int IN_THREAD = (B == 0) ? 0 : (B < kChunk ? B : kChunk);  // in-register block span
  constexpr int LANE_SPAN = (B > kChunk) ? B / kChunk : 1;              // lanes per block
  extern __shared__ uint8_t dsmem_raw[];
  uint8_t* dsmem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(dsmem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ float red[16];
  __shared__ float red_max[16];
  __shared__ __align__(8) uint64_t full_bar[4];
  __shared__ int abort_flag;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int W = blockDim.x >> 5;
  const int64_t K = a.K;
  const int64_t j0 = int64_t(tid) * kChunk;  // first element of this thread's chunk
  const bool have = j0 < K;
  const int cnt = FULL ? (have ? kChunk : 0)
                       : (have ? static_cast<int>(K - j0 < kChunk ? K - j0 : kChunk) : 0);
  const bool fullchunk = FULL ? have : cnt == kChunk;
  const bool vec = a.vec_ok != 0;
  // element i of this thread's chunk exists (folds to `have` when FULL)
  auto in = [&](int i) { return FULL ? have : (i < cnt); };
  const bool gated = a.branch != nullptr;
  const int inputs = gated ? 2 : 1;
  const int64_t row_bytes = K * int64_t(sizeof(T));
  const int64_t buf_stride = (row_bytes + 1023) & ~int64_t(1023);  // 1024-aligned buffers
  const int64_t stride = gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full_bar[s], 1);
    abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();

  // Box rows of one input row, and TMA loads per input row (box_rows each).
  const int row_box_rows = static_cast<int>(row_bytes / 128);
  auto issue = [&](int64_t row, int s) {
    uint8_t* dst = dsmem + int64_t(s) * inputs * buf_stride;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive_expect_tx(&full_bar[s], static_cast<uint32_t>(inputs * row_bytes));
    for (int c = 0; c < row_box_rows; c += box_rows) {
      tma_load_3d(dst + c * 128, &map_x, &full_bar[s], 0, c, static_cast<int32_t>(row));
      if (gated)
        tma_load_3d(dst + buf_stride + c * 128, &map_b, &full_bar[s], 0, c,
                    static_cast<int32_t>(row));
    }
  };
  if (stages > 0 && tid == 0) {
    for (int s = 0; s < stages; ++s) {
      const int64_t row = blockIdx.x + s * stride;
      if (row < a.rows) issue(row, s);
    }
  }

  float v[kChunk];
  int it = 0;
  for (int64_t row = blockIdx.x; row < a.rows; row += stride, ++it) {
    const int s = stages > 0 ? it % stages : 0;
    // ---- load the chunk (and apply the gated residual update) -------------
    const uint8_t* xs = nullptr;  // swizzled ring slot (staged) ...
    const uint8_t* bs = nullptr;
    const T* xg = reinterpret_cast<const T*>(a.x) + row * K;  // ... or the row in HBM
    const T* bg = gated ? reinterpret_cast<const T*>(a.branch) + row * K : nullptr;
    if (stages > 0) {
      // One thread waits (bounded); the barrier then releases the CTA and a
      // single non-blocking probe gives every thread the acquire on the data.
      const uint32_t parity = static_cast<uint32_t>((it / stages) & 1);
      if (tid == 0)
        mbar_wait_bounded(&full_bar[s], parity, &abort_flag, a.status, DEV_TIMEOUT_PRODUCER);
      __syncthreads();
      if (abort_flag) break;
      (void)mbar_try_wait(&full_bar[s], parity);
      xs = dsmem + int64_t(s) * inputs * buf_stride;
      if (gated) bs = xs + buf_stride;
    }
    // Elements [j0 + i, j0 + i + 8) of this thread's chunk -> registers, from
    // the swizzled ring slot (staged rows hold whole chunks: 16-bit types use
    // one 128-byte box row per chunk, fp32 two) or straight from HBM.
    auto load8_at = [&](const uint8_t* sbase, const T* gbase, int i, float* out) {
      if (sbase != nullptr) {
        if constexpr (sizeof(T) == 2) {
          const uint4 raw = *swz_slot(sbase, tid, i / 8);  // one 16-byte shared load
          cvt8<T>(raw, out);
        } else {
          const int br = 2 * tid + (i >= 32 ? 1 : 0);
          const int sl = (i % 32) / 4;
          const uint4 p = *swz_slot(sbase, br, sl);
          const uint4 q = *swz_slot(sbase, br, sl + 1);
          out[0] = __uint_as_float(p.x); out[1] = __uint_as_float(p.y);
          out[2] = __uint_as_float(p.z); out[3] = __uint_as_float(p.w);
          out[4] = __uint_as_float(q.x); out[5] = __uint_as_float(q.y);
          out[6] = __uint_as_float(q.z); out[7] = __uint_as_float(q.w);
        }
      } else if (fullchunk && vec) {
        if constexpr (sizeof(T) == 2) {
          cvt8<T>(__ldg(reinterpret_cast<const uint4*>(gbase + j0 + i)), out);
        } else {
          const float4 p = __ldg(reinterpret_cast<const float4*>(gbase + j0 + i));
          const float4 q = __ldg(reinterpret_cast<const float4*>(gbase + j0 + i + 4));
          out[0] = p.x; out[1] = p.y; out[2] = p.z; out[3] = p.w;
          out[4] = q.x; out[5] = q.y; out[6] = q.z; out[7] = q.w;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) out[e] = in(i + e) ? to_f32(gbase[j0 + i + e]) : 0.0f;
      }
    };
    if (have) {
#pragma unroll
      for (int i = 0; i < kChunk; i += 8) load8_at(xs, xg, i, v + i);
    } else {
#pragma unroll
      for (int i = 0; i < kChunk; ++i) v[i] = 0.0f;
    }
    if (gated && have) {
      const int64_t goff = a.gate_row_map ? int64_t(a.gate_row_map[row]) * K : 0;
      T* rrow = reinterpret_cast<T*>(a.r_out) + row * K;
      const bool pvec = fullchunk && a.params_vec;
#pragma unroll
      for (int i = 0; i < kChunk; i += 8) {
        if (in(i)) {
          float br[8], g[8];
          load8_at(bs, bg, i, br);
          param8(a.gate, a.gate_dtype, goff + j0 + i, pvec, g);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (in(i + e)) v[i + e] = round_through<T>(__fmaf_rn(br[e], g[e], v[i + e]));
          if (fullchunk && vec) {
            if constexpr (sizeof(T) == 2) {
              uint4 raw;
              T* h = reinterpret_cast<T*>(&raw);
#pragma unroll
              for (int e = 0; e < 8; ++e) h[e] = from_f32<T>(v[i + e]);
              *reinterpret_cast<uint4*>(rrow + j0 + i) = raw;
            } else {
              *reinterpret_cast<float4*>(rrow + j0 + i) =
                  make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
              *reinterpret_cast<float4*>(rrow + j0 + i + 4) =
                  make_float4(v[i + 4], v[i + 5], v[i + 6], v[i + 7]);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (in(i + e)) rrow[j0 + i + e] = from_f32<T>(v[i + e]);
          }
        }
      }
    }
    if (stages > 0) {
      __syncthreads();  // every thread has read ring slot s
      const int64_t next = row + int64_t(stages) * stride;
      if (tid == 0 && next < a.rows) issue(next, s);
    }

    // ---- normalization statistics ----------------------------------------
    float mean = 0.0f, inv = 1.0f;
    float sq_part = 0.0f;  // RMS folding: this thread's share of sum(x^2)
    if (a.rms_quant != RMSQ_NONE) {
      // RMS statistics of the ORIGINAL row; the direct form normalizes now,
      // the folded form keeps the inverse RMS for the row scale.
      sq_part = chunk_sum<1>(v, cnt, 0.0f);
      if (a.rms_quant == RMSQ_DIRECT) {
        const float moment = __fdiv_rn(cta_sum(sq_part, red, W), static_cast<float>(K));
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(moment, a.eps)));
      }
      const bool pvec = fullchunk && a.params_vec;
#pragma unroll
      for (int i = 0; i < kChunk; i += 8) {
        if (in(i)) {
          float g[8];
          if (pvec) {
            param8(a.gamma, DT_F32, j0 + i, true, g);
          } else {  // ragged rows (any K without rotation): never read past gamma[K - 1]
            const float* gp = reinterpret_cast<const float*>(a.gamma) + j0 + i;
#pragma unroll
            for (int e = 0; e < 8; ++e) g[e] = in(i + e) ? __ldg(gp + e) : 0.0f;
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (in(i + e)) {
              const float t = (a.rms_quant == RMSQ_DIRECT) ? __fmul_rn(v[i + e], inv) : v[i + e];
              v[i + e] = __fmul_rn(t, g[e]);
            }
          }
        }
      }
    } else if (a.norm != NORM_NONE) {
      const float acc = (a.norm == NORM_LAYER) ? chunk_sum<0>(v, cnt, 0.0f)
                                               : chunk_sum<1>(v, cnt, 0.0f);
      const float kf = static_cast<float>(K);
      const float first = __fdiv_rn(cta_sum(acc, red, W), kf);
      float moment = first;
      if (a.norm == NORM_LAYER) {
        mean = first;
        moment = __fdiv_rn(cta_sum(chunk_sum<2>(v, cnt, mean), red, W), kf);
      }
      inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(moment, a.eps)));

      // ---- modulation, optional rounding --------------------------------
      const int64_t moff = a.row_map ? int64_t(a.row_map[row]) * K : 0;
      const bool pvec = fullchunk && a.params_vec;
#pragma unroll
      for (int i = 0; i < kChunk; i += 8) {
        if (in(i)) {
          float g[8], sc[8], sh[8];
          param8(a.gamma, a.gamma_dtype, j0 + i, pvec, g);
          param8(a.scale, a.scale_dtype, moff + j0 + i, pvec, sc);
          param8(a.shift, a.shift_dtype, moff + j0 + i, pvec, sh);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (in(i + e)) {
              const float t = __fmul_rn(__fmul_rn(__fsub_rn(v[i + e], mean), inv), g[e]);
              float y = __fmaf_rn(t, __fadd_rn(1.0f, sc[e]), sh[e]);
              if (a.round_output) y = round_through<T>(y);
              v[i + e] = y;
            }
          }
        }
      }
    }
    // ---- signs -----------------------------------------------------------
    if (a.signs) {
      if (fullchunk && a.params_vec) {
#pragma unroll
        for (int i = 0; i < kChunk; i += 16) {
          const uint4 sg = __ldg(reinterpret_cast<const uint4*>(a.signs + j0 + i));
          const int8_t* s8 = reinterpret_cast<const int8_t*>(&sg);
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (s8[e] < 0) v[i + e] = -v[i + e];
        }
      } else {
#pragma unroll
        for (int i = 0; i < kChunk; ++i)
          if (in(i) && a.signs[j0 + i] < 0) v[i] = -v[i];
      }
    }

    // ---- block Walsh-Hadamard transform (natural Sylvester order) ---------
    if constexpr (B > 0) {
#pragma unroll
      for (int h = 1; h < IN_THREAD; h <<= 1) {
#pragma unroll
        for (int i = 0; i < kChunk; ++i) {
          if ((i & h) == 0) {
            const float lo = v[i], hi = v[i + h];
            v[i] = __fadd_rn(lo, hi);
            v[i + h] = __fsub_rn(lo, hi);
          }
        }
      }
#pragma unroll
      for (int off = 1; off < LANE_SPAN; off <<= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < kChunk; ++i) {
          const float own = v[i];
          const float peer = __shfl_xor_sync(0xffffffffu, own, off);
          v[i] = upper ? __fsub_rn(peer, own) : __fadd_rn(own, peer);
        }
      }
#pragma unroll
      for (int i = 0; i < kChunk; ++i) v[i] = __fmul_rn(v[i], a.inv_sqrt_block);
    }

    if constexpr (OUT == OUT_ROW && sizeof(T) == 2) {
      // staged comparator: the modulated row in the input dtype (B == 0)
      T* yrow = reinterpret_cast<T*>(a.y) + row * K;
      if (fullchunk && vec) {
#pragma unroll
        for (int i = 0; i < kChunk; i += 8) {
          uint4 raw;
          T* h = reinterpret_cast<T*>(&raw);
#pragma unroll
          for (int e = 0; e < 8; ++e) h[e] = from_f32<T>(v[i + e]);
          *reinterpret_cast<uint4*>(yrow + j0 + i) = raw;
        }
      } else {
#pragma unroll
        for (int i = 0; i < kChunk; ++i)
          if (in(i)) yrow[j0 + i] = from_f32<T>(v[i]);
      }
    } else if constexpr (OUT == OUT_F32 || OUT == OUT_ROW) {
      float* yrow = a.y + row * K;
      if (fullchunk && vec) {
#pragma unroll
        for (int i = 0; i < kChunk; i += 4)
          *reinterpret_cast<float4*>(yrow + j0 + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < kChunk; ++i)
          if (in(i)) yrow[j0 + i] = v[i];
      }
    } else if (a.rms_quant != RMSQ_NONE) {
      // ---- RMS preparation: peak of the rotated row, folded scale, codes ---
      float peak;
      if (a.rms_quant == RMSQ_FOLD) {
        const float2 sm = cta_sum_max(sq_part, chunk_absmax(v, cnt), red, red_max, W);
        const float moment = __fdiv_rn(sm.x, static_cast<float>(K));
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(moment, a.eps)));
        peak = sm.y;
      } else {
        peak = cta_max(chunk_absmax(v, cnt), red, W);
        inv = 1.0f;
      }
      const float scale = (peak == 0.0f) ? 1.0f : __fdiv_rn(__fmul_rn(peak, inv), 127.0f);
      if (tid == 0) a.s[row] = scale;
      int8_t* qrow = reinterpret_cast<int8_t*>(a.q) + row * K;
      if (fullchunk && vec && (K % 16) == 0 && peak >= 0x1p-100f) {
#pragma unroll
        for (int w0 = 0; w0 < kChunk / 4; w0 += 4) {
          uint32_t words[4];
          rel_i8_fast16(v + 4 * w0, peak, words);
          *reinterpret_cast<uint4*>(qrow + j0 + 4 * w0) =
              make_uint4(words[0], words[1], words[2], words[3]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < kChunk; ++i)
          if (in(i)) qrow[j0 + i] = static_cast<int8_t>(rel_i8_code(v[i], peak));
      }
    } else {
      // ---- row peak, per-row scale, codes ----------------------------------
      const float peak = cta_max(chunk_absmax(v, cnt), red, W);
      const float qmax = (OUT == OUT_E4M3) ? 448.0f : 127.0f;
      const float scale = (peak == 0.0f) ? 1.0f : __fdiv_rn(peak, qmax);
      const float rinv = __frcp_rn(scale);
      const bool fast = scale >= 0x1p-100f;
      if (tid == 0) a.s[row] = scale;
      uint8_t* qrow = reinterpret_cast<uint8_t*>(a.q) + row * K;
      if (fullchunk && vec && (K % 16) == 0) {
        if constexpr (OUT == OUT_E4M3) {
#pragma unroll
          for (int w0 = 0; w0 < kChunk / 4; w0 += 4) {
            uint32_t words[4];
            e4m3_words<4>(v + 4 * w0, scale, rinv, fast, words);
            *reinterpret_cast<uint4*>(qrow + j0 + 4 * w0) =
                make_uint4(words[0], words[1], words[2], words[3]);
          }
        } else {
#pragma unroll
          for (int w0 = 0; w0 < kChunk / 4; w0 += 4) {
            uint32_t words[4];
            if (fast) {
              quant_i8_fast16(v + 4 * w0, scale, rinv, words);
            } else {  // scale below 2^-100: divide exactly
#pragma unroll
              for (int w = 0; w < 4; ++w) {
                const float* p = v + 4 * (w0 + w);
                words[w] = (quant_i8(p[0], scale, rinv, false) & 0xFF) |
                           ((quant_i8(p[1], scale, rinv, false) & 0xFF) << 8) |
                           ((quant_i8(p[2], scale, rinv, false) & 0xFF) << 16) |
                           ((quant_i8(p[3], scale, rinv, false) & 0xFF) << 24);
              }
            }
            *reinterpret_cast<uint4*>(qrow + j0 + 4 * w0) =
                make_uint4(words[0], words[1], words[2], words[3]);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < kChunk; ++i) {
          if (in(i)) {
            if constexpr (OUT == OUT_E4M3)
              qrow[j0 + i] = static_cast<uint8_t>(quant_e4m3(v[i], scale, rinv, fast));
            else
              qrow[j0 + i] = static_cast<uint8_t>(quant_i8(v[i], scale, rinv, fast));
          }
        }
      }
    }
  }
  if (stages > 0 && abort_flag && tid == 0) {
    // A wait gave up: let the copies already issued land before the CTA exits.
    for (int s2 = 0; s2 < stages; ++s2) {
      const unsigned long long t0 = globaltimer_ns();
      for (uint32_t ph = 0; ph < 2; ++ph) {
        while (!mbar_try_wait(&full_bar[s2], ph)) {
          if (globaltimer_ns() - t0 > kWaitLimitNs) break;
        }
      }
    }
  }
}

template <typename T, int B, int OUT, bool FULL>
static cudaError_t launch_f(const RowPrepArgs& a, const RowMaps& maps, cudaStream_t stream) {
  auto kern = row_prep_kernel<T, B, OUT, FULL>;
  const int threads = a.warps * 32;
  const int64_t row_bytes = a.K * int64_t(sizeof(T));
  const int inputs = a.branch ? 2 : 1;
  const int64_t buf_stride = (row_bytes + 1023) & ~int64_t(1023);
  int stages = 0;
  if (maps.valid) {
    const int64_t per_stage = buf_stride * inputs;
    stages = per_stage <= 24 * 1024 ? 4 : (per_stage <= 48 * 1024 ? 3 : (per_stage <= 96 * 1024 ? 2 : 0));
  }
  const int smem = stages > 0 ? static_cast<int>(stages * buf_stride * inputs) + 1024 : 0;
  static std::atomic<long long> shape[kMaxLaunchDevices];
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e = launch_shape(reinterpret_cast<const void*>(kern), threads, smem, shape, &dev,
                               &sms, &per_sm);
  if (e != cudaSuccess) return e;
  int64_t grid = int64_t(sms) * per_sm;
  if (grid > a.rows) grid = a.rows;
  kern<<<static_cast<unsigned>(grid), threads, smem, stream>>>(maps.x, maps.b, a, stages,
                                                               maps.box_rows);
  return cudaGetLastError();
}

template <typename T, int B, int OUT>
static cudaError_t launch_t(const RowPrepArgs& a, const RowMaps& maps, cudaStream_t stream) {
  if constexpr (B >= 64) {
    return launch_f<T, B, OUT, true>(a, maps, stream);  // K % B == 0 implies whole chunks
  } else {
    if (a.K % kChunk == 0) return launch_f<T, B, OUT, true>(a, maps, stream);
    return launch_f<T, B, OUT, false>(a, maps, stream);
  }
}

template <typename T, int OUT>
static cudaError_t launch_b(const RowPrepArgs& a, const RowMaps& m, int block,
                           cudaStream_t stream) {
  switch (block) {
    case 0: return launch_t<T, 0, OUT>(a, m, stream);
    case 32: return launch_t<T, 32, OUT>(a, m, stream);
    case 64: return launch_t<T, 64, OUT>(a, m, stream);
    case 128: return launch_t<T, 128, OUT>(a, m, stream);
    case 256: return launch_t<T, 256, OUT>(a, m, stream);
    case 512: return launch_t<T, 512, OUT>(a, m, stream);
    case 1024: return launch_t<T, 1024, OUT>(a, m, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
static cudaError_t launch_o(const RowPrepArgs& a, const RowMaps& m, int block, int out,
                           cudaStream_t stream) {
  switch (out) {
    case OUT_INT8: return launch_b<T, OUT_INT8>(a, m, block, stream);
    case OUT_E4M3: return launch_b<T, OUT_E4M3>(a, m, block, stream);
    case OUT_F32: return launch_b<T, OUT_F32>(a, m, block, stream);
    case OUT_ROW: return block == 0 ? launch_t<T, 0, OUT_ROW>(a, m, stream) : cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace m5b
