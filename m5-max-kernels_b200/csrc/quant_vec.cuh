// Per-vector helpers of the per-token quantization (16-byte vectors of 8
// bf16 / fp16 or 4 fp32 values): row peak, INT8 codes from correctly rounded
// quotients, E4M3 codes, code stores.  Shared by the quantize kernel
// (quant.cu) and the fused quantize + GEMM kernel (gemm.cu).
//
// Reference arithmetic: src/m5kernels/numerics.py:29-46 (quantize_reference):
//   scale = peak / 127 (int8) or peak / 448 (E4M3), 1 for an all-zero row;
//   code  = clip(rint(x / scale), +-127) or E4M3_RNE_saturating(x / scale).
#pragma once
#include <type_traits>

#include "common.cuh"
#include "m5b_internal.h"

namespace m5b {
namespace qv {

// Running row peak max|x|.  16-bit inputs stay packed: one
// max.xorsign.abs per pair of words (the magnitudes are exact, the sign bits
// are cleared at the end); fp32 inputs use FMNMX with |.|.
template <typename T>
struct Peak {
  uint32_t h = 0u;
  float f = 0.0f;
  __device__ __forceinline__ void add(const uint4& raw) {
    if constexpr (sizeof(T) == 2) {
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        h = max_xorsign_abs_bf16x2(
            h, max_xorsign_abs_bf16x2(max_xorsign_abs_bf16x2(raw.x, raw.y),
                                      max_xorsign_abs_bf16x2(raw.z, raw.w)));
      } else {
        h = max_xorsign_abs_f16x2(
            h, max_xorsign_abs_f16x2(max_xorsign_abs_f16x2(raw.x, raw.y),
                                     max_xorsign_abs_f16x2(raw.z, raw.w)));
      }
    } else {
      f = fmaxf(f, fmaxf(fmaxf(fabsf(__uint_as_float(raw.x)), fabsf(__uint_as_float(raw.y))),
                         fmaxf(fabsf(__uint_as_float(raw.z)), fabsf(__uint_as_float(raw.w)))));
    }
  }
  __device__ __forceinline__ float value() const {
    if constexpr (sizeof(T) == 2) {
      // |x| of a 16-bit float is its bit pattern with the sign cleared, and for
      // finite values that pattern orders like the value.
      const uint32_t m = h & 0x7FFF7FFFu;
      const uint32_t hi = m >> 16, lo = m & 0xFFFFu;
      const uint16_t best = static_cast<uint16_t>(hi > lo ? hi : lo);
      return to_f32(*reinterpret_cast<const T*>(&best));
    } else {
      return f;
    }
  }
};

// Elements per 16-byte vector.
template <typename T>
constexpr int kVec = 16 / sizeof(T);

template <typename T>
__device__ __forceinline__ void unpack(const uint4& raw, float* out) {
  if constexpr (sizeof(T) == 2) {
    const T* h = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] = to_f32(h[e]);
  } else {
    const float* f = reinterpret_cast<const float*>(&raw);
#pragma unroll
    for (int e = 0; e < 4; ++e) out[e] = f[e];
  }
}

// INT8 codes of one 16-byte vector (8 bf16/fp16 or 4 fp32 values) packed
// into words, from the correctly rounded quotients of packed pairs
// (i8_pair_div).  Requires scale >= kI8DivMinScale.
template <typename T>
__device__ __forceinline__ void pack_i8_vec(const uint4& raw, const I8Div& d, uint32_t* words) {
  constexpr int PAIRS = sizeof(T) == 2 ? 4 : 2;
  float2 m[PAIRS];
#pragma unroll
  for (int p = 0; p < PAIRS; ++p) {
    float2 v;
    if constexpr (sizeof(T) == 2) {
      const uint32_t w = reinterpret_cast<const uint32_t*>(&raw)[p];
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        v = make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
      } else {
        const __half2 h = *reinterpret_cast<const __half2*>(&w);
        v = __half22float2(h);
      }
    } else {
      v = make_float2(reinterpret_cast<const float*>(&raw)[2 * p],
                      reinterpret_cast<const float*>(&raw)[2 * p + 1]);
    }
    m[p] = i8_pair_div(v, d);
  }
#pragma unroll
  for (int w = 0; w < PAIRS / 2; ++w)
    words[w] = pack4_low_bytes(m[2 * w].x, m[2 * w].y, m[2 * w + 1].x, m[2 * w + 1].y);
}

static __device__ __forceinline__ uint32_t code_i8_exact(float v, float scale) {
  float r = rintf(__fdiv_rn(v, scale));
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return static_cast<uint32_t>(static_cast<int>(r)) & 0xFFu;
}

// Codes of one 16-byte vector into `words` (V/4 words).
template <typename T, int OUT>
__device__ __forceinline__ void vec_codes(const uint4& raw, float scale, float inv, bool fast,
                                          uint32_t* words) {
  constexpr int V = kVec<T>;
  float v[V];
  if constexpr (OUT == OUT_E4M3) {
    unpack<T>(raw, v);
    e4m3_words<V / 4>(v, scale, inv, fast, words);
  } else {
    if (fast && scale >= kI8DivMinScale) {
      pack_i8_vec<T>(raw, i8_div(inv, scale), words);
    } else {  // scale below 2^-90: divide exactly
      unpack<T>(raw, v);
#pragma unroll
      for (int w = 0; w < V / 4; ++w)
        words[w] = code_i8_exact(v[4 * w], scale) | (code_i8_exact(v[4 * w + 1], scale) << 8) |
                   (code_i8_exact(v[4 * w + 2], scale) << 16) |
                   (code_i8_exact(v[4 * w + 3], scale) << 24);
    }
  }
}

template <typename T>
__device__ __forceinline__ void store_codes(uint8_t* qr, int64_t j, const uint32_t* words) {
  if constexpr (kVec<T> == 8)
    *reinterpret_cast<uint2*>(qr + j * 8) = make_uint2(words[0], words[1]);
  else
    *reinterpret_cast<uint32_t*>(qr + j * 4) = words[0];
}

}  // namespace qv
}  // namespace m5b
