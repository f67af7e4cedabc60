// Per-token symmetric quantization of plain rows (no normalization, no
// rotation): the online activation quantization of the W8A8 / FP8 GEMM.
//
// Reference contract: src/m5kernels/metal.py:106-123 (quantize) with the
// arithmetic of src/m5kernels/numerics.py:29-46 (quantize_reference):
//   scale = peak / 127 (int8) or peak / 448 (E4M3), 1 for an all-zero row;
//   code  = clip(rint(x / scale), +-127) or E4M3_RNE_saturating(x / scale).
//
// One HBM read per row: each of the CTA's 256 threads loads its VPT 16-byte
// vectors of the row at once (lane-interleaved, 512 contiguous bytes per warp
// instruction) and keeps them packed in registers (a bf16 row of 16384 is 32
// registers per thread), reduces max |x| on the packed 16-bit pairs, then
// quantizes the same registers with packed-FP32 arithmetic and stores the
// codes 8 bytes per lane.  Rows wider than 256 x 16 vectors stream twice
// (peak pass from HBM, code pass from L2).  HBM traffic per row:
// K * sizeof(T) read, K written, 4 for the scale.
#include <type_traits>

#include "common.cuh"
#include "m5b_internal.h"

namespace m5b {

namespace {

constexpr int kThreads = 256;
constexpr int kTieQueue = 64;  // queued near-tie vectors per warp and row
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23: RNE to integer for |t| < 2^22

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
// into words by bracketed rounding of packed pairs (i8_pair).  Returns the
// bracket disagreement bits: nonzero means some element may round
// differently from the reference, and the vector is redone by
// i8_words_near_tie.
template <typename T>
__device__ __forceinline__ uint32_t pack_i8_vec(const uint4& raw, const I8Bracket& br,
                                                uint32_t* words) {
  constexpr int PAIRS = sizeof(T) == 2 ? 4 : 2;
  float2 m[PAIRS];
  uint32_t acc = 0u;
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
    m[p] = i8_pair(v, br, acc);
  }
#pragma unroll
  for (int w = 0; w < PAIRS / 2; ++w)
    words[w] = pack4_low_bytes(m[2 * w].x, m[2 * w].y, m[2 * w + 1].x, m[2 * w + 1].y);
  return acc;
}

// The exact codes of a vector that holds a product next to a half-integer:
// per element the reciprocal-product code, and for an element within 2^-14
// of a half-integer the division-free decision of int8_code_near_tie.  Kept
// out of line: it runs for a small fraction of vectors.  Requires
// scale >= 2^-100.
template <typename T>
__device__ __noinline__ uint2 i8_words_near_tie(uint4 raw, float scale, float inv) {
  constexpr int V = kVec<T>;
  constexpr float kNear = 0.5f - 0x1p-14f;
  float v[V];
  unpack<T>(raw, v);
  uint32_t w[2] = {0u, 0u};
#pragma unroll
  for (int e = 0; e < V; ++e) {
    const float t = __fmul_rn(v[e], inv);
    float m = __fadd_rn(t, kMagic);
    const float r = __fadd_rn(m, -kMagic);
    if (fabsf(__fsub_rn(t, r)) > kNear)
      m = __fadd_rn(int8_code_near_tie(v[e], scale, t, r), kMagic);
    w[e >> 2] |= (__float_as_uint(m) & 0xFFu) << (8 * (e & 3));
  }
  return make_uint2(w[0], w[1]);
}

__device__ __forceinline__ uint32_t code_i8_exact(float v, float scale) {
  float r = rintf(__fdiv_rn(v, scale));
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  return static_cast<uint32_t>(static_cast<int>(r)) & 0xFFu;
}

__device__ __forceinline__ uint32_t code_e4m3(float v, float scale, float inv, bool fast) {
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

// Codes of one 16-byte vector into `words` (V/4 words).
template <typename T, int OUT>
__device__ __forceinline__ void vec_codes(const uint4& raw, float scale, float inv, bool fast,
                                          uint32_t* words) {
  constexpr int V = kVec<T>;
  float v[V];
  if constexpr (OUT == OUT_E4M3) {
    unpack<T>(raw, v);
#pragma unroll
    for (int w = 0; w < V / 4; ++w)
      words[w] = code_e4m3(v[4 * w], scale, inv, fast) |
                 (code_e4m3(v[4 * w + 1], scale, inv, fast) << 8) |
                 (code_e4m3(v[4 * w + 2], scale, inv, fast) << 16) |
                 (code_e4m3(v[4 * w + 3], scale, inv, fast) << 24);
  } else {
    if (fast) {
      if (pack_i8_vec<T>(raw, i8_bracket(inv, scale), words) != 0u) {
        const uint2 w = i8_words_near_tie<T>(raw, scale, inv);
        words[0] = w.x;
        if constexpr (V == 8) words[1] = w.y;
      }
    } else {  // scale below 2^-100: the reciprocal product is not trustworthy
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

__device__ __forceinline__ float cta_peak(float peak, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = peak;
  __syncthreads();
  peak = red[0];
#pragma unroll
  for (int w = 1; w < kThreads / 32; ++w) peak = fmaxf(peak, red[w]);
  __syncthreads();
  return peak;
}

// VPT > 0: each thread holds VPT vectors of the row in registers (one HBM
// read).  VPT == 0: two streaming passes for very wide rows.
template <typename T, int OUT, int VPT>
__global__ void __launch_bounds__(kThreads)
    quant_rows_kernel(const T* __restrict__ x, int64_t rows, int64_t K, uint8_t* __restrict__ q,
                      float* __restrict__ s) {
  constexpr int V = kVec<T>;
  __shared__ float red[kThreads / 32];
  __shared__ uint4 tie_raw[kThreads / 32][kTieQueue];
  __shared__ int tie_idx[kThreads / 32][kTieQueue];
  __shared__ int tie_n[kThreads / 32];
  const int tid = threadIdx.x;
  const int nvec = static_cast<int>(K / V);  // K % V == 0 on this path
  const float qmax = OUT == OUT_E4M3 ? 448.0f : 127.0f;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * K);
    uint8_t* qr = q + row * K;
    if constexpr (VPT > 0) {
      uint4 raw[VPT];
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int j = tid + i * kThreads;
        raw[i] = j < nvec ? __ldg(xr + j) : make_uint4(0, 0, 0, 0);
      }
      Peak<T> pk;
#pragma unroll
      for (int i = 0; i < VPT; ++i) pk.add(raw[i]);
      const float peak = cta_peak(pk.value(), red);
      const float scale = peak == 0.0f ? 1.0f : __fdiv_rn(peak, qmax);
      const float inv = __frcp_rn(scale);
      const bool fast = scale >= 0x1p-100f;
      if (tid == 0) s[row] = scale;
      if (OUT == OUT_INT8 && fast) {
        // Bracketed codes for every vector; a vector whose brackets disagree
        // (a quotient next to a half-integer) is queued and redone exactly
        // after the pass by the whole warp, one queued vector per lane, so
        // the exact path does not serialise the warp vector by vector.
        const I8Bracket br = i8_bracket(inv, scale);
        const int warp = tid >> 5, lane = tid & 31;
        if (lane == 0) tie_n[warp] = 0;
        __syncwarp();
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
          const int j = tid + i * kThreads;
          if (j < nvec) {
            uint32_t words[V / 4];
            const uint32_t acc = pack_i8_vec<T>(raw[i], br, words);
            store_codes<T>(qr, j, words);
            if (acc != 0u) {
              const int slot = atomicAdd(&tie_n[warp], 1);
              if (slot < kTieQueue) {
                tie_raw[warp][slot] = raw[i];
                tie_idx[warp][slot] = j;
              } else {  // queue full: redo in place
                const uint2 w = i8_words_near_tie<T>(raw[i], scale, inv);
                store_codes<T>(qr, j, reinterpret_cast<const uint32_t*>(&w));
              }
            }
          }
        }
        __syncwarp();
        const int n = min(tie_n[warp], kTieQueue);
        for (int k = lane; k < n; k += 32) {
          const uint2 w = i8_words_near_tie<T>(tie_raw[warp][k], scale, inv);
          store_codes<T>(qr, tie_idx[warp][k], reinterpret_cast<const uint32_t*>(&w));
        }
        __syncwarp();
      } else {
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
          const int j = tid + i * kThreads;
          if (j < nvec) {
            uint32_t words[V / 4];
            vec_codes<T, OUT>(raw[i], scale, inv, fast, words);
            store_codes<T>(qr, j, words);
          }
        }
      }
    } else {
      Peak<T> p0, p1, p2, p3;
      int j = tid;
      for (; j + 3 * kThreads < nvec; j += 4 * kThreads) {
        const uint4 a = __ldg(xr + j), b = __ldg(xr + j + kThreads);
        const uint4 c = __ldg(xr + j + 2 * kThreads), d = __ldg(xr + j + 3 * kThreads);
        p0.add(a);
        p1.add(b);
        p2.add(c);
        p3.add(d);
      }
      for (; j < nvec; j += kThreads) p0.add(__ldg(xr + j));
      const float peak =
          cta_peak(fmaxf(fmaxf(p0.value(), p1.value()), fmaxf(p2.value(), p3.value())), red);
      const float scale = peak == 0.0f ? 1.0f : __fdiv_rn(peak, qmax);
      const float inv = __frcp_rn(scale);
      const bool fast = scale >= 0x1p-100f;
      if (tid == 0) s[row] = scale;
      for (j = tid; j < nvec; j += kThreads) {
        uint32_t words[V / 4];
        vec_codes<T, OUT>(__ldg(xr + j), scale, inv, fast, words);
        store_codes<T>(qr, j, words);
      }
    }
  }
}

template <typename T, int OUT, int VPT>
cudaError_t launch_quant_v(const RowPrepArgs& a, cudaStream_t stream) {
  auto kern = quant_rows_kernel<T, OUT, VPT>;
  static std::atomic<long long> shape[kMaxLaunchDevices];
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e =
      launch_shape(reinterpret_cast<const void*>(kern), kThreads, 0, shape, &dev, &sms, &per_sm);
  if (e != cudaSuccess) return e;
  int64_t grid = int64_t(sms) * per_sm;
  if (grid > a.rows) grid = a.rows;
  kern<<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(
      reinterpret_cast<const T*>(a.x), a.rows, a.K, reinterpret_cast<uint8_t*>(a.q), a.s);
  return cudaGetLastError();
}

template <typename T, int OUT>
cudaError_t launch_quant_t(const RowPrepArgs& a, cudaStream_t stream) {
  const int64_t nvec = a.K / kVec<T>;
  if (nvec <= 1 * kThreads) return launch_quant_v<T, OUT, 1>(a, stream);
  if (nvec <= 2 * kThreads) return launch_quant_v<T, OUT, 2>(a, stream);
  if (nvec <= 4 * kThreads) return launch_quant_v<T, OUT, 4>(a, stream);
  if (nvec <= 8 * kThreads) return launch_quant_v<T, OUT, 8>(a, stream);
  if (nvec <= 16 * kThreads) return launch_quant_v<T, OUT, 16>(a, stream);
  return launch_quant_v<T, OUT, 0>(a, stream);
}

}  // namespace

// True when the lean kernel applies: plain quantization of aligned rows whose
// width is a whole number of 16-byte vectors and whose codes can be stored
// 8 (fp32: 4) bytes at a time.
bool quant_rows_applicable(const RowPrepArgs& a, int x_dtype, int block, int out) {
  if (block != 0 || a.norm != NORM_NONE || a.branch || a.signs || out == OUT_F32) return false;
  const int vec = x_dtype == DT_F32 ? 4 : 8;
  const uintptr_t xa = reinterpret_cast<uintptr_t>(a.x), qa = reinterpret_cast<uintptr_t>(a.q);
  return (a.K % vec) == 0 && (xa % 16) == 0 && (qa % vec) == 0;
}

cudaError_t launch_quant_rows(const RowPrepArgs& a, const RowMaps& /*m*/, int x_dtype, int out,
                              cudaStream_t stream) {
  const bool e4 = out == OUT_E4M3;
  switch (x_dtype) {
    case DT_BF16:
      return e4 ? launch_quant_t<__nv_bfloat16, OUT_E4M3>(a, stream)
                : launch_quant_t<__nv_bfloat16, OUT_INT8>(a, stream);
    case DT_F16:
      return e4 ? launch_quant_t<__half, OUT_E4M3>(a, stream)
                : launch_quant_t<__half, OUT_INT8>(a, stream);
    case DT_F32:
      return e4 ? launch_quant_t<float, OUT_E4M3>(a, stream)
                : launch_quant_t<float, OUT_INT8>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace m5b
