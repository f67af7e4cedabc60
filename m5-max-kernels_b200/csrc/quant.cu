// Per-token symmetric quantization of plain rows (no normalization, no
// rotation): the online activation quantization of the W8A8 / FP8 GEMM.
//
// Reference contract: src/m5kernels/metal.py:27-44 (quantize) with the
// arithmetic of src/m5kernels/numerics.py:29-46 (quantize_reference):
//   scale = peak / 127 (int8) or peak / 448 (E4M3), 1 for an all-zero row;
//   code  = clip(rint(x / scale), +-127) or E4M3_RNE_saturating(x / scale).
//
// One HBM read per row: each of the CTA's 256 threads loads its VPT 16-byte
// vectors of the row at once (lane-interleaved, 512 contiguous bytes per warp
// instruction) and keeps them packed in registers (a bf16 row of 16384 is 32
// registers per thread), reduces max |x| on the packed 16-bit pairs, then
// quantizes the same registers with packed-FP32 arithmetic and stores the
// codes 8 bytes per lane.  While a row is processed, the CTA's next row is
// already streaming into L2 (one bulk prefetch per row).  Rows wider than
// 256 x 16 vectors stream twice (peak pass from HBM, code pass from L2).  HBM
// traffic per row: K * sizeof(T) read, K written, 4 for the scale.
#include <cstdlib>
#include <type_traits>

#include "common.cuh"
#include "m5b_internal.h"
#include "quant_vec.cuh"

namespace m5b {

namespace {

using namespace qv;


template <int NT>
__device__ __forceinline__ float cta_peak(float peak, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = peak;
  __syncthreads();
  peak = red[0];
#pragma unroll
  for (int w = 1; w < NT / 32; ++w) peak = fmaxf(peak, red[w]);
  __syncthreads();
  return peak;
}

// NT threads per row.  VPT > 0: each thread holds VPT vectors of the row in
// registers (one HBM read).  VPT == 0: two streaming passes for very wide
// rows.  EXACT: the row is exactly VPT * NT vectors, so no vector needs a
// bounds guard.
template <typename T, int OUT, int VPT, bool EXACT, int NT>
__global__ void __launch_bounds__(NT)
    quant_rows_kernel(const T* __restrict__ x, int64_t rows, int64_t K, uint8_t* __restrict__ q,
                      float* __restrict__ s) {
  constexpr int V = kVec<T>;
  __shared__ float red[NT / 32];
  const int tid = threadIdx.x;
  const int nvec = static_cast<int>(K / V);  // K % V == 0 on this path
  const float qmax = OUT == OUT_E4M3 ? 448.0f : 127.0f;
  // A GEMM launched after this kernel with programmatic serialization may
  // begin its set-up now; it waits for this grid's completion before it
  // reads the codes and scales.
  grid_dependents_launch();
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * K);
    uint8_t* qr = q + row * K;
    // This CTA's next row starts streaming into L2 now, so its reads overlap
    // the dependent chain of this row (peak, barrier, codes, stores) instead
    // of following it.  Rows here are whole 16-byte vectors on 16-byte
    // aligned bases (quant_rows_applicable).
    if (VPT > 0 && tid == 0 && row + gridDim.x < rows)
      prefetch_l2_bulk(x + (row + gridDim.x) * K, static_cast<uint32_t>(K * sizeof(T)));
    if constexpr (VPT > 0) {
      uint4 raw[VPT];
#pragma unroll
      for (int i = 0; i < VPT; ++i) {
        const int j = tid + i * NT;
        // streaming loads: the activations are read once, and the codes
        // written here (read next by the GEMM) should keep their L2 lines
        raw[i] = (EXACT || j < nvec) ? __ldcs(xr + j) : make_uint4(0, 0, 0, 0);
      }
      Peak<T> pk;
#pragma unroll
      for (int i = 0; i < VPT; ++i) pk.add(raw[i]);
      const float peak = cta_peak<NT>(pk.value(), red);
      const float scale = peak == 0.0f ? 1.0f : __fdiv_rn(peak, qmax);
      const float inv = __frcp_rn(scale);
      const bool fast = scale >= 0x1p-100f;
      if (tid == 0) s[row] = scale;
      if (OUT == OUT_INT8 && scale >= kI8DivMinScale) {
        // Codes from the correctly rounded quotients of packed pairs
        // (i8_pair_div): the same operations for every vector, no branch.
        const I8Div d = i8_div(inv, scale);
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
          const int j = tid + i * NT;
          if (EXACT || j < nvec) {
            uint32_t words[V / 4];
            pack_i8_vec<T>(raw[i], d, words);
            store_codes<T>(qr, j, words);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < VPT; ++i) {
          const int j = tid + i * NT;
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
      for (; j + 3 * NT < nvec; j += 4 * NT) {
        const uint4 a = __ldg(xr + j), b = __ldg(xr + j + NT);
        const uint4 c = __ldg(xr + j + 2 * NT), d = __ldg(xr + j + 3 * NT);
        p0.add(a);
        p1.add(b);
        p2.add(c);
        p3.add(d);
      }
      for (; j < nvec; j += NT) p0.add(__ldg(xr + j));
      const float peak =
          cta_peak<NT>(fmaxf(fmaxf(p0.value(), p1.value()), fmaxf(p2.value(), p3.value())), red);
      const float scale = peak == 0.0f ? 1.0f : __fdiv_rn(peak, qmax);
      const float inv = __frcp_rn(scale);
      const bool fast = scale >= 0x1p-100f;
      if (tid == 0) s[row] = scale;
      for (j = tid; j < nvec; j += NT) {
        uint32_t words[V / 4];
        vec_codes<T, OUT>(__ldg(xr + j), scale, inv, fast, words);
        store_codes<T>(qr, j, words);
      }
    }
  }
}

template <typename T, int OUT, int VPT, int NT>
cudaError_t launch_quant_v(const RowPrepArgs& a, cudaStream_t stream) {
  const bool exact = VPT > 0 && a.K / kVec<T> == int64_t(VPT) * NT;
  auto kern = exact ? quant_rows_kernel<T, OUT, VPT, VPT != 0, NT>
                    : quant_rows_kernel<T, OUT, VPT, false, NT>;
  static std::atomic<long long> shape[2][kMaxLaunchDevices];
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e = launch_shape(reinterpret_cast<const void*>(kern), NT, 0, shape[exact], &dev,
                               &sms, &per_sm);
  if (e != cudaSuccess) return e;
  int64_t grid = int64_t(sms) * per_sm;
  if (grid > a.rows) grid = a.rows;
  kern<<<static_cast<unsigned>(grid), NT, 0, stream>>>(
      reinterpret_cast<const T*>(a.x), a.rows, a.K, reinterpret_cast<uint8_t*>(a.q), a.s);
  return cudaGetLastError();
}

template <typename T, int OUT>
cudaError_t launch_quant_t(const RowPrepArgs& a, cudaStream_t stream) {
  const int64_t nvec = a.K / kVec<T>;
  constexpr int kNT = 256;
  if (nvec <= 1 * kNT) return launch_quant_v<T, OUT, 1, kNT>(a, stream);
  if (nvec <= 2 * kNT) return launch_quant_v<T, OUT, 2, kNT>(a, stream);
  if (nvec <= 4 * kNT) return launch_quant_v<T, OUT, 4, kNT>(a, stream);
  if (nvec <= 8 * kNT) return launch_quant_v<T, OUT, 8, kNT>(a, stream);
  if (nvec <= 16 * kNT) return launch_quant_v<T, OUT, 16, kNT>(a, stream);
  return launch_quant_v<T, OUT, 0, kNT>(a, stream);
}

}  // namespace

// True when the lean kernel applies: plain quantization of aligned rows whose
// width is a whole number of 16-byte vectors and whose codes can be stored
// 8 (fp32: 4) bytes at a time.
bool quant_rows_applicable(const RowPrepArgs& a, int x_dtype, int block, int out) {
  if (block != 0 || a.norm != NORM_NONE || a.rms_quant != RMSQ_NONE || a.branch || a.signs ||
      out == OUT_F32)
    return false;
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
