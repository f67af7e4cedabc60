// Operand split of the FP32 GEMM mode (three TF32 tensor-core products).
//
// Reference contract: src/m5kernels/metal.py:158-269 (gemm, mode "fp32":
// FP32 operands, FP32 result) with the quality bar of
// src/m5kernels/engine.py:473 (relative L2 <= 1e-4 against the float64
// product).  tcgen05 has no FP32-input MMA; its kind::tf32 reads the top 19
// bits of each FP32 operand.  Writing x = hi + lo with hi = x truncated to
// TF32 (exact) and lo = x - hi (exact in FP32, |lo| < 2^-10 |x|),
//   A B^T = A_hi B_hi^T + A_hi B_lo^T + A_lo B_hi^T + A_lo B_lo^T,
// and the last term is below 2^-20 of the product, so a TF32 GEMM over the
// concatenated operands
//   A3 = [A_hi | A_hi | A_lo],   B3 = [B_hi | B_lo | B_hi]
// has the accuracy of an FP32 GEMM (lo itself loses its own bits past TF32:
// another 2^-10 of a 2^-10 term).  The columns are cut into S chunks of CK
// (a multiple of 4; the host runs one GEMM per chunk and adds the chunks'
// results in FP32), so a row is laid out [chunk][part][CK]: each chunk's
// three parts are contiguous and a whole number of 16-byte TMA strides.
// Columns past K are zero (they add nothing to any dot product).  An infinity or NaN
// enters once, in the first (hi x hi) part, with zeros in the other two, so
// it meets the other operand's hi part only (IEEE inf x 0 = NaN stays so).
//
// HBM-bound: 4 bytes read and 12 written per element; grid-stride over the
// [rows, S x CK] elements, one element per thread per step (coalesced in
// both the source and each of the three destination parts).
#include <cstdint>

#include "common.cuh"
#include "m5b_internal.h"

namespace m5b {
namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads)
    tf32_split_kernel(const float* __restrict__ x, int64_t rows, int64_t k, int64_t chunks,
                      int64_t ck, float* __restrict__ out, int lo_part) {
  const int64_t kp = chunks * ck;  // padded columns per row
  const int64_t total = rows * kp;
  const int64_t stride = int64_t(gridDim.x) * kThreads;
  for (int64_t i = int64_t(blockIdx.x) * kThreads + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / kp;
    const int64_t c = i - r * kp;
    const int64_t s = c / ck, j = c - s * ck;
    const float v = c < k ? __ldcs(x + r * k + c) : 0.0f;
    const uint32_t bits = __float_as_uint(v);
    float* o = out + r * 3 * kp + s * 3 * ck + j;
    if ((bits & 0x7F800000u) != 0x7F800000u) {  // finite: split at the TF32 mantissa
      const float hi = __uint_as_float(bits & 0xFFFFE000u);
      const float lo = __fsub_rn(v, hi);         // exact
      o[0] = hi;
      o[ck] = lo_part == 1 ? lo : hi;
      o[2 * ck] = lo_part == 2 ? lo : hi;
    } else {  // inf / NaN once, in the hi x hi product (no inf x 0 from the others)
      o[0] = v;
      o[ck] = 0.0f;
      o[2 * ck] = 0.0f;
    }
  }
}

}  // namespace

cudaError_t launch_tf32_split(const float* x, int64_t rows, int64_t k, int64_t chunks, int64_t ck,
                              float* out, int lo_part, cudaStream_t stream) {
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const int64_t need = (rows * chunks * ck + kThreads - 1) / kThreads;
  int64_t grid = int64_t(sms) * 8;
  if (grid > need) grid = need;
  if (grid < 1) grid = 1;
  tf32_split_kernel<<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(x, rows, k, chunks, ck,
                                                                           out, lo_part);
  return cudaGetLastError();
}

}  // namespace m5b
