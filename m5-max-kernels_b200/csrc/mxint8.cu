// MXINT8 block quantization: 32-element blocks along each row, one shared
// power-of-two scale per block (an E8M0 exponent byte), INT8 codes.
//
// Reference contract: src/m5kernels/metal.py:27-44 (quantize, mode "mxint8")
// and shaders/quantize.metal:13-18,34-35 with the arithmetic of
// src/m5kernels/numerics.py:32-40 (quantize_reference):
//   peak = max |x| over the block
//   e    = clip(floor(log2(peak)) - 6, -127, 127), 0 for an all-zero block
//   q    = clip(rint(x / 2^e), -127, 127)         (int8; the S1.6 /64 of OCP
//                                                  MXINT8 folded into the scale)
//   byte = e + 127                                 (E8M0)
// floor(log2(peak)) is taken exactly, as the binary exponent of the fp32
// peak (subnormals included).  x / 2^e is an exact power-of-two scaling (a
// product that would be subnormal is below 1/2 and rounds to 0 either way),
// so the codes are exact round-half-even integers.
//
// HBM-bound: K*sizeof(T) bytes read, K + K/32 written per row.  A row of K
// elements (K % 32 == 0) holds whole blocks, so the tensor is a flat run of
// blocks: each thread loads one 16-byte vector (8 bf16/fp16 or 4 fp32
// values), the G = 32 / (values per vector) lanes of a block combine their
// peaks with xor shuffles, every lane writes its codes and the block's first
// lane its exponent byte.  Warps stride over the tensor in lock step, so the
// shuffles always see full warps.
#include <cstdint>

#include "common.cuh"
#include "m5b200.h"
#include "m5b_internal.h"
#include "quant_vec.cuh"

namespace m5b {
namespace {

constexpr int kThreads = 256;

// floor(log2(p)) of a positive finite fp32 value, exactly.
__device__ __forceinline__ int floor_log2(float p) {
  const uint32_t bits = __float_as_uint(p);
  const int biased = static_cast<int>((bits >> 23) & 0xFFu);
  if (biased != 0) return biased - 127;
  const uint32_t mant = bits & 0x7FFFFFu;  // subnormal: value = mant * 2^-149
  return (31 - __clz(static_cast<int>(mant))) - 149;
}

// 2^-e as fp32 for e in [-127, 127] (2^-127 is the subnormal 0x00400000).
__device__ __forceinline__ float pow2_neg(int e) {
  return e >= 127 ? __uint_as_float(0x00400000u) : __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
}

__device__ __forceinline__ uint32_t mx_code(float x, float m) {
  int c = __float2int_rn(__fmul_rn(x, m));
  c = c > 127 ? 127 : (c < -127 ? -127 : c);
  return static_cast<uint32_t>(c) & 0xFFu;
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
    mxint8_kernel(const T* __restrict__ x, int64_t nvec, uint8_t* __restrict__ q,
                  uint8_t* __restrict__ ebytes) {
  constexpr int V = qv::kVec<T>;  // values per 16-byte vector
  constexpr int G = 32 / V;       // lanes per 32-value block
  const int lane = threadIdx.x & 31;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  const int64_t stride = int64_t(gridDim.x) * kThreads;
  for (int64_t base = int64_t(blockIdx.x) * kThreads + (threadIdx.x & ~31); base < nvec;
       base += stride) {
    const int64_t v = base + lane;
    const bool in = v < nvec;
    const uint4 raw = in ? __ldcs(xv + v) : make_uint4(0, 0, 0, 0);
    qv::Peak<T> pk;
    pk.add(raw);
    float peak = pk.value();
#pragma unroll
    for (int off = 1; off < G; off <<= 1) peak = fmaxf(peak, __shfl_xor_sync(0xffffffffu, peak, off));
    int e = 0;
    if (peak > 0.0f) {
      e = floor_log2(peak) - 6;
      e = e < -127 ? -127 : (e > 127 ? 127 : e);
    }
    if (!in) continue;
    const float m = pow2_neg(e);
    float vals[V];
    qv::unpack<T>(raw, vals);
    uint32_t w[V / 4];
#pragma unroll
    for (int i = 0; i < V / 4; ++i)
      w[i] = mx_code(vals[4 * i], m) | (mx_code(vals[4 * i + 1], m) << 8) |
             (mx_code(vals[4 * i + 2], m) << 16) | (mx_code(vals[4 * i + 3], m) << 24);
    if constexpr (V == 8)
      reinterpret_cast<uint2*>(q)[v] = make_uint2(w[0], w[1]);
    else
      reinterpret_cast<uint32_t*>(q)[v] = w[0];
    if ((lane & (G - 1)) == 0) ebytes[v / G] = static_cast<uint8_t>(e + 127);
  }
}

template <typename T>
cudaError_t launch_mx(const void* x, int64_t n, void* q, uint8_t* e, cudaStream_t stream) {
  auto kern = mxint8_kernel<T>;
  static std::atomic<long long> shape[kMaxLaunchDevices];
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t err = launch_shape(reinterpret_cast<const void*>(kern), kThreads, 0, shape, &dev,
                                 &sms, &per_sm);
  if (err != cudaSuccess) return err;
  const int64_t nvec = n / qv::kVec<T>;
  int64_t grid = int64_t(sms) * per_sm;
  const int64_t need = (nvec + kThreads - 1) / kThreads;
  if (grid > need) grid = need;
  kern<<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(
      reinterpret_cast<const T*>(x), nvec, reinterpret_cast<uint8_t*>(q), e);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_mxint8(const void* x, int x_dtype, int64_t n, void* q, uint8_t* e,
                          cudaStream_t stream) {
  switch (x_dtype) {
    case DT_BF16: return launch_mx<__nv_bfloat16>(x, n, q, e, stream);
    case DT_F16: return launch_mx<__half>(x, n, q, e, stream);
    case DT_F32: return launch_mx<float>(x, n, q, e, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace m5b
