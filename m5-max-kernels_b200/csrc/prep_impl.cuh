// Row-preparation kernels: one CTA per activation row.
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
//
// Data layout in HBM: row-major [rows, K] activations; codes [rows, K] int8 /
// uint8 (E4M3 bits); scales fp32 [rows].  Each row is read once (128-bit loads,
// a warp reads 512 contiguous bytes of bf16 per instruction) and its codes are
// written once: 3K + 4 bytes per row for bf16 in / int8 out.
//
// Thread layout: a row is split into "units" of max(B, 256) elements.  Lane l
// of a warp owns elements l*8 .. l*8+7 of each 256-element slice of a unit, so
// Hadamard strides 1, 2, 4 are register butterflies, strides 8 .. 128 are
// warp shuffles (lane xor 1 .. 16) and strides 256 .. 512 are register
// butterflies across the slices a lane holds.  Units go round-robin to warps
// (unit = slot * W + warp).  Reductions (sum, sum of squares, max) are
// deterministic: per-thread sequential in (slot, slice, element) order, then a
// xor-butterfly over the warp, then warps 0..W-1 summed in order.  The C
// restatement in oracle/ follows the same order, which is what makes the
// codes and scales bit-comparable.
#pragma once
#include "common.cuh"
#include "m5b_internal.h"

namespace m5b {

constexpr int kMaxValues = 64;  // FP32 values a thread keeps in registers

template <typename T>
__device__ __forceinline__ void load8(const T* __restrict__ p, int64_t j0, int64_t K, bool vec,
                                      float (&out)[8]) {
  if (vec && j0 + 8 <= K) {
    if constexpr (sizeof(T) == 2) {
      uint4 raw = __ldg(reinterpret_cast<const uint4*>(p + j0));
      const T* h = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int e = 0; e < 8; ++e) out[e] = to_f32(h[e]);
    } else {
      float4 lo = __ldg(reinterpret_cast<const float4*>(p + j0));
      float4 hi = __ldg(reinterpret_cast<const float4*>(p + j0 + 4));
      out[0] = lo.x; out[1] = lo.y; out[2] = lo.z; out[3] = lo.w;
      out[4] = hi.x; out[5] = hi.y; out[6] = hi.z; out[7] = hi.w;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] = (j0 + e < K) ? to_f32(p[j0 + e]) : 0.0f;
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* __restrict__ p, int64_t j0, int64_t K, bool vec,
                                       const float (&v)[8]) {
  if (vec && j0 + 8 <= K) {
    if constexpr (sizeof(T) == 2) {
      uint4 raw;
      T* h = reinterpret_cast<T*>(&raw);
#pragma unroll
      for (int e = 0; e < 8; ++e) h[e] = from_f32<T>(v[e]);
      *reinterpret_cast<uint4*>(p + j0) = raw;
    } else {
      *reinterpret_cast<float4*>(p + j0) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(p + j0 + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (j0 + e < K) p[j0 + e] = from_f32<T>(v[e]);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// Sum the per-warp partials in warp order; every thread gets the same value.
__device__ __forceinline__ float block_sum(float v, float* red, int W) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = red[0];
  for (int w = 1; w < W; ++w) t = __fadd_rn(t, red[w]);
  __syncthreads();
  return t;
}
__device__ __forceinline__ float block_max(float v, float* red, int W) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = red[0];
  for (int w = 1; w < W; ++w) t = fmaxf(t, red[w]);
  __syncthreads();
  return t;
}

template <typename T, int B, int OUT>
__global__ void __launch_bounds__(512) row_prep_kernel(const RowPrepArgs a) {
  constexpr int UNIT = (B > 256) ? B : 256;
  constexpr int VPU = UNIT / 256;                    // 8-element slices per lane per unit
  constexpr int SLOTS = kMaxValues / (8 * VPU);      // units a warp can hold
  constexpr int LANE_SPAN = (B == 0) ? 1 : ((B < 256 ? B : 256) / 8);  // lanes per block slice
  __shared__ float red[32];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = a.warps;
  const int64_t row = blockIdx.x;
  const int64_t K = a.K;
  const int units = static_cast<int>((K + UNIT - 1) / UNIT);
  const bool vec = a.vec_ok != 0;

  const T* __restrict__ xrow = reinterpret_cast<const T*>(a.x) + row * K;
  float v[SLOTS][VPU][8];

  // ---- load (and gated residual update) ---------------------------------
  const T* __restrict__ brow = a.branch ? reinterpret_cast<const T*>(a.branch) + row * K : nullptr;
  const int64_t gate_off = (a.gate && a.gate_row_map) ? int64_t(a.gate_row_map[row]) * K : 0;
#pragma unroll
  for (int s = 0; s < SLOTS; ++s) {
    const int u = s * W + warp;
#pragma unroll
    for (int vv = 0; vv < VPU; ++vv) {
      const int64_t j0 = int64_t(u) * UNIT + vv * 256 + lane * 8;
      if (u < units) {
        load8<T>(xrow, j0, K, vec, v[s][vv]);
        if (brow) {
          float br[8];
          load8<T>(brow, j0, K, vec, br);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (j0 + e < K) {
              const float g = load_param(a.gate, a.gate_dtype, gate_off + j0 + e);
              v[s][vv][e] = round_through<T>(__fmaf_rn(br[e], g, v[s][vv][e]));
            }
          }
          store8<T>(reinterpret_cast<T*>(a.r_out) + row * K, j0, K, vec, v[s][vv]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[s][vv][e] = 0.0f;
      }
    }
  }

  // ---- normalization statistics --------------------------------------------
  float mean = 0.0f, inv = 1.0f;
  if (a.norm != NORM_NONE) {
    float acc = 0.0f;
#pragma unroll
    for (int s = 0; s < SLOTS; ++s) {
      const int u = s * W + warp;
      if (u < units) {
#pragma unroll
        for (int vv = 0; vv < VPU; ++vv) {
          const int64_t j0 = int64_t(u) * UNIT + vv * 256 + lane * 8;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (j0 + e < K) {
              const float x = v[s][vv][e];
              acc = (a.norm == NORM_LAYER) ? __fadd_rn(acc, x) : __fmaf_rn(x, x, acc);
            }
          }
        }
      }
    }
    const float kf = static_cast<float>(K);
    const float first = __fdiv_rn(block_sum(acc, red, W), kf);
    float moment = first;
    if (a.norm == NORM_LAYER) {
      mean = first;
      float acc2 = 0.0f;
#pragma unroll
      for (int s = 0; s < SLOTS; ++s) {
        const int u = s * W + warp;
        if (u < units) {
#pragma unroll
          for (int vv = 0; vv < VPU; ++vv) {
            const int64_t j0 = int64_t(u) * UNIT + vv * 256 + lane * 8;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              if (j0 + e < K) {
                const float d = __fsub_rn(v[s][vv][e], mean);
                acc2 = __fmaf_rn(d, d, acc2);
              }
            }
          }
        }
      }
      moment = __fdiv_rn(block_sum(acc2, red, W), kf);
    }
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(moment, a.eps)));
  }

  // ---- modulation, optional rounding, signs ----------------------------------
  const int64_t mod_off = a.row_map ? int64_t(a.row_map[row]) * K : 0;
#pragma unroll
  for (int s = 0; s < SLOTS; ++s) {
    const int u = s * W + warp;
    if (u < units) {
#pragma unroll
      for (int vv = 0; vv < VPU; ++vv) {
        const int64_t j0 = int64_t(u) * UNIT + vv * 256 + lane * 8;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int64_t j = j0 + e;
          if (j < K) {
            float y = v[s][vv][e];
            if (a.norm != NORM_NONE) {
              const float g = load_param(a.gamma, a.gamma_dtype, j);
              const float sc = load_param(a.scale, a.scale_dtype, mod_off + j);
              const float sh = load_param(a.shift, a.shift_dtype, mod_off + j);
              const float t = __fmul_rn(__fmul_rn(__fsub_rn(y, mean), inv), g);
              y = __fmaf_rn(t, __fadd_rn(1.0f, sc), sh);
              if (a.round_output) y = round_through<T>(y);
            }
            if (a.signs && a.signs[j] < 0) y = -y;
            v[s][vv][e] = y;
          }
        }
      }
    }
  }

  // ---- block Walsh-Hadamard transform (natural Sylvester order) -------------
  if constexpr (B > 0) {
#pragma unroll
    for (int s = 0; s < SLOTS; ++s) {
      const int u = s * W + warp;
      if (u < units) {  // warp-uniform: shuffles below see all 32 lanes
#pragma unroll
        for (int vv = 0; vv < VPU; ++vv) {
#pragma unroll
          for (int st = 1; st < 8; st <<= 1) {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              if ((e & st) == 0) {
                const float lo = v[s][vv][e], hi = v[s][vv][e + st];
                v[s][vv][e] = __fadd_rn(lo, hi);
                v[s][vv][e + st] = __fsub_rn(lo, hi);
              }
            }
          }
#pragma unroll
          for (int off = 1; off < LANE_SPAN; off <<= 1) {
            const bool upper = (lane & off) != 0;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float own = v[s][vv][e];
              const float peer = __shfl_xor_sync(0xffffffffu, own, off);
              v[s][vv][e] = upper ? __fsub_rn(peer, own) : __fadd_rn(own, peer);
            }
          }
        }
#pragma unroll
        for (int st = 1; st < VPU; st <<= 1) {
#pragma unroll
          for (int vv = 0; vv < VPU; ++vv) {
            if ((vv & st) == 0) {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float lo = v[s][vv][e], hi = v[s][vv + st][e];
                v[s][vv][e] = __fadd_rn(lo, hi);
                v[s][vv + st][e] = __fsub_rn(lo, hi);
              }
            }
          }
        }
#pragma unroll
        for (int vv = 0; vv < VPU; ++vv)
#pragma unroll
          for (int e = 0; e < 8; ++e) v[s][vv][e] = __fmul_rn(v[s][vv][e], a.inv_sqrt_block);
      }
    }
  }

  // ---- FP32 rotated output (standalone rotation) ----------------------------
  if constexpr (OUT == OUT_F32) {
    float* yrow = a.y + row * K;
#pragma unroll
    for (int s = 0; s < SLOTS; ++s) {
      const int u = s * W + warp;
      if (u < units) {
#pragma unroll
        for (int vv = 0; vv < VPU; ++vv)
          store8<float>(yrow, int64_t(u) * UNIT + vv * 256 + lane * 8, K, vec, v[s][vv]);
      }
    }
    return;
  } else {
    // ---- row peak and symmetric per-row scale ------------------------------
    float peak = 0.0f;
#pragma unroll
    for (int s = 0; s < SLOTS; ++s)
#pragma unroll
      for (int vv = 0; vv < VPU; ++vv)
#pragma unroll
        for (int e = 0; e < 8; ++e) peak = fmaxf(peak, fabsf(v[s][vv][e]));
    peak = block_max(peak, red, W);
    const float qmax = (OUT == OUT_E4M3) ? 448.0f : 127.0f;
    const float scale = (peak == 0.0f) ? 1.0f : __fdiv_rn(peak, qmax);
    if (threadIdx.x == 0) a.s[row] = scale;

    uint8_t* qrow = reinterpret_cast<uint8_t*>(a.q) + row * K;
#pragma unroll
    for (int s = 0; s < SLOTS; ++s) {
      const int u = s * W + warp;
      if (u < units) {
#pragma unroll
        for (int vv = 0; vv < VPU; ++vv) {
          const int64_t j0 = int64_t(u) * UNIT + vv * 256 + lane * 8;
          uint8_t c[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if constexpr (OUT == OUT_E4M3)
              c[e] = e4m3_code(v[s][vv][e], scale);
            else
              c[e] = static_cast<uint8_t>(int8_code(v[s][vv][e], scale));
          }
          if (vec && j0 + 8 <= K) {
            uint2 packed;
            packed.x = uint32_t(c[0]) | (uint32_t(c[1]) << 8) | (uint32_t(c[2]) << 16) |
                       (uint32_t(c[3]) << 24);
            packed.y = uint32_t(c[4]) | (uint32_t(c[5]) << 8) | (uint32_t(c[6]) << 16) |
                       (uint32_t(c[7]) << 24);
            *reinterpret_cast<uint2*>(qrow + j0) = packed;
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (j0 + e < K) qrow[j0 + e] = c[e];
          }
        }
      }
    }
  }
}

template <typename T, int B, int OUT>
static cudaError_t launch_t(const RowPrepArgs& a, cudaStream_t stream) {
  const unsigned threads = static_cast<unsigned>(a.warps) * 32u;
  row_prep_kernel<T, B, OUT><<<static_cast<unsigned>(a.rows), threads, 0, stream>>>(a);
  return cudaGetLastError();
}

template <typename T, int OUT>
static cudaError_t launch_b(const RowPrepArgs& a, int block, cudaStream_t stream) {
  switch (block) {
    case 0: return launch_t<T, 0, OUT>(a, stream);
    case 32: return launch_t<T, 32, OUT>(a, stream);
    case 64: return launch_t<T, 64, OUT>(a, stream);
    case 128: return launch_t<T, 128, OUT>(a, stream);
    case 256: return launch_t<T, 256, OUT>(a, stream);
    case 512: return launch_t<T, 512, OUT>(a, stream);
    case 1024: return launch_t<T, 1024, OUT>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
static cudaError_t launch_o(const RowPrepArgs& a, int block, int out, cudaStream_t stream) {
  switch (out) {
    case OUT_INT8: return launch_b<T, OUT_INT8>(a, block, stream);
    case OUT_E4M3: return launch_b<T, OUT_E4M3>(a, block, stream);
    case OUT_F32: return launch_b<T, OUT_F32>(a, block, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace m5b
