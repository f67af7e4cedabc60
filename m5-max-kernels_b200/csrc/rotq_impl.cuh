// Rotation + per-token quantization of plain rows: the online activation
// prep of the rotated W8A8 / FP8 projection (no normalization, no gated
// residual), and the FP32 rotation alone.
//
// Reference contracts: src/m5kernels/hadamard.py:33-77 (rotate: X D H with
// the signs applied before the Sylvester-order Walsh-Hadamard transform of
// each block of B channels, scaled by 1/sqrt(B)), hadamard_gemm.py:65-66
// (quantize(rotate(x))), numerics.py:29-46 (per-token symmetric INT8 / E4M3).
//
// This is the lean form of row_prep_kernel (prep_impl.cuh) for the common
// case; the results are identical bit for bit (same butterfly order, same
// rounding of every operation), only the schedule differs:
//   * 256-thread CTAs, two per SM, each working on G = 256 / (K/64) rows per
//     step (one thread per 64-element chunk, as in row_prep_kernel), so rows
//     of K = 4096 are handled four at a time and the CTA stays busy.
//   * A ring of row-group slots in shared memory filled by TMA (one thread
//     issues, one mbarrier per slot), two CTA barriers per step.
//   * Chunk values are held as 32 float2 pairs (elements 2k, 2k+1) so that
//     every Hadamard stage of stride >= 2, the 1/sqrt(B) scale and the INT8
//     rounding run on sm_100 packed FP32 instructions (two IEEE binary32
//     operations per instruction); cross-lane stages exchange values with
//     shuffles and combine with one packed FMA by +-1.
//   * Only this path's code is in the kernel (no norm, modulation or gate
//     branches), which keeps its instruction footprint small.
#pragma once
#include <type_traits>

#include "prep_impl.cuh"

namespace m5b {
namespace rotq {

constexpr int kThreads = 256;
constexpr int kMaxStages = 4;

__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

// Elements [64 t, 64 t + 64) of a swizzled staged row as 32 (even, odd) pairs.
template <typename T>
__device__ __forceinline__ void load_chunk(const uint8_t* base, int t, float2* v) {
  if constexpr (sizeof(T) == 2) {
#pragma unroll
    for (int sl = 0; sl < 8; ++sl) {
      const uint4 raw = *swz_slot(base, t, sl);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        if constexpr (std::is_same<T, __nv_bfloat16>::value) {
          v[4 * sl + p] = make_float2(__uint_as_float(w[p] << 16), __uint_as_float(w[p] & 0xFFFF0000u));
        } else {
          v[4 * sl + p] = __half22float2(*reinterpret_cast<const __half2*>(&w[p]));
        }
      }
    }
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int sl = 0; sl < 8; ++sl) {
        const uint4 raw = *swz_slot(base, 2 * t + h, sl);
        v[16 * h + 2 * sl] = make_float2(__uint_as_float(raw.x), __uint_as_float(raw.y));
        v[16 * h + 2 * sl + 1] = make_float2(__uint_as_float(raw.z), __uint_as_float(raw.w));
      }
    }
  }
}

// x -> -x where the sign byte is negative (bit flip of the IEEE sign).
__device__ __forceinline__ float flip(float x, uint32_t word, int byte) {
  const uint32_t bit = (word << (24 - 8 * byte)) & 0x80000000u;
  return __uint_as_float(__float_as_uint(x) ^ bit);
}

template <typename T, int B, int OUT>
__global__ void __launch_bounds__(kThreads, 2)
    rotq_kernel(const __grid_constant__ CUtensorMap map_x, const RowPrepArgs a, const int tpr,
                const int G, const int stages, const int box_rows, const int64_t buf_stride) {
  constexpr int LANE_SPAN = B / kChunk;  // lanes per Hadamard block (B >= 64)
  extern __shared__ uint8_t dsmem_raw[];
  uint8_t* dsmem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(dsmem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ float red[kThreads / 32];
  __shared__ __align__(8) uint64_t full_bar[kMaxStages];
  __shared__ int abort_flag;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int g = tid / tpr;         // row of the step
  const int t = tid - g * tpr;     // chunk of the row
  const int64_t K = a.K;
  const int64_t j0 = int64_t(t) * kChunk;
  const int64_t row_bytes = K * int64_t(sizeof(T));
  const int row_box_rows = static_cast<int>(row_bytes / 128);
  const int64_t groups = (a.rows + G - 1) / G;
  const int64_t slot_bytes = int64_t(G) * buf_stride;

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full_bar[s], 1);
    abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();

  auto issue = [&](int64_t grp, int s) {
    uint8_t* dst = dsmem + s * slot_bytes;
    const int64_t first = grp * G;
    const int n = static_cast<int>(a.rows - first < G ? a.rows - first : G);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive_expect_tx(&full_bar[s], static_cast<uint32_t>(n * row_bytes));
    for (int r = 0; r < n; ++r)
      for (int c = 0; c < row_box_rows; c += box_rows)
        tma_load_3d(dst + r * buf_stride + c * 128, &map_x, &full_bar[s], 0, c,
                    static_cast<int32_t>(first + r));
  };
  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      const int64_t grp = blockIdx.x + int64_t(s) * gridDim.x;
      if (grp < groups) issue(grp, s);
    }
  }

  const float2 isb = f2(a.inv_sqrt_block);
  int it = 0;
  for (int64_t grp = blockIdx.x; grp < groups; grp += gridDim.x, ++it) {
    const int s = it % stages;
    const uint32_t parity = static_cast<uint32_t>((it / stages) & 1);
    if (tid == 0)
      mbar_wait_bounded(&full_bar[s], parity, &abort_flag, a.status, DEV_TIMEOUT_PRODUCER);
    __syncthreads();
    if (abort_flag) break;
    (void)mbar_try_wait(&full_bar[s], parity);  // acquire of the TMA writes for every thread
    const int64_t row = grp * G + g;
    const bool live = g < G && row < a.rows;

    float2 v[32];
    if (live) {
      load_chunk<T>(dsmem + s * slot_bytes + g * buf_stride, t, v);
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = f2(0.0f);
    }
    // ---- signs (D) ---------------------------------------------------------
    if (a.signs != nullptr && live) {
#pragma unroll
      for (int i = 0; i < kChunk; i += 16) {
        const uint4 sg = __ldg(reinterpret_cast<const uint4*>(a.signs + j0 + i));
        const uint32_t w[4] = {sg.x, sg.y, sg.z, sg.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float2& p0 = v[(i + 4 * q) / 2];
          float2& p1 = v[(i + 4 * q) / 2 + 1];
          p0.x = flip(p0.x, w[q], 0);
          p0.y = flip(p0.y, w[q], 1);
          p1.x = flip(p1.x, w[q], 2);
          p1.y = flip(p1.y, w[q], 3);
        }
      }
    }
    // ---- Walsh-Hadamard transform of each B block (natural Sylvester order)
#pragma unroll
    for (int k = 0; k < 32; ++k) {  // stride 1: the two halves of a pair
      const float lo = v[k].x, hi = v[k].y;
      v[k] = make_float2(__fadd_rn(lo, hi), __fsub_rn(lo, hi));
    }
#pragma unroll
    for (int hp = 1; hp < 32; hp <<= 1) {  // strides 2 .. 32 (pair strides 1 .. 16)
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        if ((k & hp) == 0) {
          const float2 lo = v[k], hi = v[k + hp];
          v[k] = __fadd2_rn(lo, hi);
          v[k + hp] = __ffma2_rn(hi, f2(-1.0f), lo);  // lo - hi, one rounding
        }
      }
    }
#pragma unroll
    for (int off = 1; off < LANE_SPAN; off <<= 1) {  // strides 64 .. B/2 across lanes
      const float2 sg = f2((lane & off) ? -1.0f : 1.0f);  // upper: peer - own
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const float2 peer = make_float2(__shfl_xor_sync(0xffffffffu, v[k].x, off),
                                        __shfl_xor_sync(0xffffffffu, v[k].y, off));
        v[k] = __ffma2_rn(v[k], sg, peer);
      }
    }
#pragma unroll
    for (int k = 0; k < 32; ++k) v[k] = __fmul2_rn(v[k], isb);

    if constexpr (OUT == OUT_F32) {
      __syncthreads();  // slot s consumed
      if (tid == 0 && grp + int64_t(stages) * gridDim.x < groups)
        issue(grp + int64_t(stages) * gridDim.x, s);
      if (live) {
        float4* y = reinterpret_cast<float4*>(a.y + row * K + j0);
#pragma unroll
        for (int k = 0; k < 32; k += 2) y[k / 2] = make_float4(v[k].x, v[k].y, v[k + 1].x, v[k + 1].y);
      }
    } else {
      // ---- row peak ---------------------------------------------------------
      float m = 0.0f;
#pragma unroll
      for (int k = 0; k < 32; ++k) m = fmaxf(m, fmaxf(fabsf(v[k].x), fabsf(v[k].y)));
      const int span = tpr < 32 ? tpr : 32;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
        if (off < span) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      if (tpr >= 32 && lane == 0) red[tid >> 5] = m;
      __syncthreads();  // slot s consumed; warp peaks visible
      if (tid == 0 && grp + int64_t(stages) * gridDim.x < groups)
        issue(grp + int64_t(stages) * gridDim.x, s);
      if (tpr > 32) {
        const int w0 = (g * tpr) >> 5;
        m = red[w0];
        for (int w = 1; w < (tpr >> 5); ++w) m = fmaxf(m, red[w0 + w]);
      }
      if (live) {
        const float qmax = (OUT == OUT_E4M3) ? 448.0f : 127.0f;
        const float scale = (m == 0.0f) ? 1.0f : __fdiv_rn(m, qmax);
        const float rinv = __frcp_rn(scale);
        const bool fast = scale >= 0x1p-100f;
        if (t == 0) a.s[row] = scale;
        uint4* qrow = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(a.q) + row * K + j0);
#pragma unroll
        for (int grp16 = 0; grp16 < 4; ++grp16) {
          const float2* p = v + 8 * grp16;
          uint32_t words[4];
          if constexpr (OUT == OUT_E4M3) {
#pragma unroll
            for (int w = 0; w < 4; ++w)
              words[w] = quant_e4m3(p[2 * w].x, scale, rinv, fast) |
                         (quant_e4m3(p[2 * w].y, scale, rinv, fast) << 8) |
                         (quant_e4m3(p[2 * w + 1].x, scale, rinv, fast) << 16) |
                         (quant_e4m3(p[2 * w + 1].y, scale, rinv, fast) << 24);
          } else if (fast) {
            const float2 inv2 = f2(rinv);
            float dmax = 0.0f;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              uint32_t u[4];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const float2 tq = __fmul2_rn(p[2 * w + h], inv2);
                const float2 mq = __fadd2_rn(tq, f2(kRoundMagic));
                const float2 rq = __fadd2_rn(mq, f2(-kRoundMagic));
                const float2 dq = __ffma2_rn(rq, f2(-1.0f), tq);
                dmax = fmaxf(dmax, fmaxf(fabsf(dq.x), fabsf(dq.y)));
                u[2 * h] = __float_as_uint(mq.x);
                u[2 * h + 1] = __float_as_uint(mq.y);
              }
              words[w] = __byte_perm(__byte_perm(u[0], u[1], 0x0040),
                                     __byte_perm(u[2], u[3], 0x0040), 0x5410);
            }
            if (dmax > 0.5f - 0x1p-14f) {
              const Vals16 in{make_float4(p[0].x, p[0].y, p[1].x, p[1].y),
                              make_float4(p[2].x, p[2].y, p[3].x, p[3].y),
                              make_float4(p[4].x, p[4].y, p[5].x, p[5].y),
                              make_float4(p[6].x, p[6].y, p[7].x, p[7].y)};
              const uint4 qv = quant_i8_near_tie16(in, scale, rinv);
              words[0] = qv.x;
              words[1] = qv.y;
              words[2] = qv.z;
              words[3] = qv.w;
            }
          } else {  // scale below 2^-100: divide exactly
#pragma unroll
            for (int w = 0; w < 4; ++w)
              words[w] = (quant_i8(p[2 * w].x, scale, rinv, false) & 0xFF) |
                         ((quant_i8(p[2 * w].y, scale, rinv, false) & 0xFF) << 8) |
                         ((quant_i8(p[2 * w + 1].x, scale, rinv, false) & 0xFF) << 16) |
                         ((quant_i8(p[2 * w + 1].y, scale, rinv, false) & 0xFF) << 24);
          }
          qrow[grp16] = make_uint4(words[0], words[1], words[2], words[3]);
        }
      }
    }
  }
  if (abort_flag && tid == 0) {
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

// The lean kernel takes rows without normalization or gate, rotated with
// B >= 64, staged by TMA (16-byte aligned, K % 64 == 0), with 16-byte aligned
// signs and outputs, and rows whose chunks tile the 256-thread CTA (K / 64 a
// power of two below 32, or a multiple of 32 up to 256), and whose row-group
// slot (rows padded to 1024 bytes for the swizzle) is at most 64 KB.
inline bool applicable(const RowPrepArgs& a, const RowMaps& m, int block, int elem_bytes) {
  if (a.norm != NORM_NONE || a.branch != nullptr || block < 64 || !m.valid || !a.vec_ok)
    return false;
  if (a.signs != nullptr && !a.params_vec) return false;
  if (a.K % kChunk) return false;
  const int64_t tpr = a.K / kChunk;
  if (tpr < 32 ? (32 % tpr) != 0 : (tpr % 32 != 0 || tpr > kThreads)) return false;
  const int64_t buf_stride = (a.K * elem_bytes + 1023) & ~int64_t(1023);
  return (kThreads / tpr) * buf_stride <= 64 * 1024;
}

template <typename T, int B, int OUT>
cudaError_t launch_b(const RowPrepArgs& a, const RowMaps& m, cudaStream_t stream) {
  auto kern = rotq_kernel<T, B, OUT>;
  const int tpr = static_cast<int>(a.K / kChunk);
  const int G = kThreads / tpr;
  const int threads = ((G * tpr + 31) / 32) * 32;
  const int64_t row_bytes = a.K * int64_t(sizeof(T));
  const int64_t buf_stride = (row_bytes + 1023) & ~int64_t(1023);
  const int64_t slot = G * buf_stride;
  int stages = static_cast<int>((110 * 1024) / slot);
  stages = stages < 2 ? 2 : (stages > 3 ? 3 : stages);
  const int smem = static_cast<int>(stages * slot) + 1024;
  static std::atomic<long long> shape[kMaxLaunchDevices];
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e = launch_shape(reinterpret_cast<const void*>(kern), threads, smem, shape, &dev,
                               &sms, &per_sm);
  if (e != cudaSuccess) return e;
  const int64_t groups = (a.rows + G - 1) / G;
  int64_t grid = int64_t(sms) * per_sm;
  if (grid > groups) grid = groups;
  kern<<<static_cast<unsigned>(grid), threads, smem, stream>>>(m.x, a, tpr, G, stages, m.box_rows,
                                                               buf_stride);
  return cudaGetLastError();
}

template <typename T, int OUT>
cudaError_t launch_o(const RowPrepArgs& a, const RowMaps& m, int block, cudaStream_t stream) {
  switch (block) {
    case 64: return launch_b<T, 64, OUT>(a, m, stream);
    case 128: return launch_b<T, 128, OUT>(a, m, stream);
    case 256: return launch_b<T, 256, OUT>(a, m, stream);
    case 512: return launch_b<T, 512, OUT>(a, m, stream);
    case 1024: return launch_b<T, 1024, OUT>(a, m, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t launch(const RowPrepArgs& a, const RowMaps& m, int block, int out,
                   cudaStream_t stream) {
  switch (out) {
    case OUT_INT8: return launch_o<T, OUT_INT8>(a, m, block, stream);
    case OUT_E4M3: return launch_o<T, OUT_E4M3>(a, m, block, stream);
    case OUT_F32: return launch_o<T, OUT_F32>(a, m, block, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace rotq
}  // namespace m5b
