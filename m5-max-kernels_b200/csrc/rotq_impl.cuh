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
//   * 256-thread CTAs, two per SM, split into independent pipeline units of
//     max(K/64, 32) threads (one thread per 64-element chunk, as in
//     row_prep_kernel): a unit of K = 4096 is two warps on one row, a unit of
//     K = 1024 is one warp on two rows.  Each unit has its own ring of row
//     slots in shared memory filled by TMA (its first thread issues, one
//     mbarrier per slot) and synchronises with a named barrier (or
//     __syncwarp), so the units of a CTA never wait for one another.
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
constexpr int kMaxUnits = kThreads / 32;

__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

// Elements [64 t, 64 t + 64) of a swizzled staged row as 32 (even, odd)
// pairs, with the Hadamard signs applied (sg: the chunk's 64 sign bytes, or
// null).  For 16-bit inputs the signs flip the two sign bits of a packed pair
// before it is widened (one byte permute + one 3-input logic op per pair).
template <typename T>
__device__ __forceinline__ void load_chunk(const uint8_t* base, int t, const int8_t* sg,
                                           float2* v) {
  if constexpr (sizeof(T) == 2) {
#pragma unroll
    for (int h = 0; h < 4; ++h) {  // 16 elements per sign vector
      uint4 sv = make_uint4(0u, 0u, 0u, 0u);
      if (sg != nullptr) sv = __ldg(reinterpret_cast<const uint4*>(sg) + h);
      const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int sl = 2 * h + q;
        const uint4 raw = *swz_slot(base, t, sl);
        uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          // sign bytes of elements 2p, 2p+1 of this slot -> bits 15 and 31
          const uint32_t word = sw[2 * q + p / 2];
          const uint32_t m = (p & 1) ? __byte_perm(word, 0u, 0x3424) : __byte_perm(word, 0u, 0x1404);
          w[p] ^= m & 0x80008000u;
          if constexpr (std::is_same<T, __nv_bfloat16>::value) {
            v[4 * sl + p] = make_float2(__uint_as_float(w[p] << 16), __uint_as_float(w[p] & 0xFFFF0000u));
          } else {
            v[4 * sl + p] = __half22float2(*reinterpret_cast<const __half2*>(&w[p]));
          }
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
    if (sg != nullptr) {
#pragma unroll
      for (int i = 0; i < kChunk; i += 16) {
        const uint4 sv = __ldg(reinterpret_cast<const uint4*>(sg + i));
        const uint32_t w[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float2& p0 = v[(i + 4 * q) / 2];
          float2& p1 = v[(i + 4 * q) / 2 + 1];
          p0.x = __uint_as_float(__float_as_uint(p0.x) ^ ((w[q] << 24) & 0x80000000u));
          p0.y = __uint_as_float(__float_as_uint(p0.y) ^ ((w[q] << 16) & 0x80000000u));
          p1.x = __uint_as_float(__float_as_uint(p1.x) ^ ((w[q] << 8) & 0x80000000u));
          p1.y = __uint_as_float(__float_as_uint(p1.y) ^ (w[q] & 0x80000000u));
        }
      }
    }
  }
}

__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Pipeline units: a unit is max(K/64, 32) threads working on RPU = unit / (K/64)
// rows at a time, with its own ring of `stages` slots and mbarriers, so the
// units of a CTA never wait for one another (a named barrier, or __syncwarp
// for one-warp units, synchronises a unit).
template <typename T, int B, int OUT>
__global__ void __launch_bounds__(kThreads, 2)
    rotq_kernel(const __grid_constant__ CUtensorMap map_x, const RowPrepArgs a, const int tpr,
                const int stages, const int box_rows, const int64_t buf_stride) {
  constexpr int LANE_SPAN = B / kChunk;  // lanes per Hadamard block (B >= 64)
  extern __shared__ uint8_t dsmem_raw[];
  uint8_t* dsmem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(dsmem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ float red[kThreads / 32];
  __shared__ __align__(8) uint64_t full_bar[kMaxUnits * kMaxStages];
  __shared__ int abort_flag[kMaxUnits];

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int PW = tpr >= 32 ? tpr : 32;  // threads per unit
  const int RPU = PW / tpr;             // rows per unit step
  const int U = blockDim.x / PW;        // units per CTA
  const int u = tid / PW;
  const int tu = tid - u * PW;
  const int rr = tu / tpr;              // row of the unit step
  const int t = tu - rr * tpr;          // chunk of the row
  const bool leader = tu == 0;
  const int64_t K = a.K;
  const int64_t j0 = int64_t(t) * kChunk;
  const int64_t row_bytes = K * int64_t(sizeof(T));
  const int row_box_rows = static_cast<int>(row_bytes / 128);
  const int64_t steps_total = (a.rows + RPU - 1) / RPU;  // row groups of RPU rows
  const int64_t slot_bytes = int64_t(RPU) * buf_stride;
  uint8_t* ring = dsmem + int64_t(u) * stages * slot_bytes;
  uint64_t* bars = full_bar + u * kMaxStages;
  const int64_t first_step = int64_t(blockIdx.x) * U + u;
  const int64_t step_stride = int64_t(gridDim.x) * U;
  auto unit_sync = [&]() {
    if (PW == 32)
      __syncwarp();
    else
      named_sync(1 + u, PW);
  };

  if (tid == 0) {
    for (int i = 0; i < U * kMaxStages; ++i) mbar_init(&full_bar[i], 1);
    for (int i = 0; i < U; ++i) abort_flag[i] = 0;
    fence_mbarrier_init();
  }
  __syncthreads();

  auto issue = [&](int64_t st, int s) {
    uint8_t* dst = ring + s * slot_bytes;
    const int64_t first = st * RPU;
    const int n = static_cast<int>(a.rows - first < RPU ? a.rows - first : RPU);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive_expect_tx(&bars[s], static_cast<uint32_t>(n * row_bytes));
    for (int r = 0; r < n; ++r)
      for (int c = 0; c < row_box_rows; c += box_rows)
        tma_load_3d(dst + r * buf_stride + c * 128, &map_x, &bars[s], 0, c,
                    static_cast<int32_t>(first + r));
  };
  if (leader) {
    for (int s = 0; s < stages; ++s) {
      const int64_t st = first_step + int64_t(s) * step_stride;
      if (st < steps_total) issue(st, s);
    }
  }

  const float2 isb = f2(a.inv_sqrt_block);
  int it = 0;
  for (int64_t st = first_step; st < steps_total; st += step_stride, ++it) {
    const int s = it % stages;
    const uint32_t parity = static_cast<uint32_t>((it / stages) & 1);
    if (leader) mbar_wait_bounded(&bars[s], parity, &abort_flag[u], a.status, DEV_TIMEOUT_PRODUCER);
    unit_sync();
    if (abort_flag[u]) break;
    (void)mbar_try_wait(&bars[s], parity);  // acquire of the TMA writes for every thread
    const int64_t row = st * RPU + rr;
    const bool live = row < a.rows;

    float2 v[32];
    if (live) {
      load_chunk<T>(ring + s * slot_bytes + rr * buf_stride, t,
                    a.signs != nullptr ? a.signs + j0 : nullptr, v);
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = f2(0.0f);
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
      unit_sync();  // slot s consumed
      if (leader && st + int64_t(stages) * step_stride < steps_total)
        issue(st + int64_t(stages) * step_stride, s);
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
      if (tpr > 32 && lane == 0) red[tid >> 5] = m;
      unit_sync();  // slot s consumed; warp peaks visible
      if (leader && st + int64_t(stages) * step_stride < steps_total)
        issue(st + int64_t(stages) * step_stride, s);
      if (tpr > 32) {
        const int w0 = (u * PW) >> 5;
        m = red[w0];
        for (int w = 1; w < (PW >> 5); ++w) m = fmaxf(m, red[w0 + w]);
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
            const I8Bracket br = i8_bracket(rinv, scale);
            uint32_t acc = 0u;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              const float2 m0 = i8_pair(p[2 * w], br, acc);
              const float2 m1 = i8_pair(p[2 * w + 1], br, acc);
              words[w] = pack4_low_bytes(m0.x, m0.y, m1.x, m1.y);
            }
            if (acc != 0u) {
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
  if (leader && abort_flag[u]) {
    // A wait gave up: let the copies already issued land before the unit exits.
    for (int s2 = 0; s2 < stages; ++s2) {
      const unsigned long long t0 = globaltimer_ns();
      for (uint32_t ph = 0; ph < 2; ++ph) {
        while (!mbar_try_wait(&bars[s2], ph)) {
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
  const int pw = tpr >= 32 ? tpr : 32;  // threads per pipeline unit
  const int units = kThreads / pw;
  const int threads = units * pw;
  const int rpu = pw / tpr;
  const int64_t row_bytes = a.K * int64_t(sizeof(T));
  const int64_t buf_stride = (row_bytes + 1023) & ~int64_t(1023);
  const int64_t slot = int64_t(units) * rpu * buf_stride;  // one slot of every unit
  int stages = static_cast<int>((110 * 1024) / slot);
  stages = stages < 2 ? 2 : (stages > 3 ? 3 : stages);
  const int smem = static_cast<int>(stages * slot) + 1024;
  static std::atomic<long long> shape[kMaxLaunchDevices];
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e = launch_shape(reinterpret_cast<const void*>(kern), threads, smem, shape, &dev,
                               &sms, &per_sm);
  if (e != cudaSuccess) return e;
  const int64_t unit_steps = (a.rows + rpu - 1) / rpu;
  const int64_t ctas_needed = (unit_steps + units - 1) / units;
  int64_t grid = int64_t(sms) * per_sm;
  if (grid > ctas_needed) grid = ctas_needed;
  kern<<<static_cast<unsigned>(grid), threads, smem, stream>>>(m.x, a, tpr, stages, m.box_rows,
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
