// Lean row-preparation kernels for the common shapes: rotation (+ per-token
// quantization) of plain rows, and the fused RMS / LayerNorm + AdaLN
// modulation (+ gated residual) + rotation + quantization.
//
// Reference contracts: src/m5kernels/hadamard.py:33-77 (rotate: X D H with
// the signs applied before the Sylvester-order Walsh-Hadamard transform of
// each block of B channels, scaled by 1/sqrt(B)), hadamard_gemm.py:65-66
// (quantize(rotate(x))), numerics.py:29-46 (per-token symmetric INT8 / E4M3),
// norm_hadamard.py:122-176 and 198-265 (fused norm / gated residual forms).
//
// These are lean forms of row_prep_kernel (prep_impl.cuh); the results are
// identical bit for bit (same reduction tree, same butterfly order, same
// rounding of every operation), only the schedule differs:
//   * CTAs split into independent pipeline units of max(K/64, 32) threads
//     (one thread per 64-element chunk, as in row_prep_kernel): a unit of
//     K = 4096 is two warps on one row, a unit of K = 1024 is one warp on two
//     rows.  Each unit has its own ring of row slots in shared memory filled
//     by TMA (its first thread issues, one mbarrier per slot) and
//     synchronises with a named barrier (or __syncwarp), so the units of a
//     CTA never wait for one another.
//   * Chunk values are held as 32 float2 pairs (elements 2k, 2k+1) so that
//     the chunk sums, the modulation, the gated update, every Hadamard stage
//     of stride >= 2, the 1/sqrt(B) scale and the INT8 rounding run on sm_100
//     packed FP32 instructions (two IEEE binary32 operations per
//     instruction); cross-lane stages exchange values with shuffles and
//     combine with one packed FMA by +-1.
//   * Each mode (plain, norm, gated norm) is its own instantiation, which
//     keeps the instruction footprint small.
#pragma once
#include <type_traits>

#include "prep_impl.cuh"

namespace m5b {
namespace rotq {

constexpr int kThreads = 256;
constexpr int kMaxStages = 4;
constexpr int kMaxUnits = kThreads / 32;
enum Mode : int { kPlain = 0, kNorm = 1, kNormGated = 2 };

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

// Eight elements [8 i, 8 i + 8) of chunk t of a swizzled staged row.
template <typename T>
__device__ __forceinline__ void load8(const uint8_t* base, int t, int i, float2* out) {
  if constexpr (sizeof(T) == 2) {
    const uint4 raw = *swz_slot(base, t, i);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      if constexpr (std::is_same<T, __nv_bfloat16>::value)
        out[p] = make_float2(__uint_as_float(w[p] << 16), __uint_as_float(w[p] & 0xFFFF0000u));
      else
        out[p] = __half22float2(*reinterpret_cast<const __half2*>(&w[p]));
    }
  } else {
    const int br = 2 * t + (i >= 4 ? 1 : 0);
    const int sl = (i % 4) * 2;
    const uint4 p = *swz_slot(base, br, sl);
    const uint4 q = *swz_slot(base, br, sl + 1);
    out[0] = make_float2(__uint_as_float(p.x), __uint_as_float(p.y));
    out[1] = make_float2(__uint_as_float(p.z), __uint_as_float(p.w));
    out[2] = make_float2(__uint_as_float(q.x), __uint_as_float(q.y));
    out[3] = make_float2(__uint_as_float(q.z), __uint_as_float(q.w));
  }
}

// Eight values of a parameter table of the input dtype T as raw bits,
// loaded ahead of their use (the tables are read from L2 / L1 on every row,
// so the next group's loads are issued before the current group is
// computed).
template <typename T>
struct Raw8 {
  uint4 w[sizeof(T) == 4 ? 2 : 1];
};
template <typename T>
__device__ __forceinline__ Raw8<T> raw8_load(const void* base, int64_t j) {
  Raw8<T> r;
  const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(base) + j);
  r.w[0] = __ldg(p);
  if constexpr (sizeof(T) == 4) r.w[1] = __ldg(p + 1);
  return r;
}
// Value pair q (elements 2q, 2q+1) of a Raw8.
template <typename T>
__device__ __forceinline__ float2 raw8_pair(const Raw8<T>& r, int q) {
  if constexpr (sizeof(T) == 4) {
    const uint4& v = r.w[q >> 1];
    return (q & 1) ? make_float2(__uint_as_float(v.z), __uint_as_float(v.w))
                   : make_float2(__uint_as_float(v.x), __uint_as_float(v.y));
  } else {
    const uint32_t x = q == 0 ? r.w[0].x : q == 1 ? r.w[0].y : q == 2 ? r.w[0].z : r.w[0].w;
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
      return make_float2(__uint_as_float(x << 16), __uint_as_float(x & 0xFFFF0000u));
    else
      return __half22float2(*reinterpret_cast<const __half2*>(&x));
  }
}

// Table slices through shared memory: the 32 chunks of a warp cover 4 KB of
// a 16-bit table row.  The warp loads the 4 KB coalesced (lane l takes 16-byte
// vectors l, l + 32, ...) and stores each vector where its owning lane reads
// it, in the same swizzled layout as a staged activation row (chunk at 128-byte
// row `lane`, 16-byte slot s at s ^ (lane & 7)); owners then read their
// 128 bytes conflict-free.  Per-lane 16-byte loads from global memory would
// touch 32 lines per instruction instead of 4.
__device__ __forceinline__ void stage_table16(uint8_t* wbuf, const void* seg, int lane) {
  const uint4* g4 = reinterpret_cast<const uint4*>(seg);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint4 v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __ldg(g4 + lane + 32 * (4 * h + i));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = lane + 32 * (4 * h + i);
      const int owner = idx >> 3, slot = idx & 7;
      *reinterpret_cast<uint4*>(wbuf + owner * 128 + ((slot ^ (owner & 7)) << 4)) = v[i];
    }
  }
}

// Round a pair through T (RNE) and back.
template <typename T>
__device__ __forceinline__ float2 round2(float2 y) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    return __bfloat1622float2(__float22bfloat162_rn(y));
  else if constexpr (std::is_same<T, __half>::value)
    return __half22float2(__float22half2_rn(y));
  else
    return y;
}

// Store 8 values (already representable in T) at dst.
template <typename T>
__device__ __forceinline__ void store8(T* dst, const float2* v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    __nv_bfloat162 h[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) h[p] = __float22bfloat162_rn(v[p]);
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(h);
  } else if constexpr (std::is_same<T, __half>::value) {
    __half2 h[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) h[p] = __float22half2_rn(v[p]);
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(h);
  } else {
    reinterpret_cast<float4*>(dst)[0] = make_float4(v[0].x, v[0].y, v[1].x, v[1].y);
    reinterpret_cast<float4*>(dst)[1] = make_float4(v[2].x, v[2].y, v[3].x, v[3].y);
  }
}

// Canonical sum over a 64-element chunk held as 32 pairs: its four
// 16-element chunks (chunk16_sum) combined pairwise.  KIND 0: v, 1: v*v,
// 2: (v-mean)^2.
template <int KIND>
__device__ __forceinline__ float chunk_sum2(const float2* v, float mean) {
  float c[4];
  const float2 nm = f2(-mean);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (KIND == 2) {
      float2 d[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) d[k] = __fadd2_rn(v[8 * i + k], nm);
      c[i] = chunk16_sum<true>(d);
    } else {
      c[i] = chunk16_sum<KIND == 1>(v + 8 * i);
    }
  }
  return __fadd_rn(__fadd_rn(c[0], c[1]), __fadd_rn(c[2], c[3]));
}

// Pipeline units: a unit is max(K/64, 32) threads working on RPU = unit / (K/64)
// rows at a time, with its own ring of `stages` slots and mbarriers, so the
// units of a CTA never wait for one another (a named barrier, or __syncwarp
// for one-warp units, synchronises a unit).
// Plain rows: two 256-thread CTAs per SM (128 registers).  Normalized rows
// run 1-2 units per CTA (shared memory bounds them to ~8 warps per SM), so
// they may use more registers.
template <typename T, int B, int OUT, int MODE>
__global__ void __launch_bounds__(kThreads, MODE == kPlain ? 2 : 1)
    lean_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_b,
                const RowPrepArgs a, const int tpr, const int stages, const int box_rows,
                const int64_t buf_stride, const int tbl_off) {
  constexpr int LANE_SPAN = B / kChunk;  // lanes per Hadamard block (B >= 64)
  constexpr int INPUTS = MODE == kNormGated ? 2 : 1;
  extern __shared__ uint8_t dsmem_raw[];
  uint8_t* dsmem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(dsmem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ float red[kThreads / 32];
  __shared__ float red_sum[kThreads / 32];
  __shared__ float red_var[kThreads / 32];
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
  const int64_t row_slot = int64_t(INPUTS) * buf_stride;  // one row's inputs
  const int64_t slot_bytes = int64_t(RPU) * row_slot;
  uint8_t* ring = dsmem + int64_t(u) * stages * slot_bytes;
  // Normalized rows with K >= 2048: 8 KB per warp for table slices (tbl_off > 0)
  uint8_t* tbl_a = dsmem + tbl_off + (tid >> 5) * 8192;
  uint8_t* tbl_b = tbl_a + 4096;
  (void)tbl_off;
  uint64_t* bars = full_bar + u * kMaxStages;
  const int64_t first_step = int64_t(blockIdx.x) * U + u;
  const int64_t step_stride = int64_t(gridDim.x) * U;
  auto unit_sync = [&]() {
    if (PW == 32)
      __syncwarp();
    else
      named_sync(1 + u, PW);
  };
  // Canonical row sum: lanes continue the pairwise tree over chunk index,
  // then the unit's warps pairwise in index order, the total added to +0.
  // Also a unit barrier.
  auto unit_sum = [&](float v, float* buf) -> float {
    const int span = tpr < 32 ? tpr : 32;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1)
      if (off < span) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    if (tpr > 32 && lane == 0) buf[tid >> 5] = v;
    unit_sync();
    if (tpr > 32) {
      const int w0 = (u * PW) >> 5, W = PW >> 5;
      float part[kThreads / 32];
#pragma unroll
      for (int w = 0; w < kThreads / 32; ++w) part[w] = w < W ? buf[w0 + w] : 0.0f;
#pragma unroll
      for (int step = 1; step < kThreads / 32; step <<= 1)
#pragma unroll
        for (int w = 0; w + step < kThreads / 32; w += 2 * step)
          part[w] = __fadd_rn(part[w], part[w + step]);
      v = part[0];
    }
    return __fadd_rn(v, 0.0f);
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
    mbar_arrive_expect_tx(&bars[s], static_cast<uint32_t>(n * INPUTS * row_bytes));
    for (int r = 0; r < n; ++r)
      for (int c = 0; c < row_box_rows; c += box_rows) {
        tma_load_3d(dst + r * row_slot + c * 128, &map_x, &bars[s], 0, c,
                    static_cast<int32_t>(first + r));
        if constexpr (MODE == kNormGated)
          tma_load_3d(dst + r * row_slot + buf_stride + c * 128, &map_b, &bars[s], 0, c,
                      static_cast<int32_t>(first + r));
      }
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
    const uint8_t* xslot = ring + s * slot_bytes + rr * row_slot;
    auto refill = [&]() {
      if (leader && st + int64_t(stages) * step_stride < steps_total)
        issue(st + int64_t(stages) * step_stride, s);
    };

    float2 v[32];
    if constexpr (MODE == kPlain) {
      if (live) {
        load_chunk<T>(xslot, t, a.signs != nullptr ? a.signs + j0 : nullptr, v);
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] = f2(0.0f);
      }
    } else {
      if (live) {
#pragma unroll
        for (int i = 0; i < 8; ++i) load8<T>(xslot, t, i, v + 4 * i);
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] = f2(0.0f);
      }
      if constexpr (MODE == kNormGated) {
        // R' = cast_T(R + branch * gate), written once.
        if (live) {
          const int64_t goff = a.gate_row_map ? int64_t(a.gate_row_map[row]) * K : 0;
          T* rrow = reinterpret_cast<T*>(a.r_out) + row * K + j0;
          stage_table16(tbl_a, reinterpret_cast<const T*>(a.gate) + goff + (j0 - 64 * lane), lane);
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            Raw8<T> gc;
            gc.w[0] = *swz_slot(tbl_a, lane, i);
            float2 br[4];
            load8<T>(xslot + buf_stride, t, i, br);
#pragma unroll
            for (int p = 0; p < 4; ++p)
              v[4 * i + p] = round2<T>(
                  __ffma2_rn(br[p], raw8_pair<T>(gc, p), v[4 * i + p]));
            store8<T>(rrow + 8 * i, v + 4 * i);
          }
        }
      }
      // ---- normalization statistics (canonical tree) -----------------------
      const float kf = static_cast<float>(K);
      const float first = __fdiv_rn(
          unit_sum(a.norm == NORM_LAYER ? chunk_sum2<0>(v, 0.0f) : chunk_sum2<1>(v, 0.0f), red_sum),
          kf);
      refill();  // every thread of the unit has read slot s
      float mean = 0.0f, moment = first;
      if (a.norm == NORM_LAYER) {
        mean = first;
        moment = __fdiv_rn(unit_sum(chunk_sum2<2>(v, mean), red_var), kf);
      }
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(moment, a.eps)));
      // ---- modulation, optional rounding, signs ------------------------------
      if (live) {
        const int64_t moff = a.row_map ? int64_t(a.row_map[row]) * K : 0;
        const float2 nm = f2(-mean), inv2 = f2(inv);
        // gamma and scale slices, then t = ((v - mean) * inv) * gamma in place;
        // then the shift slice and y = fma(t, 1 + scale, shift).
        const int64_t wcol = j0 - 64 * lane;  // the warp's first column
        __syncwarp();  // every lane is done with the gate slice
        stage_table16(tbl_a, reinterpret_cast<const T*>(a.gamma) + wcol, lane);
        stage_table16(tbl_b, reinterpret_cast<const T*>(a.scale) + moff + wcol, lane);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          Raw8<T> gc;
          gc.w[0] = *swz_slot(tbl_a, lane, i);
#pragma unroll
          for (int p = 0; p < 4; ++p)
            v[4 * i + p] = __fmul2_rn(__fmul2_rn(__fadd2_rn(v[4 * i + p], nm), inv2),
                                      raw8_pair<T>(gc, p));
        }
        __syncwarp();
        stage_table16(tbl_a, reinterpret_cast<const T*>(a.shift) + moff + wcol, lane);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          Raw8<T> cc, hc;
          cc.w[0] = *swz_slot(tbl_b, lane, i);
          hc.w[0] = *swz_slot(tbl_a, lane, i);
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const float2 one_sc = __fadd2_rn(f2(1.0f), raw8_pair<T>(cc, p));
            float2 y = __ffma2_rn(v[4 * i + p], one_sc, raw8_pair<T>(hc, p));
            if (a.round_output) y = round2<T>(y);
            v[4 * i + p] = y;
          }
        }
        __syncwarp();  // slices read before the next row's gate slice
        if (a.signs != nullptr) {
#pragma unroll
          for (int i = 0; i < kChunk; i += 16) {
            const uint4 sv = __ldg(reinterpret_cast<const uint4*>(a.signs + j0 + i));
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
      if constexpr (MODE == kPlain) refill();
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
      unit_sync();  // warp peaks visible (plain mode: slot s consumed)
      if constexpr (MODE == kPlain) refill();
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
            // the 8 pairs are 16 consecutive floats in element order
            e4m3_words<4>(reinterpret_cast<const float*>(p), scale, rinv, fast, words);
          } else if (scale >= kI8DivMinScale) {
            // correctly rounded quotients of the packed pairs (i8_pair_div)
            const I8Div d = i8_div(rinv, scale);
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              const float2 m0 = i8_pair_div(p[2 * w], d);
              const float2 m1 = i8_pair_div(p[2 * w + 1], d);
              words[w] = pack4_low_bytes(m0.x, m0.y, m1.x, m1.y);
            }
          } else {  // scale below 2^-90: divide exactly
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

// The lean kernels take rows staged by TMA (16-byte aligned, K % 64 == 0)
// with 16-byte aligned outputs, signs and parameter tables, whose chunks
// tile a unit (K / 64 a power of two below 32, or a multiple of 32 up to
// 256), rotated with B >= 64 (B <= 256 with normalization).  Plain rows also
// need a row-group slot (rows padded to 1024 bytes for the swizzle) of at
// most 64 KB; normalized rows a two-stage ring of at most 200 KB.
inline int mode_of(const RowPrepArgs& a) {
  if (a.rms_quant != RMSQ_NONE) return -1;  // row_prep_kernel's RMS folding form
  if (a.norm == NORM_NONE) return a.branch ? -1 : kPlain;
  return a.branch ? kNormGated : kNorm;
}

inline bool applicable(const RowPrepArgs& a, const RowMaps& m, int block, int out,
                       int elem_bytes, int x_dtype) {
  const int mode = mode_of(a);
  if (mode < 0 || block < 64 || !m.valid || !a.vec_ok) return false;
  if (mode != kPlain && (block > 256 || out == OUT_F32 || !a.params_vec || a.K < 2048)) return false;
  // normalized rows: 16-bit inputs with modulation (and gate) tables of the
  // input dtype (fp32 rows do not fit the registers of this schedule)
  if (mode != kPlain && (elem_bytes != 2 || a.gamma_dtype != x_dtype || a.scale_dtype != x_dtype ||
                         a.shift_dtype != x_dtype || (a.gate && a.gate_dtype != x_dtype)))
    return false;
  if (a.signs != nullptr && !a.params_vec) return false;
  if (a.K % kChunk) return false;
  const int64_t tpr = a.K / kChunk;
  if (tpr < 32 ? (32 % tpr) != 0 : (tpr % 32 != 0 || tpr > kThreads)) return false;
  const int64_t buf_stride = (a.K * elem_bytes + 1023) & ~int64_t(1023);
  const int64_t pw = tpr >= 32 ? tpr : 32;
  const int64_t unit_slot = (mode == kNormGated ? 2 : 1) * (pw / tpr) * buf_stride;
  if (mode == kPlain) return (kThreads / pw) * unit_slot <= 64 * 1024;
  return 2 * unit_slot <= 200 * 1024;
}

template <typename T, int B, int OUT, int MODE>
cudaError_t launch_m(const RowPrepArgs& a, const RowMaps& m, cudaStream_t stream) {
  auto kern = lean_kernel<T, B, OUT, MODE>;
  const int tpr = static_cast<int>(a.K / kChunk);
  const int pw = tpr >= 32 ? tpr : 32;  // threads per pipeline unit
  const int rpu = pw / tpr;
  const int64_t row_bytes = a.K * int64_t(sizeof(T));
  const int64_t buf_stride = (row_bytes + 1023) & ~int64_t(1023);
  const int64_t unit_slot = int64_t(MODE == kNormGated ? 2 : 1) * rpu * buf_stride;
  int units, stages;
  // normalized rows (>= 2048 elements) stage their table slices per warp
  const int64_t tbl_per_unit = MODE != kPlain ? int64_t(pw / 32) * 8192 : 0;
  if (MODE == kPlain) {
    units = kThreads / pw;
    stages = static_cast<int>((110 * 1024) / (units * unit_slot));
    stages = stages < 2 ? 2 : (stages > 3 ? 3 : stages);
  } else {
    // Two stages per unit; as many units per CTA as keep the CTA near
    // 72 KB, so that three CTAs share an SM where the rows allow it.
    stages = 2;
    units = static_cast<int>((72 * 1024) / (stages * unit_slot + tbl_per_unit));
    units = units < 1 ? 1 : (units > kThreads / pw ? kThreads / pw : units);
  }
  const int threads = units * pw;
  const int tbl_off = tbl_per_unit ? static_cast<int>(int64_t(stages) * units * unit_slot) : 0;
  const int smem =
      static_cast<int>(int64_t(stages) * units * unit_slot + units * tbl_per_unit) + 1024;
  static std::atomic<long long> shape[kMaxLaunchDevices];
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e = launch_shape(reinterpret_cast<const void*>(kern), threads, smem, shape, &dev,
                               &sms, &per_sm);
  if (e != cudaSuccess) return e;
  const int64_t unit_steps = (a.rows + rpu - 1) / rpu;
  const int64_t ctas_needed = (unit_steps + units - 1) / units;
  int64_t grid = int64_t(sms) * per_sm;
  if (grid > ctas_needed) grid = ctas_needed;
  kern<<<static_cast<unsigned>(grid), threads, smem, stream>>>(
      m.x, MODE == kNormGated ? m.b : m.x, a, tpr, stages, m.box_rows, buf_stride, tbl_off);
  return cudaGetLastError();
}

template <typename T, int MODE, int OUT>
cudaError_t launch_bo(const RowPrepArgs& a, const RowMaps& m, int block, cudaStream_t stream) {
  switch (block) {
    case 64: return launch_m<T, 64, OUT, MODE>(a, m, stream);
    case 128: return launch_m<T, 128, OUT, MODE>(a, m, stream);
    case 256: return launch_m<T, 256, OUT, MODE>(a, m, stream);
    default: break;
  }
  if constexpr (MODE == kPlain) {
    switch (block) {
      case 512: return launch_m<T, 512, OUT, MODE>(a, m, stream);
      case 1024: return launch_m<T, 1024, OUT, MODE>(a, m, stream);
      default: break;
    }
  }
  return cudaErrorInvalidValue;
}

template <typename T, int MODE>
cudaError_t launch_mode(const RowPrepArgs& a, const RowMaps& m, int block, int out,
                        cudaStream_t stream) {
  switch (out) {
    case OUT_INT8: return launch_bo<T, MODE, OUT_INT8>(a, m, block, stream);
    case OUT_E4M3: return launch_bo<T, MODE, OUT_E4M3>(a, m, block, stream);
    case OUT_F32:
      if constexpr (MODE == kPlain) return launch_bo<T, MODE, OUT_F32>(a, m, block, stream);
      return cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t launch(const RowPrepArgs& a, const RowMaps& m, int block, int out,
                   cudaStream_t stream) {
  switch (mode_of(a)) {
    case kPlain: return launch_mode<T, kPlain>(a, m, block, out, stream);
    default: break;
  }
  if constexpr (sizeof(T) == 2) {
    switch (mode_of(a)) {
      case kNorm: return launch_mode<T, kNorm>(a, m, block, out, stream);
      case kNormGated: return launch_mode<T, kNormGated>(a, m, block, out, stream);
      default: break;
    }
  }
  return cudaErrorInvalidValue;
}

}  // namespace rotq
}  // namespace m5b
