// Register-streamed row preparation: sixteen elements per thread.
//
// Same operator contracts as row_prep_kernel (prep_impl.cuh) and bit-identical
// results (same reduction tree, butterfly order and rounding of every
// operation); a different schedule for rows of 1024 to 8192 16-bit elements:
//   * thread s of a row owns elements [16 s, 16 s + 16): its 32 bytes are
//     contiguous, a warp reads 1 KB of the row with two coalesced 16-byte
//     loads per thread, straight into registers.  No shared-memory row ring:
//     the next row's loads are issued before the current row is computed;
//     one row per CTA (K / 16 threads), at most 64 registers per thread
//     (four 256-thread CTAs per SM for K = 4096).
//   * the canonical chunk of 64 elements ([64 t, 64 t + 64), eight
//     accumulators a[e] taking elements e, e + 8, ..., e + 56 in order) spans
//     the four threads of a quad: the accumulators pass down the quad with
//     shuffles, each thread adding its elements in order, so every chunk sum
//     is the one a thread holding the whole chunk computes.  Lanes then
//     combine chunks with a xor tree (chunk index bits 0-2 are lane bits
//     2-4), warps in fours (a 2048-element "old warp" of the canonical tree)
//     and those pairwise, padded to 16 with zeros.
//   * Hadamard strides 1-8 are register butterflies on packed pairs, strides
//     16-512 shuffles (lane xor 1, 2, 4, 8, 16), so B <= 512.
//   * modulation / gate / gamma slices are per-thread data (a thread always
//     handles the same 16 columns); they are kept in shared memory in a
//     conflict-free per-thread layout and reloaded only when the row's table
//     index changes.
// Modes: plain rotation (+ quantization), norm + AdaLN (+ gated residual),
// RMS scale folding (folded / direct); 16-bit inputs.
#pragma once
#include <type_traits>

#include "prep_impl.cuh"

namespace m5b {
namespace rows16 {

enum Mode : int { kPlain = 0, kNorm = 1, kNormGated = 2, kRms = 3 };
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }

// Sixteen 16-bit values (32 bytes) as two 16-byte words.
struct Raw16 {
  uint4 lo, hi;
};

__device__ __forceinline__ Raw16 ld_raw(const void* p) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
  Raw16 r;
  r.lo = __ldg(q);
  r.hi = __ldg(q + 1);
  return r;
}
// Streaming loads of activations (read once): no L1 allocation.
__device__ __forceinline__ Raw16 ld_raw_stream(const void* p) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
  Raw16 r;
  r.lo = __ldcs(q);
  r.hi = __ldcs(q + 1);
  return r;
}

// Pair k (elements 2k, 2k+1) of a Raw16 of T, as floats.
template <typename T>
__device__ __forceinline__ float2 pair_of(const Raw16& r, int k) {
  const uint4& w = k < 4 ? r.lo : r.hi;
  const int i = k & 3;
  const uint32_t x = i == 0 ? w.x : i == 1 ? w.y : i == 2 ? w.z : w.w;
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    return make_float2(__uint_as_float(x << 16), __uint_as_float(x & 0xFFFF0000u));
  else
    return __half22float2(*reinterpret_cast<const __half2*>(&x));
}

template <typename T>
__device__ __forceinline__ void unpack16(const Raw16& r, float2* v) {
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] = pair_of<T>(r, k);
}

template <typename T>
__device__ __forceinline__ float2 round2(float2 y) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    return __bfloat1622float2(__float22bfloat162_rn(y));
  else
    return __half22float2(__float22half2_rn(y));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float2 y) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const __nv_bfloat162 h = __float22bfloat162_rn(y);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __half2 h = __float22half2_rn(y);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

// Store sixteen values (already representable in T) as 32 bytes.
template <typename T>
__device__ __forceinline__ void st16(void* dst, const float2* v) {
  uint4* d = reinterpret_cast<uint4*>(dst);
  d[0] = make_uint4(pack2<T>(v[0]), pack2<T>(v[1]), pack2<T>(v[2]), pack2<T>(v[3]));
  d[1] = make_uint4(pack2<T>(v[4]), pack2<T>(v[5]), pack2<T>(v[6]), pack2<T>(v[7]));
}

// Per-thread table slots in shared memory: slot h (16 bytes) of thread t at
// (h * nthreads + t) * 16, so a warp's accesses are 512 contiguous bytes.
__device__ __forceinline__ uint4* tslot(uint8_t* base, int nthreads, int t, int h) {
  return reinterpret_cast<uint4*>(base + (int64_t(h) * nthreads + t) * 16);
}

// ---------------------------------------------------------------- reductions
// Canonical chunk sum of the quad's 64 elements (see the header comment):
// KIND 0 sum v, 1 sum v*v, 2 sum (v - mean)^2.  Every lane of the quad gets
// the chunk's sum; lanes past the row get 0.
template <int KIND>
__device__ __forceinline__ float quad_chunk_sum(const float2* v, float mean, int q, int lane,
                                                bool have) {
  float2 A[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) A[p] = f2(0.0f);
  const float2 nm = f2(-mean);
  // Branch-free: every lane adds its elements at every stage, but only lane
  // q == s holds the chain's accumulators at stage s (the others' results are
  // replaced by the shuffle that follows), so the chain is unchanged.
#pragma unroll
  for (int s = 0; s < 4; ++s) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const float2 x = v[4 * h + p];
        if constexpr (KIND == 0) {
          A[p] = __fadd2_rn(A[p], x);
        } else if constexpr (KIND == 1) {
          A[p] = __ffma2_rn(x, x, A[p]);
        } else {
          const float2 d = __fadd2_rn(x, nm);
          A[p] = __ffma2_rn(d, d, A[p]);
        }
      }
    }
    if (s < 3) {  // hand the accumulators to the next thread of the quad
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        A[p].x = __shfl_up_sync(kFull, A[p].x, 1);
        A[p].y = __shfl_up_sync(kFull, A[p].y, 1);
      }
    }
  }
  float c = __fadd_rn(__fadd_rn(__fadd_rn(A[0].x, A[0].y), __fadd_rn(A[1].x, A[1].y)),
                      __fadd_rn(__fadd_rn(A[2].x, A[2].y), __fadd_rn(A[3].x, A[3].y)));
  c = __shfl_sync(kFull, c, lane | 3);
  return have ? c : 0.0f;
}

// Row total of per-quad chunk sums in the canonical tree.  `part` holds one
// float per warp (this reduction's own buffer); one CTA barrier.  After the
// barrier lane l forms old warp l's sum (four new warps, pairwise) and the
// sixteen old-warp sums (zero-padded) are combined pairwise by a xor
// butterfly over lanes 0-15 -- the same pairing as a sequential pairwise
// tree -- and broadcast from lane 0.
__device__ __forceinline__ float old_warp_sum(const float* part, int l, int nwarps, int old_warps) {
  if (l >= old_warps) return 0.0f;
  const float p0 = 4 * l < nwarps ? part[4 * l] : 0.0f;
  const float p1 = 4 * l + 1 < nwarps ? part[4 * l + 1] : 0.0f;
  const float p2 = 4 * l + 2 < nwarps ? part[4 * l + 2] : 0.0f;
  const float p3 = 4 * l + 3 < nwarps ? part[4 * l + 3] : 0.0f;
  return __fadd_rn(__fadd_rn(p0, p1), __fadd_rn(p2, p3));
}
__device__ __forceinline__ float pairwise16(float o) {
#pragma unroll
  for (int off = 1; off < 16; off <<= 1) o = __fadd_rn(o, __shfl_xor_sync(kFull, o, off));
  return __shfl_sync(kFull, o, 0);
}

__device__ __forceinline__ float row_total(float c, float* part, int warp, int lane, int nwarps,
                                           int old_warps) {
  c = __fadd_rn(c, __shfl_xor_sync(kFull, c, 4));
  c = __fadd_rn(c, __shfl_xor_sync(kFull, c, 8));
  c = __fadd_rn(c, __shfl_xor_sync(kFull, c, 16));
  if (lane == 0) part[warp] = c;
  __syncthreads();
  return pairwise16(old_warp_sum(part, lane & 15, nwarps, old_warps));
}

__device__ __forceinline__ float row_max(float m, float* part, int warp, int lane, int nwarps) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, off));
  if (lane == 0) part[warp] = m;
  __syncthreads();
  // both half-warps reduce the same 16 partials (nwarps <= 16: rows of <= 8192)
  float t = (lane & 15) < nwarps ? part[lane & 15] : 0.0f;
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) t = fmaxf(t, __shfl_xor_sync(kFull, t, off));
  return t;
}

// Sum (canonical) and max with one barrier (RMS scale folding).
__device__ __forceinline__ float2 row_total_max(float c, float m, float* part, float* part_max,
                                                int warp, int lane, int nwarps, int old_warps) {
  c = __fadd_rn(c, __shfl_xor_sync(kFull, c, 4));
  c = __fadd_rn(c, __shfl_xor_sync(kFull, c, 8));
  c = __fadd_rn(c, __shfl_xor_sync(kFull, c, 16));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(kFull, m, off));
  if (lane == 0) {
    part[warp] = c;
    part_max[warp] = m;
  }
  __syncthreads();
  const float total = pairwise16(old_warp_sum(part, lane & 15, nwarps, old_warps));
  float t = (lane & 15) < nwarps ? part_max[lane & 15] : 0.0f;
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) t = fmaxf(t, __shfl_xor_sync(kFull, t, off));
  return make_float2(total, t);
}

// ---------------------------------------------------------------- transforms
// Signs of the thread's 16 columns (16 bytes of +-1) applied to its values.
__device__ __forceinline__ void apply_signs(float2* v, const int8_t* sg) {
  const uint4 sv = __ldg(reinterpret_cast<const uint4*>(sg));
  const uint32_t w[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
  for (int qd = 0; qd < 4; ++qd) {
    float2& p0 = v[2 * qd];
    float2& p1 = v[2 * qd + 1];
    p0.x = __uint_as_float(__float_as_uint(p0.x) ^ ((w[qd] << 24) & 0x80000000u));
    p0.y = __uint_as_float(__float_as_uint(p0.y) ^ ((w[qd] << 16) & 0x80000000u));
    p1.x = __uint_as_float(__float_as_uint(p1.x) ^ ((w[qd] << 8) & 0x80000000u));
    p1.y = __uint_as_float(__float_as_uint(p1.y) ^ (w[qd] & 0x80000000u));
  }
}

// Walsh-Hadamard butterflies of each B block (natural Sylvester order,
// increasing stride), then the 1/sqrt(B) scale.
template <int B>
__device__ __forceinline__ void fwht(float2* v, int lane, float isb) {
  if constexpr (B >= 2) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {  // stride 1: the halves of a pair
      const float lo = v[k].x, hi = v[k].y;
      v[k] = make_float2(__fadd_rn(lo, hi), __fsub_rn(lo, hi));
    }
  }
#pragma unroll
  for (int hp = 1; hp < 8 && 2 * hp < B; hp <<= 1) {  // strides 2, 4, 8
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if ((k & hp) == 0) {
        const float2 lo = v[k], hi = v[k + hp];
        v[k] = __fadd2_rn(lo, hi);
        v[k + hp] = __ffma2_rn(hi, f2(-1.0f), lo);  // lo - hi, one rounding
      }
    }
  }
#pragma unroll
  for (int off = 1; off < 32 && 16 * off < B; off <<= 1) {  // strides 16 .. B/2 across lanes
    const float2 sg = f2((lane & off) ? -1.0f : 1.0f);     // upper: peer - own
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float2 peer = make_float2(__shfl_xor_sync(kFull, v[k].x, off),
                                      __shfl_xor_sync(kFull, v[k].y, off));
      v[k] = __ffma2_rn(v[k], sg, peer);
    }
  }
  if constexpr (B >= 2) {
    const float2 s = f2(isb);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = __fmul2_rn(v[k], s);
  }
}

// ---------------------------------------------------------------- kernel
// B: rotation block (0: none).  OUT: OUT_INT8 / OUT_E4M3 / OUT_F32.
// MAXT: largest CTA (512 threads: rows of up to 8192 elements).
template <typename T, int B, int OUT, int MODE, int MAXT>
__global__ void __launch_bounds__(MAXT, 65536 / (MAXT * 64))
    rows16_kernel(const RowPrepArgs a, const int tbl_bytes) {
  extern __shared__ __align__(16) uint8_t tbl[];  // per-thread table slots
  __shared__ float red[2][4][MAXT / 32];           // [row parity][reduction][warp]
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int q = lane & 3;
  const int nthreads = blockDim.x;
  const int nwarps = nthreads >> 5;
  const int64_t K = a.K;
  const int tpr = static_cast<int>(K >> 4);
  const bool have = tid < tpr;
  const int64_t j0 = int64_t(have ? tid : 0) * 16;
  const int old_warps = static_cast<int>((K + 2047) / 2048);
  const float kf = static_cast<float>(K);

  // Table slots: gated: gate [0,2), norm: gamma [2,4), scale [4,6), shift [6,8);
  // RMS: gamma (fp32) [0,4).
  uint8_t* tb = tbl;
  int64_t cur_gmap = -1, cur_map = -1;
  (void)tbl_bytes;
  if constexpr (MODE == kNorm || MODE == kNormGated) {
    if (have) {  // gamma once (shared by all rows)
      const Raw16 g = ld_raw(reinterpret_cast<const T*>(a.gamma) + j0);
      *tslot(tb, nthreads, tid, 2) = g.lo;
      *tslot(tb, nthreads, tid, 3) = g.hi;
    }
  } else if constexpr (MODE == kRms) {
    if (have) {
      const uint4* gp = reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(a.gamma) + j0);
#pragma unroll
      for (int h = 0; h < 4; ++h) *tslot(tb, nthreads, tid, h) = __ldg(gp + h);
    }
  }

  int64_t row = blockIdx.x;
  Raw16 nx{}, nb{};
  if (have && row < a.rows) {
    nx = ld_raw_stream(reinterpret_cast<const T*>(a.x) + row * K + j0);
    if constexpr (MODE == kNormGated)
      nb = ld_raw_stream(reinterpret_cast<const T*>(a.branch) + row * K + j0);
  }
  int parity = 0;
  for (; row < a.rows; row += gridDim.x, parity ^= 1) {
    const Raw16 cx = nx, cb = nb;
    const int64_t next = row + gridDim.x;
    if (have && next < a.rows) {  // next row's loads in flight while this row is computed
      nx = ld_raw_stream(reinterpret_cast<const T*>(a.x) + next * K + j0);
      if constexpr (MODE == kNormGated)
        nb = ld_raw_stream(reinterpret_cast<const T*>(a.branch) + next * K + j0);
    }
    float* rs = red[parity][0];
    float* rv = red[parity][1];
    float* rm = red[parity][2];
    float2 v[8];
    unpack16<T>(cx, v);  // zeros past the row (cx is zero there)

    if constexpr (MODE == kNormGated) {
      // R' = cast_T(R + branch * gate), written once.
      if (have) {
        const int64_t gm = a.gate_row_map ? int64_t(__ldg(a.gate_row_map + row)) : 0;
        if (gm != cur_gmap) {
          const Raw16 g = ld_raw(reinterpret_cast<const T*>(a.gate) + gm * K + j0);
          *tslot(tb, nthreads, tid, 0) = g.lo;
          *tslot(tb, nthreads, tid, 1) = g.hi;
          cur_gmap = gm;
        }
        Raw16 g;
        g.lo = *tslot(tb, nthreads, tid, 0);
        g.hi = *tslot(tb, nthreads, tid, 1);
        float2 br[8];
        unpack16<T>(cb, br);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = round2<T>(__ffma2_rn(br[k], pair_of<T>(g, k), v[k]));
        st16<T>(reinterpret_cast<T*>(a.r_out) + row * K + j0, v);
      }
    }

    float inv = 1.0f;      // RMS folding: the row's inverse RMS
    float sq_chunk = 0.0f;
    if constexpr (MODE == kNorm || MODE == kNormGated) {
      const float c0 = (a.norm == NORM_LAYER) ? quad_chunk_sum<0>(v, 0.0f, q, lane, have)
                                              : quad_chunk_sum<1>(v, 0.0f, q, lane, have);
      const float first = __fdiv_rn(row_total(c0, rs, warp, lane, nwarps, old_warps), kf);
      float mean = 0.0f, moment = first;
      if (a.norm == NORM_LAYER) {
        mean = first;
        moment = __fdiv_rn(
            row_total(quad_chunk_sum<2>(v, mean, q, lane, have), rv, warp, lane, nwarps, old_warps),
            kf);
      }
      inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(moment, a.eps)));
      if (have) {
        const int64_t mm = a.row_map ? int64_t(__ldg(a.row_map + row)) : 0;
        if (mm != cur_map) {
          const Raw16 sc = ld_raw(reinterpret_cast<const T*>(a.scale) + mm * K + j0);
          const Raw16 sh = ld_raw(reinterpret_cast<const T*>(a.shift) + mm * K + j0);
          *tslot(tb, nthreads, tid, 4) = sc.lo;
          *tslot(tb, nthreads, tid, 5) = sc.hi;
          *tslot(tb, nthreads, tid, 6) = sh.lo;
          *tslot(tb, nthreads, tid, 7) = sh.hi;
          cur_map = mm;
        }
        Raw16 g, sc, sh;
        g.lo = *tslot(tb, nthreads, tid, 2);
        g.hi = *tslot(tb, nthreads, tid, 3);
        sc.lo = *tslot(tb, nthreads, tid, 4);
        sc.hi = *tslot(tb, nthreads, tid, 5);
        sh.lo = *tslot(tb, nthreads, tid, 6);
        sh.hi = *tslot(tb, nthreads, tid, 7);
        const float2 nm = f2(-mean), inv2 = f2(inv);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float2 t = __fmul2_rn(__fmul2_rn(__fadd2_rn(v[k], nm), inv2), pair_of<T>(g, k));
          float2 y = __ffma2_rn(t, __fadd2_rn(f2(1.0f), pair_of<T>(sc, k)), pair_of<T>(sh, k));
          if (a.round_output) y = round2<T>(y);
          v[k] = y;
        }
      }
    } else if constexpr (MODE == kRms) {
      // statistics of the ORIGINAL row; direct form normalizes now, folded
      // form keeps the inverse RMS for the row scale
      sq_chunk = quad_chunk_sum<1>(v, 0.0f, q, lane, have);
      if (a.rms_quant == RMSQ_DIRECT) {
        const float moment = __fdiv_rn(row_total(sq_chunk, rs, warp, lane, nwarps, old_warps), kf);
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(moment, a.eps)));
      }
      if (have) {
        float gv[16];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const uint4 w = *tslot(tb, nthreads, tid, h);
          gv[4 * h] = __uint_as_float(w.x);
          gv[4 * h + 1] = __uint_as_float(w.y);
          gv[4 * h + 2] = __uint_as_float(w.z);
          gv[4 * h + 3] = __uint_as_float(w.w);
        }
        const bool direct = a.rms_quant == RMSQ_DIRECT;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float2 t = direct ? __fmul2_rn(v[k], f2(inv)) : v[k];
          v[k] = __fmul2_rn(t, make_float2(gv[2 * k], gv[2 * k + 1]));
        }
      }
    }
    if (a.signs != nullptr && have) apply_signs(v, a.signs + j0);
    fwht<B>(v, lane, a.inv_sqrt_block);

    if constexpr (OUT == OUT_F32) {
      if (have) {
        float4* y = reinterpret_cast<float4*>(a.y + row * K + j0);
#pragma unroll
        for (int k = 0; k < 8; k += 2) y[k / 2] = make_float4(v[k].x, v[k].y, v[k + 1].x, v[k + 1].y);
      }
    } else {
      float m = 0.0f;
#pragma unroll
      for (int k = 0; k < 8; ++k) m = fmaxf(m, fmaxf(fabsf(v[k].x), fabsf(v[k].y)));
      if (!have) m = 0.0f;
      float peak;
      if constexpr (MODE == kRms) {
        if (a.rms_quant == RMSQ_FOLD) {
          const float2 sm = row_total_max(sq_chunk, m, rs, rm, warp, lane, nwarps, old_warps);
          const float moment = __fdiv_rn(sm.x, kf);
          inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(moment, a.eps)));
          peak = sm.y;
        } else {
          peak = row_max(m, rm, warp, lane, nwarps);
          inv = 1.0f;
        }
      } else {
        peak = row_max(m, rm, warp, lane, nwarps);
      }
      if (have) {
        const float vv[16] = {v[0].x, v[0].y, v[1].x, v[1].y, v[2].x, v[2].y, v[3].x, v[3].y,
                              v[4].x, v[4].y, v[5].x, v[5].y, v[6].x, v[6].y, v[7].x, v[7].y};
        uint32_t words[4];
        float scale;
        if constexpr (MODE == kRms) {
          scale = (peak == 0.0f) ? 1.0f : __fdiv_rn(__fmul_rn(peak, inv), 127.0f);
          if (peak >= 0x1p-100f) {
            rel_i8_fast16(vv, peak, words);
          } else {
#pragma unroll
            for (int w = 0; w < 4; ++w)
              words[w] = (static_cast<uint32_t>(rel_i8_code(vv[4 * w], peak)) & 0xFFu) |
                         ((static_cast<uint32_t>(rel_i8_code(vv[4 * w + 1], peak)) & 0xFFu) << 8) |
                         ((static_cast<uint32_t>(rel_i8_code(vv[4 * w + 2], peak)) & 0xFFu) << 16) |
                         ((static_cast<uint32_t>(rel_i8_code(vv[4 * w + 3], peak)) & 0xFFu) << 24);
          }
        } else {
          const float qmax = (OUT == OUT_E4M3) ? 448.0f : 127.0f;
          scale = (peak == 0.0f) ? 1.0f : __fdiv_rn(peak, qmax);
          const float rinv = __frcp_rn(scale);
          const bool fast = scale >= 0x1p-100f;
          if constexpr (OUT == OUT_E4M3) {
#pragma unroll
            for (int w = 0; w < 4; ++w) words[w] = e4m3_word(vv + 4 * w, scale, rinv, fast);
          } else if (fast) {
            quant_i8_fast16(vv, scale, rinv, words);
          } else {
#pragma unroll
            for (int w = 0; w < 4; ++w)
              words[w] = (quant_i8(vv[4 * w], scale, rinv, false) & 0xFF) |
                         ((quant_i8(vv[4 * w + 1], scale, rinv, false) & 0xFF) << 8) |
                         ((quant_i8(vv[4 * w + 2], scale, rinv, false) & 0xFF) << 16) |
                         ((quant_i8(vv[4 * w + 3], scale, rinv, false) & 0xFF) << 24);
          }
        }
        if (tid == 0) a.s[row] = scale;
        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(a.q) + row * K + j0) =
            make_uint4(words[0], words[1], words[2], words[3]);
      }
    }
  }
}

// ---------------------------------------------------------------- dispatch
inline int mode_of(const RowPrepArgs& a) {
  if (a.rms_quant != RMSQ_NONE) return a.branch || a.norm != NORM_NONE ? -1 : kRms;
  if (a.norm == NORM_NONE) return a.branch ? -1 : kPlain;
  return a.branch ? kNormGated : kNorm;
}

// Rows of 1024..8192 16-bit elements (K % 64 == 0), 16-byte aligned rows,
// outputs, signs and tables of the input dtype (fp32 gamma for RMS folding);
// rotation blocks up to 512.  (Rows of 16384 would need 1024-thread CTAs at
// 64 registers, one per SM: the lean kernel of rotq_impl.cuh is faster there,
// measured 71 vs 78 us on H128 rotation + INT8 of M4096 K16384.)
inline bool applicable(const RowPrepArgs& a, int block, int out, int elem_bytes, int x_dtype) {
  const int mode = mode_of(a);
  if (mode < 0 || elem_bytes != 2 || !a.vec_ok || !a.params_vec) return false;
  if (a.K % 64 || a.K < 1024 || a.K > 8192) return false;
  if (block != 0 && (block < 2 || block > 512)) return false;
  if (out == OUT_ROW) return false;
  if (mode == kNorm || mode == kNormGated) {
    if (a.gamma_dtype != x_dtype || a.scale_dtype != x_dtype || a.shift_dtype != x_dtype ||
        (a.gate && a.gate_dtype != x_dtype))
      return false;
    if (out == OUT_F32) return false;
  }
  if (mode == kRms && out != OUT_INT8) return false;
  return true;
}

template <typename T, int B, int OUT, int MODE, int MAXT>
cudaError_t launch_k(const RowPrepArgs& a, cudaStream_t stream) {
  auto kern = rows16_kernel<T, B, OUT, MODE, MAXT>;
  const int tpr = static_cast<int>(a.K / 16);
  const int threads = (tpr + 31) & ~31;
  int slots = 0;
  if (MODE == kNorm || MODE == kNormGated) slots = 8;
  if (MODE == kRms) slots = 4;
  const int smem = slots * threads * 16;
  static std::atomic<long long> shape[kMaxLaunchDevices];
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e = launch_shape(reinterpret_cast<const void*>(kern), threads, smem, shape, &dev,
                               &sms, &per_sm);
  if (e != cudaSuccess) return e;
  int64_t grid = int64_t(sms) * per_sm;
  if (grid > a.rows) grid = a.rows;
  kern<<<static_cast<unsigned>(grid), threads, smem, stream>>>(a, smem);
  return cudaGetLastError();
}

template <typename T, int B, int OUT, int MODE>
cudaError_t launch_t(const RowPrepArgs& a, cudaStream_t stream) {
  return launch_k<T, B, OUT, MODE, 512>(a, stream);
}

template <typename T, int OUT, int MODE>
cudaError_t launch_b(const RowPrepArgs& a, int block, cudaStream_t stream) {
  switch (block) {
    case 0: return launch_t<T, 0, OUT, MODE>(a, stream);
    case 32: return launch_t<T, 32, OUT, MODE>(a, stream);
    case 64: return launch_t<T, 64, OUT, MODE>(a, stream);
    case 128: return launch_t<T, 128, OUT, MODE>(a, stream);
    case 256: return launch_t<T, 256, OUT, MODE>(a, stream);
    case 512: return launch_t<T, 512, OUT, MODE>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T, int MODE>
cudaError_t launch_o(const RowPrepArgs& a, int block, int out, cudaStream_t stream) {
  switch (out) {
    case OUT_INT8: return launch_b<T, OUT_INT8, MODE>(a, block, stream);
    case OUT_E4M3:
      if constexpr (MODE != kRms) return launch_b<T, OUT_E4M3, MODE>(a, block, stream);
      return cudaErrorInvalidValue;
    case OUT_F32:
      if constexpr (MODE == kPlain) return launch_b<T, OUT_F32, MODE>(a, block, stream);
      return cudaErrorInvalidValue;
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t launch(const RowPrepArgs& a, int block, int out, cudaStream_t stream) {
  switch (mode_of(a)) {
    case kPlain: return launch_o<T, kPlain>(a, block, out, stream);
    case kNorm: return launch_o<T, kNorm>(a, block, out, stream);
    case kNormGated: return launch_o<T, kNormGated>(a, block, out, stream);
    case kRms: return launch_o<T, kRms>(a, block, out, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace rows16
}  // namespace m5b
