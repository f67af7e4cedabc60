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
//   * a thread's 16 elements are one chunk of the canonical reduction tree
//     (chunk16_sum); lanes continue the pairwise tree over chunk index with a
//     xor butterfly, and the warps' partials combine pairwise (padded to 16).
//     LayerNorm keeps the centered values x - mean of its second pass for the
//     normalization, and divides by K as a multiply when K is a power of two
//     (the same correctly rounded quotient).
//   * Hadamard strides 1-8 are register butterflies on packed pairs, strides
//     16-512 shuffles (lane xor 1, 2, 4, 8, 16), so B <= 512.
//   * modulation / gate / gamma slices are per-thread data (a thread always
//     handles the same 16 columns); they are kept in shared memory in a
//     conflict-free per-thread layout (the modulation's 1 + scale and shift
//     as fp32, ready to use) and reloaded only when the row's table index
//     changes.
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

// The two 16-bit values of a word of T, as floats.
template <typename T>
__device__ __forceinline__ float2 word_pair(uint32_t x) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    return make_float2(__uint_as_float(x << 16), __uint_as_float(x & 0xFFFF0000u));
  else
    return __half22float2(*reinterpret_cast<const __half2*>(&x));
}

// a * b + c for the two 16-bit values of the words a and b (lane-wise), with
// fp32 c: sm_100's mixed-precision FMA, one rounding -- the same value as
// fmaf(float(a), float(b), c) -- without unpacking a and b first.
template <typename T>
__device__ __forceinline__ float2 fma_words16(uint32_t a, uint32_t b, float2 c) {
  float2 d;
  if constexpr (std::is_same<T, __nv_bfloat16>::value)
    asm("{\n.reg .b16 al, ah, bl, bh;\nmov.b32 {al, ah}, %2;\nmov.b32 {bl, bh}, %3;\n"
        "fma.rn.f32.bf16 %0, al, bl, %4;\nfma.rn.f32.bf16 %1, ah, bh, %5;\n}"
        : "=f"(d.x), "=f"(d.y) : "r"(a), "r"(b), "f"(c.x), "f"(c.y));
  else
    asm("{\n.reg .b16 al, ah, bl, bh;\nmov.b32 {al, ah}, %2;\nmov.b32 {bl, bh}, %3;\n"
        "fma.rn.f32.f16 %0, al, bl, %4;\nfma.rn.f32.f16 %1, ah, bh, %5;\n}"
        : "=f"(d.x), "=f"(d.y) : "r"(a), "r"(b), "f"(c.x), "f"(c.y));
  return d;
}

// Pair k (elements 2k, 2k+1) of a Raw16 of T, as floats.
template <typename T>
__device__ __forceinline__ float2 pair_of(const Raw16& r, int k) {
  const uint4& w = k < 4 ? r.lo : r.hi;
  const int i = k & 3;
  return word_pair<T>(i == 0 ? w.x : i == 1 ? w.y : i == 2 ? w.z : w.w);
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
// Row total of the threads' chunk sums in the canonical tree: lanes xor 1..16
// (a pairwise tree over chunk index), one float per warp in `part` (this
// reduction's own buffer), one CTA barrier, then the warps pairwise (zero
// padded to 16) by a xor butterfly over lanes 0-15; the total is added to +0.
__device__ __forceinline__ float warps_pairwise16(const float* part, int lane, int nwarps) {
  float o = (lane & 15) < nwarps ? part[lane & 15] : 0.0f;
#pragma unroll
  for (int off = 1; off < 16; off <<= 1) o = __fadd_rn(o, __shfl_xor_sync(kFull, o, off));
  return __fadd_rn(o, 0.0f);
}

__device__ __forceinline__ float row_total(float c, float* part, int warp, int lane, int nwarps) {
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) c = __fadd_rn(c, __shfl_xor_sync(kFull, c, off));
  if (lane == 0) part[warp] = c;
  __syncthreads();
  return warps_pairwise16(part, lane, nwarps);
}

// x / K, correctly rounded: a multiply by the exact reciprocal when K is a
// power of two.
__device__ __forceinline__ float div_k(float x, float kf, float rk, bool pow2) {
  return pow2 ? __fmul_rn(x, rk) : __fdiv_rn(x, kf);
}

// Maximum of a non-negative float over the warp (one redux instruction).
__device__ __forceinline__ float warp_max(float m) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(m));
  return r;
}

__device__ __forceinline__ float row_max(float m, float* part, int warp, int lane, int nwarps) {
  m = warp_max(m);
  if (lane == 0) part[warp] = m;
  __syncthreads();
  // every warp reduces the same partials (nwarps <= 16: rows of <= 8192)
  return warp_max((lane & 15) < nwarps ? part[lane & 15] : 0.0f);
}

// Sum (canonical) and max with one barrier (RMS scale folding).
__device__ __forceinline__ float2 row_total_max(float c, float m, float* part, float* part_max,
                                                int warp, int lane, int nwarps) {
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) c = __fadd_rn(c, __shfl_xor_sync(kFull, c, off));
  m = warp_max(m);
  if (lane == 0) {
    part[warp] = c;
    part_max[warp] = m;
  }
  __syncthreads();
  const float total = warps_pairwise16(part, lane, nwarps);
  return make_float2(total, warp_max((lane & 15) < nwarps ? part_max[lane & 15] : 0.0f));
}

// ---------------------------------------------------------------- transforms
// Sign bit (0x80000000 or 0) of element e of the thread's 16 columns, from
// their 16 sign bytes (+-1) read as four words.
__device__ __forceinline__ uint32_t sign_bit(const uint32_t* sw, int e) {
  return (sw[e >> 2] << (24 - 8 * (e & 3))) & 0x80000000u;
}
__device__ __forceinline__ void sign_words(const int8_t* sg, uint32_t* sw) {
  const uint4 s4 = __ldg(reinterpret_cast<const uint4*>(sg));
  sw[0] = s4.x;
  sw[1] = s4.y;
  sw[2] = s4.z;
  sw[3] = s4.w;
}
__device__ __forceinline__ float flip(float x, uint32_t bit) {
  return __uint_as_float(__float_as_uint(x) ^ bit);
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
// Registers: 64 a thread (four 256-thread or two 512-thread CTAs per SM),
// except the gated form on rows of <= 4096 (MAXT = 256), which keeps the next
// row's branch and input words in flight beside its tables: capped at 80 it
// runs spill-free at three CTAs per SM, measured 40.1 against 45.2 us (64
// registers and 32 bytes of spills) on C4's M4096 K4096 prep.
template <typename T, int B, int OUT, int MODE, int MAXT>
__global__ void __launch_bounds__(MAXT) __maxnreg__(MODE == kNormGated && MAXT == 256 ? 80 : 64)
    rows16_kernel(const RowPrepArgs a, const int tbl_bytes) {
  extern __shared__ __align__(16) uint8_t tbl[];  // per-thread table slots
  __shared__ float red[2][4][MAXT / 32];           // [row parity][reduction][warp]
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nthreads = blockDim.x;
  const int nwarps = nthreads >> 5;
  const int64_t K = a.K;
  const int tpr = static_cast<int>(K >> 4);
  const bool have = tid < tpr;
  const int j0 = (have ? tid : 0) * 16;  // first column of this thread
  const float kf = static_cast<float>(K);
  const bool k_pow2 = (K & (K - 1)) == 0;
  const float rk = k_pow2 ? 1.0f / kf : 0.0f;  // exact when K is a power of two

  // Table slots: gated: gate [0,2), norm: gamma [2,4), s * (1 + scale) (fp32)
  // [4,8), s * shift (fp32) [8,12); RMS: s * gamma (fp32) [0,4); plain: the
  // packed sign masks [0,2) (s: the Hadamard signs of the thread's columns).
  uint8_t* tb = tbl;
  int cur_gmap = -1, cur_map = -1;  // table rows now in shared memory (maps are int32)
  (void)tbl_bytes;
  if constexpr (MODE == kNorm || MODE == kNormGated) {
    if (have) {  // gamma once (shared by all rows)
      const Raw16 g = ld_raw(reinterpret_cast<const T*>(a.gamma) + j0);
      *tslot(tb, nthreads, tid, 2) = g.lo;
      *tslot(tb, nthreads, tid, 3) = g.hi;
    }
  } else if constexpr (MODE == kRms) {
    if (have) {  // gamma (fp32) with the Hadamard signs folded in: s * (t * g) = t * (s * g)
      uint32_t sw[4] = {0u, 0u, 0u, 0u};
      if (a.signs != nullptr) sign_words(a.signs + j0, sw);
      const uint4* gp = reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(a.gamma) + j0);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const uint4 w = __ldg(gp + h);
        *tslot(tb, nthreads, tid, h) =
            make_uint4(w.x ^ sign_bit(sw, 4 * h), w.y ^ sign_bit(sw, 4 * h + 1),
                       w.z ^ sign_bit(sw, 4 * h + 2), w.w ^ sign_bit(sw, 4 * h + 3));
      }
    }
  } else {
    if (have && a.signs != nullptr) {  // sign masks of the packed 16-bit pairs
      uint32_t sw[4];
      sign_words(a.signs + j0, sw);
      uint32_t mk[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mk[k] = (sign_bit(sw, 2 * k) >> 16) | sign_bit(sw, 2 * k + 1);
      *tslot(tb, nthreads, tid, 0) = make_uint4(mk[0], mk[1], mk[2], mk[3]);
      *tslot(tb, nthreads, tid, 1) = make_uint4(mk[4], mk[5], mk[6], mk[7]);
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
    if constexpr (MODE == kPlain) {
      if (have && a.signs != nullptr) {  // X D: sign flips on the packed input
        const uint4 m0 = *tslot(tb, nthreads, tid, 0), m1 = *tslot(tb, nthreads, tid, 1);
        Raw16 sx;
        sx.lo = make_uint4(cx.lo.x ^ m0.x, cx.lo.y ^ m0.y, cx.lo.z ^ m0.z, cx.lo.w ^ m0.w);
        sx.hi = make_uint4(cx.hi.x ^ m1.x, cx.hi.y ^ m1.y, cx.hi.z ^ m1.z, cx.hi.w ^ m1.w);
        unpack16<T>(sx, v);
      } else {
        unpack16<T>(cx, v);  // zeros past the row (cx is zero there)
      }
    } else {
      unpack16<T>(cx, v);  // zeros past the row (cx is zero there)
    }

    if constexpr (MODE == kNormGated) {
      // R' = cast_T(R + branch * gate), written once.
      if (have) {
        const int gm = a.gate_row_map ? __ldg(a.gate_row_map + row) : 0;
        if (gm != cur_gmap) {
          const Raw16 g = ld_raw(reinterpret_cast<const T*>(a.gate) + int64_t(gm) * K + j0);
          *tslot(tb, nthreads, tid, 0) = g.lo;
          *tslot(tb, nthreads, tid, 1) = g.hi;
          cur_gmap = gm;
        }
        // one 16-byte half at a time; each R' word is converted once, stored
        // and unpacked again for the normalization
        uint4* rdst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.r_out) + row * K + j0);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const uint4 gw = *tslot(tb, nthreads, tid, half);
          const uint4 bw = half ? cb.hi : cb.lo;
          const uint32_t gv[4] = {gw.x, gw.y, gw.z, gw.w};
          const uint32_t bv[4] = {bw.x, bw.y, bw.z, bw.w};
          uint32_t rw[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int k = 4 * half + i;
            rw[i] = pack2<T>(fma_words16<T>(bv[i], gv[i], v[k]));
            v[k] = word_pair<T>(rw[i]);
          }
          rdst[half] = make_uint4(rw[0], rw[1], rw[2], rw[3]);
        }
      }
    }

    float inv = 1.0f;      // RMS folding: the row's inverse RMS
    float sq_chunk = 0.0f;
    if constexpr (MODE == kNorm || MODE == kNormGated) {
      const bool layer = a.norm == NORM_LAYER;
      const float c0 = !have ? 0.0f : layer ? chunk16_sum<false>(v) : chunk16_sum<true>(v);
      const float first = div_k(row_total(c0, rs, warp, lane, nwarps), kf, rk, k_pow2);
      float moment = first;
      if (layer) {
        // centered values, kept for the normalization: (x - mean) is the
        // same rounded difference in both places
        const float2 nm = f2(-first);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = __fadd2_rn(v[k], nm);
        moment = div_k(row_total(have ? chunk16_sum<true>(v) : 0.0f, rv, warp, lane, nwarps), kf,
                       rk, k_pow2);
      }
      inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(moment, a.eps)));
      if (have) {
        const int mm = a.row_map ? __ldg(a.row_map + row) : 0;
        if (mm != cur_map) {
          // the modulation's 1 + scale (rounded once, as where it is used)
          // and shift, kept as fp32
          // The Hadamard signs are folded in as well: with s = +-1,
          // fma(t, s * o, s * sh) = s * fma(t, o, sh) and rounding to the
          // input dtype commutes with the sign, so the modulated, rounded,
          // sign-flipped value is the one computed in that order.
          // (one 16-byte half of the thread's columns at a time: few live
          // registers in this rarely taken branch)
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const uint4 scw =
                __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.scale) + int64_t(mm) * K + j0) + half);
            const uint4 shw =
                __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.shift) + int64_t(mm) * K + j0) + half);
            const uint2 sgw = a.signs != nullptr
                                  ? __ldg(reinterpret_cast<const uint2*>(a.signs + j0) + half)
                                  : make_uint2(0u, 0u);
            const uint32_t scv[4] = {scw.x, scw.y, scw.z, scw.w};
            const uint32_t shv[4] = {shw.x, shw.y, shw.z, shw.w};
            const uint32_t sgv[2] = {sgw.x, sgw.y};
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const float2 o0 = __fadd2_rn(f2(1.0f), word_pair<T>(scv[2 * hh]));
              const float2 o1 = __fadd2_rn(f2(1.0f), word_pair<T>(scv[2 * hh + 1]));
              const float2 s0 = word_pair<T>(shv[2 * hh]), s1 = word_pair<T>(shv[2 * hh + 1]);
              const uint32_t b0 = sign_bit(sgv + hh, 0), b1 = sign_bit(sgv + hh, 1);
              const uint32_t b2 = sign_bit(sgv + hh, 2), b3 = sign_bit(sgv + hh, 3);
              const int h = 2 * half + hh;
              *tslot(tb, nthreads, tid, 4 + h) =
                  make_uint4(__float_as_uint(o0.x) ^ b0, __float_as_uint(o0.y) ^ b1,
                             __float_as_uint(o1.x) ^ b2, __float_as_uint(o1.y) ^ b3);
              *tslot(tb, nthreads, tid, 8 + h) =
                  make_uint4(__float_as_uint(s0.x) ^ b0, __float_as_uint(s0.y) ^ b1,
                             __float_as_uint(s1.x) ^ b2, __float_as_uint(s1.y) ^ b3);
            }
          }
          cur_map = mm;
        }
        Raw16 g;
        g.lo = *tslot(tb, nthreads, tid, 2);
        g.hi = *tslot(tb, nthreads, tid, 3);
        const float2 inv2 = f2(inv);
#pragma unroll
        for (int h = 0; h < 4; ++h) {  // v holds x - mean (LayerNorm) or x (RMS)
          const uint4 ow = *tslot(tb, nthreads, tid, 4 + h);
          const uint4 sw = *tslot(tb, nthreads, tid, 8 + h);
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int k = 2 * h + e;
            const float2 ops = e == 0 ? make_float2(__uint_as_float(ow.x), __uint_as_float(ow.y))
                                      : make_float2(__uint_as_float(ow.z), __uint_as_float(ow.w));
            const float2 shf = e == 0 ? make_float2(__uint_as_float(sw.x), __uint_as_float(sw.y))
                                      : make_float2(__uint_as_float(sw.z), __uint_as_float(sw.w));
            const float2 t = __fmul2_rn(__fmul2_rn(v[k], inv2), pair_of<T>(g, k));
            float2 y = __ffma2_rn(t, ops, shf);
            if (a.round_output) y = round2<T>(y);
            v[k] = y;
          }
        }
      }
    } else if constexpr (MODE == kRms) {
      // statistics of the ORIGINAL row; direct form normalizes now, folded
      // form keeps the inverse RMS for the row scale
      sq_chunk = have ? chunk16_sum<true>(v) : 0.0f;
      if (a.rms_quant == RMSQ_DIRECT) {
        const float moment = div_k(row_total(sq_chunk, rs, warp, lane, nwarps), kf, rk, k_pow2);
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
    // (the signs D are already in: packed input flips, or folded into the tables)
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
          const float2 sm = row_total_max(sq_chunk, m, rs, rm, warp, lane, nwarps);
          const float moment = div_k(sm.x, kf, rk, k_pow2);
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
            e4m3_words<4>(vv, scale, rinv, fast, words);
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
  if (MODE == kNorm || MODE == kNormGated) slots = 12;
  if (MODE == kRms) slots = 4;
  if (MODE == kPlain) slots = 2;  // packed sign masks
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
  if constexpr (MODE == kNormGated)
    if (a.K <= 4096) return launch_k<T, B, OUT, MODE, 256>(a, stream);
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
