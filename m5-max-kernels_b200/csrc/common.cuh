// Shared device helpers for the m5b200 sm_100a kernels.
//
// Everything here is plain CUDA / inline PTX for Blackwell (sm_100a):
//   * exact-rounding scalar helpers (bf16/fp16 round trips, RNE int8, E4M3),
//   * mbarrier / TMA / tcgen05 wrappers used by the GEMM,
//   * bounded waits: every spin on an mbarrier gives up after a wall-clock
//     limit, records an error code in the device status word and lets the
//     kernel unwind, so a broken pipeline ends with an error instead of a hang.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace m5b {

// ---------------------------------------------------------------------------
// Element types understood by the row kernels (values match include/m5b200.h)
// ---------------------------------------------------------------------------
enum DType : int { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2, DT_I8 = 3, DT_U8 = 4, DT_I32 = 5 };

template <typename T> struct DTypeOf;
template <> struct DTypeOf<float> { static constexpr int value = DT_F32; };
template <> struct DTypeOf<__half> { static constexpr int value = DT_F16; };
template <> struct DTypeOf<__nv_bfloat16> { static constexpr int value = DT_BF16; };

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Round an FP32 value through T with round-to-nearest-even and back.
template <typename T> __device__ __forceinline__ float round_through(float v) {
  return to_f32(from_f32<T>(v));
}

// Load one element of a small parameter table whose dtype is only known at
// run time (gamma / scale / shift / gate may be bf16, fp16 or fp32).
__device__ __forceinline__ float load_param(const void* base, int dtype, int64_t i) {
  switch (dtype) {
    case DT_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
    case DT_F16: return __half2float(reinterpret_cast<const __half*>(base)[i]);
    default: return reinterpret_cast<const float*>(base)[i];
  }
}

// Symmetric INT8 code: clip(rint(v / scale), -127, 127) with IEEE division.
__device__ __forceinline__ int8_t int8_code(float v, float scale) {
  float z = rintf(__fdiv_rn(v, scale));
  z = fminf(fmaxf(z, -127.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(z));
}

// rint(RN(x / s)) for a value whose reciprocal product t = RN(x * RN(1/s))
// lies within 2^-14 of the half-integer h next to r = RNE(t).  Division-free:
//   e = RN(x - h*s) (one FMA) has the exact sign of x/s - h and is zero iff
//   x/s == h; RN(x/s) == h exactly when |x - h*s| < s * ulp(h)/2, and RN(x/s)
//   lies past h (on e's side) when it is larger.  Only |e| == s*ulp(h)/2,
//   where e's own rounding hides which case holds, falls back to an IEEE
//   division.  Requires s >= 2^-100 and |x| <= 127.0001 * s.
__device__ __forceinline__ float int8_code_near_tie(float x, float s, float t, float r) {
  const float h = __fadd_rn(r, copysignf(0.5f, __fsub_rn(t, r)));
  const float e = __fmaf_rn(-h, s, x);
  const uint32_t biased = (__float_as_uint(h) >> 23) & 0xFFu;  // |h| >= 0.5
  const float half_ulp_s = __fmul_rn(s, __uint_as_float((biased - 24u) << 23));
  const float ae = fabsf(e);
  float q;
  if (ae < half_ulp_s)
    q = __fsub_rn(__fadd_rn(h, 12582912.0f), 12582912.0f);  // RN(x/s) == h: ties to even
  else if (ae > half_ulp_s)
    q = __fadd_rn(h, copysignf(0.5f, e));
  else
    q = rintf(__fdiv_rn(x, s));
  return fminf(fmaxf(q, -127.0f), 127.0f);
}

// INT8 codes of packed pairs from the correctly rounded quotient, without a
// division: with y = RN(1/s), q = RN(x y) and the residual r = x - q s (exact
// in one FMA), RN(q + r y) is RN(x / s) -- Markstein's correction step
// (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Develop. 34(1), 1990), which holds when
// no intermediate underflows.  With s >= kI8DivMinScale every intermediate is
// a normal number for |x| >= s/4, the only values whose code can be nonzero;
// below that the result is within a few ulps of x/s and rounds to 0 like it.
// Adding 1.5*2^23 then rounds to the nearest integer, ties to even (rint), and
// the low byte of the sum is the two's-complement int8 code; |x| <= 127.0001 s
// keeps it inside +-127, so no clip is needed.  Branch-free: every element
// costs the same four packed operations per pair.
constexpr float kI8DivMinScale = 0x1p-90f;
struct I8Div {
  float2 y, ns;  // RN(1/s), -s
};
__device__ __forceinline__ I8Div i8_div(float inv, float scale) {
  return I8Div{make_float2(inv, inv), make_float2(-scale, -scale)};
}
// RN(x / s) of a packed pair (the corrected quotient itself): exact wherever
// |x / s| >= 2^-12 and s >= kI8DivMinScale (the RMS folding's codes,
// prep_impl.cuh, use it there).  The sign of a zero quotient is not kept.
__device__ __forceinline__ float2 quot_pair_div(float2 x, const I8Div& d) {
  const float2 q = __fmul2_rn(x, d.y);
  const float2 r = __ffma2_rn(q, d.ns, x);  // x - q s, exact
  return __ffma2_rn(r, d.y, q);             // RN(x / s)
}
__device__ __forceinline__ float2 i8_pair_div(float2 x, const I8Div& d) {
  return __fadd2_rn(quot_pair_div(x, d), make_float2(12582912.0f, 12582912.0f));
}

// Four int8 codes (low bytes of a, b, c, d) packed into one word.
__device__ __forceinline__ uint32_t pack4_low_bytes(float a, float b, float c, float d) {
  return __byte_perm(__byte_perm(__float_as_uint(a), __float_as_uint(b), 0x0040),
                     __byte_perm(__float_as_uint(c), __float_as_uint(d), 0x0040), 0x5410);
}

// max(|a|, |b|) lane-wise on packed 16-bit floats, one instruction; the sign
// bit of the result is garbage (the xor of the inputs' signs).
__device__ __forceinline__ uint32_t max_xorsign_abs_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t max_xorsign_abs_f16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.xorsign.abs.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Exact E4M3 codes of four values (divide, then convert); out of line: it
// runs only for words whose brackets disagree (a product within 2^-18 of a
// rounding boundary) and for scales below 2^-100.
static __device__ __noinline__ uint32_t e4m3_word_exact(float a, float b, float c, float d,
                                                        float scale) {
  return __nv_cvt_float2_to_fp8x2(make_float2(__fdiv_rn(a, scale), __fdiv_rn(b, scale)),
                                  __NV_SATFINITE, __NV_E4M3) |
         (static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(
              make_float2(__fdiv_rn(c, scale), __fdiv_rn(d, scale)), __NV_SATFINITE, __NV_E4M3))
          << 16);
}

// OCP E4M3 codes (round to nearest even, saturated to +-448) of x / scale for
// NW words of 4 values (v[4w .. 4w+3] -> bytes 0..3 of word w), with the
// paired conversion.  Exactness: with a power-of-two scale (exact
// reciprocal) v * inv is the quotient itself and is converted once;
// otherwise v * inv * (1 -+ 2^-18) bracket RN(v / scale) and the conversion
// is monotone, so a word whose lower and upper bracket codes agree has those
// codes.  The words whose brackets disagree are collected in one mask and
// only those are divided exactly (one rarely taken branch per NW words).
// `fast` is false for scales below 2^-100 (every value divided exactly).
template <int NW>
__device__ __forceinline__ void e4m3_words(const float* v, float scale, float inv, bool fast,
                                           uint32_t* words) {
  if (!fast) {
#pragma unroll
    for (int w = 0; w < NW; ++w)
      words[w] = e4m3_word_exact(v[4 * w], v[4 * w + 1], v[4 * w + 2], v[4 * w + 3], scale);
    return;
  }
  const float2 inv2 = make_float2(inv, inv);
  if ((__float_as_uint(scale) & 0x007FFFFFu) == 0u) {  // exact reciprocal
#pragma unroll
    for (int w = 0; w < NW; ++w)
      words[w] = __nv_cvt_float2_to_fp8x2(__fmul2_rn(make_float2(v[4 * w], v[4 * w + 1]), inv2),
                                          __NV_SATFINITE, __NV_E4M3) |
                 (static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(
                      __fmul2_rn(make_float2(v[4 * w + 2], v[4 * w + 3]), inv2), __NV_SATFINITE,
                      __NV_E4M3))
                  << 16);
    return;
  }
  const float2 dn = make_float2(1.0f - 0x1p-18f, 1.0f - 0x1p-18f);
  const float2 up = make_float2(1.0f + 0x1p-18f, 1.0f + 0x1p-18f);
  uint32_t bad = 0u;
#pragma unroll
  for (int w = 0; w < NW; ++w) {
    const float2 t0 = __fmul2_rn(make_float2(v[4 * w], v[4 * w + 1]), inv2);
    const float2 t1 = __fmul2_rn(make_float2(v[4 * w + 2], v[4 * w + 3]), inv2);
    const uint32_t lo = __nv_cvt_float2_to_fp8x2(__fmul2_rn(t0, dn), __NV_SATFINITE, __NV_E4M3) |
                        (static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(
                             __fmul2_rn(t1, dn), __NV_SATFINITE, __NV_E4M3))
                         << 16);
    const uint32_t hi = __nv_cvt_float2_to_fp8x2(__fmul2_rn(t0, up), __NV_SATFINITE, __NV_E4M3) |
                        (static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(
                             __fmul2_rn(t1, up), __NV_SATFINITE, __NV_E4M3))
                         << 16);
    words[w] = lo;
    bad |= (lo != hi ? 1u : 0u) << w;
  }
  if (bad != 0u) {
#pragma unroll
    for (int w = 0; w < NW; ++w)
      if ((bad >> w) & 1u)
        words[w] = e4m3_word_exact(v[4 * w], v[4 * w + 1], v[4 * w + 2], v[4 * w + 3], scale);
  }
}

// Q/K post-processing on packed pairs (GEMM epilogue and the staged kernel).
// A packed bf16 pair as two floats (exact).
__device__ __forceinline__ float2 bf16x2_f2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}
__device__ __forceinline__ uint32_t f2_bf16x2(float2 v) {
  const __nv_bfloat162 h = __float22bfloat162_rn(v);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t u4w(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Split-half RoPE of one 16-byte chunk pair; the same IEEE operations per
// element as the scalar form:
//   ul = (zl * inv) * gl, uh = (zh * inv) * gh      (packed pairs)
//   zl' = bf16(ul * c - uh * s), zh' = bf16(uh * c + ul * s)   (scalar)
// Packed-pair products are used only where a product feeds another product:
// a packed multiply feeding a packed add was observed to be contracted into
// a fused multiply-add (one rounding instead of two), which the scalar
// __fmul_rn / __fadd_rn / __fsub_rn intrinsics never are.
__device__ __forceinline__ void rope_chunk16(uint4& zl, uint4& zh, const uint4& gl,
                                             const uint4& gh, const uint4& c8, const uint4& s8,
                                             float inv) {
  const float2 inv2 = make_float2(inv, inv);
  uint32_t ol[4], oh[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float2 ul = __fmul2_rn(__fmul2_rn(bf16x2_f2(u4w(zl, p)), inv2), bf16x2_f2(u4w(gl, p)));
    const float2 uh = __fmul2_rn(__fmul2_rn(bf16x2_f2(u4w(zh, p)), inv2), bf16x2_f2(u4w(gh, p)));
    const float2 c = bf16x2_f2(u4w(c8, p));
    const float2 sv = bf16x2_f2(u4w(s8, p));
    const float2 lo = make_float2(__fsub_rn(__fmul_rn(ul.x, c.x), __fmul_rn(uh.x, sv.x)),
                                  __fsub_rn(__fmul_rn(ul.y, c.y), __fmul_rn(uh.y, sv.y)));
    const float2 hi = make_float2(__fadd_rn(__fmul_rn(uh.x, c.x), __fmul_rn(ul.x, sv.x)),
                                  __fadd_rn(__fmul_rn(uh.y, c.y), __fmul_rn(ul.y, sv.y)));
    ol[p] = f2_bf16x2(lo);
    oh[p] = f2_bf16x2(hi);
  }
  zl = make_uint4(ol[0], ol[1], ol[2], ol[3]);
  zh = make_uint4(oh[0], oh[1], oh[2], oh[3]);
}
// Unrotated channels: bf16((z * inv) * g) on packed pairs.
__device__ __forceinline__ uint4 norm_chunk16(const uint4& z, const uint4& g8, float inv) {
  const float2 inv2 = make_float2(inv, inv);
  uint32_t o[4];
#pragma unroll
  for (int p = 0; p < 4; ++p)
    o[p] = f2_bf16x2(__fmul2_rn(__fmul2_rn(bf16x2_f2(u4w(z, p)), inv2), bf16x2_f2(u4w(g8, p))));
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// ---------------------------------------------------------------------------
// Device status word: error codes recorded by bounded waits.
// ---------------------------------------------------------------------------
enum DeviceError : unsigned int {
  DEV_OK = 0,
  DEV_TIMEOUT_PRODUCER = 1u << 0,
  DEV_TIMEOUT_MMA = 1u << 1,
  DEV_TIMEOUT_EPILOGUE = 1u << 2,
  DEV_TIMEOUT_DRAIN = 1u << 3,
  DEV_TIMEOUT_FIXUP = 1u << 4,  // split-K: the other pairs' partial stores did not finish
};

// Wall-clock limit for a single mbarrier wait (nanoseconds).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start before the previous kernel in the stream ends; it
// must execute grid_dependency_wait() before it reads anything that kernel
// wrote (or writes anything it reads).  grid_dependents_launch() lets the
// next such kernel start launching.  Both are no-ops without the attribute.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Shared-memory address helpers and mbarriers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of a barrier phase (no suspend window): true when the
// phase with the given parity has completed.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records `code` in *status) when the
// barrier phase did not complete within kWaitLimitNs, or when another role of
// the same CTA already aborted (*abort != 0).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort, unsigned int* status,
                                                  unsigned int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 255u) == 0u) {
      if (*abort) return false;
      if (globaltimer_ns() - start > kWaitLimitNs) {
        if (status) atomicOr(status, code);
        *abort = 1;
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (non-multicast tiled loads only)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Tiled TMA load of a 3D box into shared memory, completion on an mbarrier.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Tiled TMA store of a 3D box from shared memory (bulk-group completion).
// Out-of-range coordinates of the box are clipped by the tensor map.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src,
                                             int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// Tiled TMA store of a 2D box from shared memory (bulk-group completion).
// Out-of-range parts of the box are clipped by the tensor map.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src,
                                             int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y)
      : "memory");
}
// An L2 cache policy that makes the lines it touches the first to be evicted
// (streaming data: written once and not read again soon).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}
// tma_store_2d with an L2 cache policy (e.g. evict-first for outputs that
// the next kernel does not read, so they leave L2 while DRAM has headroom).
__device__ __forceinline__ void tma_store_2d_hint(const CUtensorMap* map, const void* smem_src,
                                                  int32_t x, int32_t y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint"
      " [%0, {%2, %3}], [%1], %4;" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// The shared memory read by this thread's committed bulk stores may be reused.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// All but the most recent of this thread's committed bulk store groups have
// read their shared memory.
__device__ __forceinline__ void bulk_wait_group_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
// This thread's committed bulk stores are complete.
__device__ __forceinline__ void bulk_wait_group0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Generic-proxy shared-memory writes become visible to the async proxy (TMA).
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Bulk prefetch of [src, src + bytes) from global memory into L2 (no
// destination, no completion to wait for).  src 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void prefetch_l2_bulk(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, TMEM accumulators)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread
// has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Shared-memory matrix descriptor for a K-major tile stored as rows of 128
// bytes with the 128-byte swizzle (the layout TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B).  Stride between 8-row groups is 1024 bytes.
__device__ __forceinline__ uint64_t smem_desc_k128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);   // start address
  d |= static_cast<uint64_t>(1u) << 16;                      // leading byte offset (unused)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;              // stride byte offset
  d |= static_cast<uint64_t>(1u) << 46;                      // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;                      // SWIZZLE_128B
  return d;
}

// MMA kinds used by the GEMM.
enum MmaKind : int { KIND_I8 = 0, KIND_F8 = 1, KIND_BF16 = 2, KIND_F16 = 3, KIND_TF32 = 4 };

// Instruction descriptor: K-major A and B, dense, M x N (M = 128, or 256 for
// a CTA pair).
__host__ __device__ constexpr uint32_t make_idesc(int kind, int m, int n) {
  // c_format: 1 = F32, 2 = S32; a/b format: S8 -> 1, E4M3 -> 0, BF16 -> 1, F16 -> 0,
  // TF32 -> 2 (kind::tf32)
  uint32_t c_fmt = (kind == KIND_I8) ? 2u : 1u;
  uint32_t ab_fmt = kind == KIND_TF32 ? 2u : (kind == KIND_I8 || kind == KIND_BF16) ? 1u : 0u;
  return (c_fmt << 4) | (ab_fmt << 7) | (ab_fmt << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

template <int KIND>
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  if constexpr (KIND == KIND_I8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (KIND == KIND_F8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (KIND == KIND_TF32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// Load 32 consecutive 32-bit TMEM columns of this warp's 32 lanes: thread i of
// the warp receives lane (base_lane + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// Store 32 consecutive 32-bit TMEM columns of this warp's 32 lanes (thread i
// writes lane base_lane + i, columns [col, col + 32)).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Untiled bulk copies (TMA engine): global -> this CTA's shared memory with
// completion on an mbarrier, and shared -> global in the bulk-group scheme.
// Addresses 16-byte aligned, sizes multiples of 16.
__device__ __forceinline__ void bulk_load_g2s(void* smem_dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void bulk_store_s2g(void* dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                   reinterpret_cast<uint64_t>(dst)),
               "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
}
// Generic-proxy global accesses and async-proxy (TMA) accesses are ordered.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (cluster of 2) for cta_group::2 tensor-core MMAs
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// Shared::cluster address of `p` (a variable of this CTA) in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// TMA tile load issued by either CTA of a pair; the transaction bytes are
// counted on the barrier of the pair's even CTA (peer bit of the address
// cleared).  No multicast: each CTA loads its own half of the operands.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map,
                                                 uint64_t* bar, int32_t x, int32_t y) {
  const uint32_t bar_leader = smem_u32(bar) & 0xFEFFFFFFu;
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_leader), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// Arrive on `bar` in both CTAs of the pair once the MMAs issued so far retire;
// `pair_mask` names the pair's two CTAs in the cluster (0b11 << even rank).
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t pair_mask = 3) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(pair_mask)
      : "memory");
}
// Bulk copy of `bytes` (a multiple of 16, 16-byte aligned) from this CTA's
// shared memory into another CTA's of the cluster (cluster address from
// map_to_rank), completing the transaction bytes on that CTA's mbarrier.
__device__ __forceinline__ void bulk_copy_s2cluster(uint32_t dst_cluster, const void* src,
                                                    uint32_t bytes, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(dst_cluster), "r"(smem_u32(src)), "r"(bytes), "r"(bar_cluster)
      : "memory");
}

template <int KIND>
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  if constexpr (KIND == KIND_I8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (KIND == KIND_F8) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (KIND == KIND_TF32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

__device__ __forceinline__ uint32_t elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t.reg .b32 r;\n\t"
      "elect.sync r|P, %1;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(pred)
      : "r"(0xffffffffu));
  return pred;
}

}  // namespace m5b
