// Staged comparators: the stages the fused kernels combine, run on their own.
//
// The reference keeps standalone versions of two preparation stages and of the
// Q/K post-processing so that a fused kernel can be compared with the same
// arithmetic split over several launches (fusion-gain reporting and exact
// staged == fused checks):
//   * gated_residual_add   R' = cast_R(R + branch * gate[gate_row_map])
//       (src/m5kernels/norm_hadamard.py:280-300, shaders/gated_residual.metal)
//   * qk_norm_rope         bf16 projection [M, N] -> per-head RMSNorm * gamma ->
//       split-half RoPE -> bf16 head-major [N/128, M, 128]
//       (src/m5kernels/qk_rope.py:185-203, shaders/qk_rope_norm.metal)
// The third, unfused_norm (norm + modulation only), is the row-preparation
// kernel of prep_impl.cuh with its row output (OUT_ROW / OUT_F32, no rotation).
//
// Each kernel repeats the FP32 operations of its fused counterpart in the same
// order, so the staged pipeline's results are bit-identical to the fused ones:
//   gated update: one fused multiply-add fmaf(branch, gate, R), one RNE cast
//     (the update inside row_prep_kernel / lean_kernel);
//   Q/K: sequential fmaf square sum over the head's 128 channels in channel
//     order, inv = 1 / sqrt(sum / 128 + eps), u = (z * inv) * gamma, RoPE
//     v_j = u_j c - u_{j+R} s, v_{j+R} = u_{j+R} c + u_j s (the GEMM's Q/K
//     epilogue in gemm.cu).
//
// Both kernels are HBM-bound.  Algorithmic bytes: gated add 3 * K * sizeof(T)
// per row (R and branch read, R' written; the gate table stays in L2); Q/K
// 4 bytes per projection element (bf16 read and written) plus the cos / sin
// rows.
#include "common.cuh"
#include "m5b_internal.h"

namespace m5b {

namespace {

constexpr int kThreads = 256;

// Eight consecutive elements of a bf16 / fp16 / fp32 array (16-byte aligned,
// whole vector in bounds) as floats.
template <typename T>
__device__ __forceinline__ void ld8(const T* p, float* out) {
  if constexpr (sizeof(T) == 2) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
    const T* h = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] = to_f32(h[e]);
  } else {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
  }
}

__device__ __forceinline__ void ld8_param(const void* base, int dtype, int64_t j, float* out) {
  switch (dtype) {
    case DT_BF16: ld8(reinterpret_cast<const __nv_bfloat16*>(base) + j, out); break;
    case DT_F16: ld8(reinterpret_cast<const __half*>(base) + j, out); break;
    default: ld8(reinterpret_cast<const float*>(base) + j, out); break;
  }
}

template <typename T>
__device__ __forceinline__ void st8(T* p, const float* v) {
  if constexpr (sizeof(T) == 2) {
    uint4 raw;
    T* h = reinterpret_cast<T*>(&raw);
#pragma unroll
    for (int e = 0; e < 8; ++e) h[e] = from_f32<T>(v[e]);
    *reinterpret_cast<uint4*>(p) = raw;
  } else {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
}

// ---------------------------------------------------------------- gated add
// Rows are distributed over persistent CTAs; the CTA's threads stride over
// the row's 8-element vectors (VEC) or its elements.
template <typename T, bool VEC>
__global__ void __launch_bounds__(kThreads)
    gated_add_kernel(const T* __restrict__ res, const T* __restrict__ br, const void* gate,
                     int gate_dtype, const int32_t* __restrict__ gate_row_map, int64_t rows,
                     int64_t K, T* __restrict__ out) {
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t goff = gate_row_map ? int64_t(__ldg(gate_row_map + row)) * K : 0;
    const T* r = res + row * K;
    const T* b = br + row * K;
    T* o = out + row * K;
    if constexpr (VEC) {
      for (int64_t j = int64_t(threadIdx.x) * 8; j < K; j += int64_t(kThreads) * 8) {
        float rv[8], bv[8], gv[8], y[8];
        ld8(r + j, rv);
        ld8(b + j, bv);
        ld8_param(gate, gate_dtype, goff + j, gv);
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = __fmaf_rn(bv[e], gv[e], rv[e]);
        st8(o + j, y);
      }
    } else {
      for (int64_t j = threadIdx.x; j < K; j += kThreads) {
        const float g = load_param(gate, gate_dtype, goff + j);
        o[j] = from_f32<T>(__fmaf_rn(to_f32(b[j]), g, to_f32(r[j])));
      }
    }
  }
}

template <typename T>
cudaError_t launch_gated_add_t(const GatedAddArgs& a, cudaStream_t stream) {
  const bool vec = a.vec_ok != 0;
  const void* kern = vec ? reinterpret_cast<const void*>(gated_add_kernel<T, true>)
                         : reinterpret_cast<const void*>(gated_add_kernel<T, false>);
  static std::atomic<long long> shape[kMaxLaunchDevices];
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e = launch_shape(kern, kThreads, 0, shape, &dev, &sms, &per_sm);
  if (e != cudaSuccess) return e;
  int64_t grid = int64_t(sms) * per_sm;
  if (grid > a.rows) grid = a.rows;
  const T* r = reinterpret_cast<const T*>(a.residual);
  const T* b = reinterpret_cast<const T*>(a.branch);
  T* o = reinterpret_cast<T*>(a.out);
  if (vec)
    gated_add_kernel<T, true><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(
        r, b, a.gate, a.gate_dtype, a.gate_row_map, a.rows, a.K, o);
  else
    gated_add_kernel<T, false><<<static_cast<unsigned>(grid), kThreads, 0, stream>>>(
        r, b, a.gate, a.gate_dtype, a.gate_row_map, a.rows, a.K, o);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- Q/K norm + RoPE
// One warp per (block of 32 rows, head).  The warp loads the block's 32 x 128
// bf16 slice (coalesced, 512 bytes per instruction) into its 8 KB staging
// area -- two 64-channel halves of 32 rows x 128 bytes, 16-byte chunks
// XOR-swizzled by row, the layout of the fused epilogue -- then lane l
// processes row l: square sum, RMS, gamma and RoPE.  With R % 8 == 0 (FAST)
// the result is written back in place and leaves as one contiguous 8 KB block
// of the head-major output; any other R stores element groups directly.
constexpr int kQkThreads = 128;
constexpr int kQkWarps = kQkThreads / 32;  // 32 KB of static staging per CTA

__device__ __forceinline__ uint8_t* qk_chunk(uint8_t* stage, int row, int ch) {
  return stage + (ch >> 3) * 4096 + row * 128 + (((ch & 7) ^ (row & 7)) << 4);
}

template <bool FAST>
__global__ void __launch_bounds__(kQkThreads)
    qk_norm_rope_kernel(const __nv_bfloat16* __restrict__ p, int64_t M, int64_t N,
                        const __nv_bfloat16* __restrict__ gamma, const __nv_bfloat16* __restrict__ cos,
                        const __nv_bfloat16* __restrict__ sin, int R, float eps,
                        __nv_bfloat16* __restrict__ out) {
  __shared__ __align__(128) uint8_t stage_all[kQkWarps][8192];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* stage = stage_all[warp];
  const int64_t heads = N / 128;
  const int64_t row_blocks = (M + 31) / 32;
  const int64_t items = row_blocks * heads;
  for (int64_t item = int64_t(blockIdx.x) * kQkWarps + warp; item < items;
       item += int64_t(gridDim.x) * kQkWarps) {
    const int64_t rb = item / heads;
    const int64_t head = item - rb * heads;
    const int64_t row0 = rb * 32;
    // ---- load the 32 x 128 slice: lane -> (row 2i + lane/16, chunk lane%16)
#pragma unroll 4
    for (int i = 0; i < 16; ++i) {
      const int r = 2 * i + (lane >> 4), c = lane & 15;
      const int64_t row = row0 + r;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (row < M) v = __ldg(reinterpret_cast<const uint4*>(p + row * N + head * 128 + c * 8));
      *reinterpret_cast<uint4*>(qk_chunk(stage, r, c)) = v;
    }
    __syncwarp();
    const int64_t row = row0 + lane;
    // ---- square sum in channel order
    float sumsq = 0.0f;
#pragma unroll 1
    for (int c = 0; c < 16; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(qk_chunk(stage, lane, c));
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float f = __bfloat162float(h[e]);
        sumsq = __fmaf_rn(f, f, sumsq);
      }
    }
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sumsq, 128.0f), eps)));
    if constexpr (FAST) {
      if (row < M) {
        const int RC = R >> 3;
        const uint4* cs4 = reinterpret_cast<const uint4*>(cos + row * R);
        const uint4* sn4 = reinterpret_cast<const uint4*>(sin + row * R);
        const uint4* gm4 = reinterpret_cast<const uint4*>(gamma);
#pragma unroll 1
        for (int q = 0; q < RC; ++q) {
          uint4 zl = *reinterpret_cast<const uint4*>(qk_chunk(stage, lane, q));
          uint4 zh = *reinterpret_cast<const uint4*>(qk_chunk(stage, lane, q + RC));
          rope_chunk16(zl, zh, __ldg(gm4 + q), __ldg(gm4 + q + RC), __ldg(cs4 + q),
                       __ldg(sn4 + q), inv);
          *reinterpret_cast<uint4*>(qk_chunk(stage, lane, q)) = zl;
          *reinterpret_cast<uint4*>(qk_chunk(stage, lane, q + RC)) = zh;
        }
#pragma unroll 1
        for (int q = 2 * RC; q < 16; ++q)
          *reinterpret_cast<uint4*>(qk_chunk(stage, lane, q)) =
              norm_chunk16(*reinterpret_cast<const uint4*>(qk_chunk(stage, lane, q)),
                           __ldg(gm4 + q), inv);
      }
      __syncwarp();
      // ---- the finished block: rows row0.. of head `head`, contiguous
      __nv_bfloat16* dst = out + (head * M + row0) * 128;
#pragma unroll 4
      for (int i = 0; i < 16; ++i) {
        const int r = 2 * i + (lane >> 4), c = lane & 15;
        if (row0 + r < M)
          *reinterpret_cast<uint4*>(dst + r * 128 + c * 8) =
              *reinterpret_cast<const uint4*>(qk_chunk(stage, r, c));
      }
    } else if (row < M) {
      auto zat = [&](int j) -> float {
        return __bfloat162float(
            *reinterpret_cast<const __nv_bfloat16*>(qk_chunk(stage, lane, j >> 3) + (j & 7) * 2));
      };
      const __nv_bfloat16* cs = cos + row * R;
      const __nv_bfloat16* sn = sin + row * R;
      __nv_bfloat16* yrow = out + (head * M + row) * 128;
#pragma unroll 1
      for (int j0 = 0; j0 < 128; j0 += 8) {
        uint4 pk;
        __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(&pk);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int j = j0 + e;
          const float uj = __fmul_rn(__fmul_rn(zat(j), inv), __bfloat162float(gamma[j]));
          float o = uj;
          if (j < 2 * R) {
            const int pj = j < R ? j + R : j - R;
            const int ang = j < R ? j : j - R;
            const float up = __fmul_rn(__fmul_rn(zat(pj), inv), __bfloat162float(gamma[pj]));
            const float c = __bfloat162float(cs[ang]);
            const float s = __bfloat162float(sn[ang]);
            o = j < R ? __fsub_rn(__fmul_rn(uj, c), __fmul_rn(up, s))
                      : __fadd_rn(__fmul_rn(uj, c), __fmul_rn(up, s));
          }
          h[e] = __float2bfloat16_rn(o);
        }
        *reinterpret_cast<uint4*>(yrow + j0) = pk;
      }
    }
    __syncwarp();  // the staging area is reused by the warp's next item
  }
}

}  // namespace

cudaError_t launch_gated_add(const GatedAddArgs& a, int x_dtype, cudaStream_t stream) {
  switch (x_dtype) {
    case DT_BF16: return launch_gated_add_t<__nv_bfloat16>(a, stream);
    case DT_F16: return launch_gated_add_t<__half>(a, stream);
    case DT_F32: return launch_gated_add_t<float>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_qk_norm_rope(const QkNormArgs& a, cudaStream_t stream) {
  const bool fast = a.fast != 0;
  const void* kern = fast ? reinterpret_cast<const void*>(qk_norm_rope_kernel<true>)
                          : reinterpret_cast<const void*>(qk_norm_rope_kernel<false>);
  static std::atomic<long long> shape[kMaxLaunchDevices];
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e = launch_shape(kern, kQkThreads, 0, shape, &dev, &sms, &per_sm);
  if (e != cudaSuccess) return e;
  const int64_t items = ((a.M + 31) / 32) * (a.N / 128);
  int64_t grid = (items + kQkWarps - 1) / kQkWarps;
  const int64_t cap = int64_t(sms) * per_sm;
  if (grid > cap) grid = cap;
  const auto* p = reinterpret_cast<const __nv_bfloat16*>(a.projected);
  const auto* gm = reinterpret_cast<const __nv_bfloat16*>(a.gamma);
  const auto* cs = reinterpret_cast<const __nv_bfloat16*>(a.cos);
  const auto* sn = reinterpret_cast<const __nv_bfloat16*>(a.sin);
  auto* o = reinterpret_cast<__nv_bfloat16*>(a.out);
  if (fast)
    qk_norm_rope_kernel<true><<<static_cast<unsigned>(grid), kQkThreads, 0, stream>>>(
        p, a.M, a.N, gm, cs, sn, a.rope_half, a.eps, o);
  else
    qk_norm_rope_kernel<false><<<static_cast<unsigned>(grid), kQkThreads, 0, stream>>>(
        p, a.M, a.N, gm, cs, sn, a.rope_half, a.eps, o);
  return cudaGetLastError();
}

}  // namespace m5b
