// Persistent tcgen05 GEMM with fused per-token x per-channel scale epilogues.
//
//   C[m, n] = epilogue( sum_k A[m, k] * B[n, k] )        A: [M, K], B: [N, K], both K-major
//
// Reference operator: src/m5kernels/metal.py:158-269 (gemm) with the epilogue
// strings at metal.py:89-128, and the Q/K projection + RMSNorm + RoPE of
// src/m5kernels/qk_rope.py:120-182 (shaders/qk_rope_projection.metal,
// shaders/qk_rope_body.metal).
//
// Structure (one CTA per SM, 6 warps; optionally CTA pairs, see PAIR below):
//   warp 0     TMA producer: 128-byte K slices of A (128 rows) and B (BN rows)
//              into a STAGES-deep ring of 128B-swizzled shared-memory tiles.
//   warp 1     TMEM allocator + single-thread tcgen05.mma issuer
//              (kind::i8 -> s32, kind::f8f6f4 E4M3 -> f32, kind::f16 -> f32,
//              kind::tf32 -> f32),
//              M=128, N=BN, K=32 bytes per instruction; tcgen05.commit frees a
//              ring slot when its MMAs retire.
//   warps 2-5  epilogue (2-9 on CTA-pair tiles, each warp then draining half
//              of the tile's columns): tcgen05.ld of the accumulator (thread =
//              one output row), scale / bias / gate / RMS+RoPE in registers;
//              16-bit outputs are staged per warp in shared memory (32 rows x
//              32 columns, 64-byte swizzle, double-buffered) and leave with
//              tiled TMA stores, other outputs with direct vector stores.
// Two TMEM accumulators (2 x BN columns) let the epilogue of tile i overlap
// the MMAs of tile i+1.  Tiles are walked in grouped-M order, CTA b taking
// tiles b, b + grid, ...  No TMA multicast is used anywhere.
//
// PAIR (cluster of two CTAs on neighbouring SMs, tcgen05 cta_group::2): the
// tile is 256 x BN.  Each CTA loads its own 128 rows of A and its own BN/2
// rows of B (plain TMA loads, transaction bytes counted on the even CTA's
// barrier); the even CTA's MMA warp issues M=256 MMAs that read both CTAs'
// shared memory and write 128 accumulator rows into each CTA's TMEM.  Per SM
// this halves the B traffic into shared memory, so a 6-deep ring fits.  When
// the last wave of 256 x BN tiles would leave more than half of the pairs
// idle, those tiles run as two 256 x BN/2 halves (second B descriptor with
// half-height boxes, N = BN/2 instruction descriptor).
//
// Rounding contract (bit-reproducible, mirrored by the C oracle):
//   quantized:  v = fp32(acc) * sa[m] * sb[n]   (int32 -> fp32 RNE, then two
//               IEEE multiplies in that order, no contraction)
//   bias:       v = v + bias                    (IEEE add)
//   gate:       out = fma(bf16(v), gate, R)     (bf16 x bf16 product is exact)
//   output:     RNE to the output dtype.
#include "common.cuh"
#include "m5b_internal.h"

namespace m5b {

constexpr int kBM = 128;

template <int BN, bool QK, bool PAIR>
struct GemmCfg {
  static constexpr int A_BYTES = kBM * 128;                 // this CTA's A rows
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;         // this CTA's B rows
  static constexpr int B_BYTES = B_ROWS * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TILE_M = PAIR ? 2 * kBM : kBM;
  // (Q/K pair tiles: 5 stages beside their 64 KB of staging.)
  static constexpr int STAGES = QK ? 5 : (STAGE_BYTES <= 32 * 1024 ? 6 : 4);
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int BAR_BYTES = (2 * STAGES + 7) * 8 + 32;
  // Epilogue warps: 4, or 8 for pair tiles (each warp drains one of the tile's
  // two heads (Q/K), or half of its columns, for its 32 rows).
  static constexpr int EPI_WARPS = PAIR ? 8 : 4;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  // Q/K: 128 rows x 128 bf16 channels per head staged at once; otherwise two
  // 2 KB buffers (32 rows x 32 16-bit columns) per epilogue warp.
  static constexpr int QK_BYTES =
      QK ? (EPI_WARPS / 4) * kBM * 256 : EPI_WARPS * 2 * 2048;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + QK_BYTES + BAR_BYTES + 16;
  static_assert(SMEM_BYTES <= 232448, "shared memory per CTA exceeds 227 KB");
};

__device__ __forceinline__ void tile_coords(int t, const GemmArgs& g, int& m_blk, int& n_blk) {
  // m_blk indexes tiles of TILE_M rows (128, or 256 for a CTA pair).
  const int group_size = g.group_m * g.num_n_blocks;
  const int group = t / group_size;
  const int first_m = group * g.group_m;
  const int rem = g.num_m_blocks - first_m;
  const int gm = rem < g.group_m ? rem : g.group_m;
  const int in_group = t - group * group_size;
  m_blk = first_m + in_group % gm;
  n_blk = in_group / gm;
}

template <int KIND>
__device__ __forceinline__ float acc_value(uint32_t bits) {
  if constexpr (KIND == KIND_I8)
    return __int2float_rn(static_cast<int>(bits));
  else
    return __uint_as_float(bits);
}

__device__ __forceinline__ float bf16_load(const void* base, int64_t i) {
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
}
__device__ __forceinline__ float bf16_round(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}
// Plain / bias / gate epilogue for one thread's 32 consecutive columns.
template <int KIND>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& g, const uint32_t (&r)[32],
                                               int64_t row, int col0, float sa) {
  const int N = g.N;
  const bool full = (col0 + 32 <= N);
  if (g.out_dtype == DT_I32) {  // raw INT32 accumulators (no epilogue arithmetic)
    if (row >= g.M) return;
    int32_t* o = reinterpret_cast<int32_t*>(g.out) + row * int64_t(N) + col0;
    if (full && (N % 4) == 0) {
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<int4*>(o + i) = make_int4(int(r[i]), int(r[i + 1]), int(r[i + 2]), int(r[i + 3]));
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col0 + i < N) o[i] = int(r[i]);
    }
    return;
  }
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float x = acc_value<KIND>(r[i]);
    if (g.quantized) {
      const int col = col0 + i;
      const float sb = (full || col < N) ? __ldg(g.b_scales + (col < N ? col : 0)) : 0.0f;
      x = __fmul_rn(__fmul_rn(x, sa), sb);
    }
    v[i] = x;
  }
  if (row >= g.M) return;
  const int64_t base = row * int64_t(N) + col0;
  if (g.epi == EPI_BIAS_VEC || g.epi == EPI_BIAS_TABLE) {
    const int64_t boff = (g.epi == EPI_BIAS_TABLE) ? int64_t(g.bias_row_map[row]) * N : 0;
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (full || col0 + i < N) v[i] = __fadd_rn(v[i], __ldg(g.bias + boff + col0 + i));
  } else if (g.epi == EPI_ADD_ROWS) {  // (plain loads: the partial may be the output)
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (full || col0 + i < N) v[i] = __fadd_rn(v[i], g.bias[base + i]);
  } else if (g.epi == EPI_GATE_VEC || g.epi == EPI_GATE_TABLE) {
    const int64_t goff = (g.epi == EPI_GATE_TABLE) ? int64_t(g.gate_row_map[row]) * N : 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (full || col0 + i < N) {
        const float branch = bf16_round(v[i]);
        const float gate = bf16_load(g.gate, goff + col0 + i);
        const float res = bf16_load(g.residual, base + i);
        v[i] = __fmaf_rn(branch, gate, res);
      }
    }
  }
  // store
  if (g.out_dtype == DT_F32) {
    float* o = reinterpret_cast<float*>(g.out) + base;
    if (full && (N % 4) == 0) {
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(o + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col0 + i < N) o[i] = v[i];
    }
  } else if (g.out_dtype == DT_F16) {
    __half* o = reinterpret_cast<__half*>(g.out) + base;
    if (full && (N % 8) == 0) {
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint4 pk;
        __half* h = reinterpret_cast<__half*>(&pk);
#pragma unroll
        for (int e = 0; e < 8; ++e) h[e] = __float2half_rn(v[i + e]);
        *reinterpret_cast<uint4*>(o + i) = pk;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col0 + i < N) o[i] = __float2half_rn(v[i]);
    }
  } else {
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(g.out) + base;
    if (full && (N % 8) == 0) {
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint4 pk;
        __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(&pk);
#pragma unroll
        for (int e = 0; e < 8; ++e) h[e] = __float2bfloat16_rn(v[i + e]);
        *reinterpret_cast<uint4*>(o + i) = pk;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col0 + i < N) o[i] = __float2bfloat16_rn(v[i]);
    }
  }
}

// The per-channel scales b_scales[col0 .. col0 + 31] of one 32-column chunk
// (0 past N): eight 16-byte loads, the same address in every lane of the
// warp, issued before the chunk's TMEM load so their latency overlaps it.
__device__ __forceinline__ void load_col_scales(const GemmArgs& g, int col0, float* sb) {
  if (!g.quantized) return;
  if (g.sb_vec && col0 + 32 <= g.N) {
    const float4* p = reinterpret_cast<const float4*>(g.b_scales + col0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 t = __ldg(p + i);
      sb[4 * i] = t.x;
      sb[4 * i + 1] = t.y;
      sb[4 * i + 2] = t.z;
      sb[4 * i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) sb[i] = col0 + i < g.N ? __ldg(g.b_scales + col0 + i) : 0.0f;
  }
}

// The same epilogue for one thread's 32 consecutive columns, rounded to the
// 16-bit output dtype and packed two per word (staged, then a TMA store).
// Columns past N are computed from zero scale / bias / gate and clipped by
// the store.  sb: the chunk's column scales (load_col_scales).
template <int KIND>
__device__ __forceinline__ void epilogue_pack16(const GemmArgs& g, const uint32_t (&r)[32],
                                                int64_t row, int col0, float sa, const float* sb,
                                                uint32_t* pk) {
  const int N = g.N;
  const bool full = (col0 + 32 <= N);
  const bool in_row = row < g.M;
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; i += 2) {  // packed pairs: two IEEE multiplies per element
    float2 x = make_float2(acc_value<KIND>(r[i]), acc_value<KIND>(r[i + 1]));
    if (g.quantized)
      x = __fmul2_rn(__fmul2_rn(x, make_float2(sa, sa)), make_float2(sb[i], sb[i + 1]));
    v[i] = x.x;
    v[i + 1] = x.y;
  }
  if (in_row) {
    const int64_t base = row * int64_t(N) + col0;
    if (g.epi == EPI_BIAS_VEC || g.epi == EPI_BIAS_TABLE) {
      const int64_t boff = (g.epi == EPI_BIAS_TABLE) ? int64_t(g.bias_row_map[row]) * N : 0;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (full || col0 + i < N) v[i] = __fadd_rn(v[i], __ldg(g.bias + boff + col0 + i));
    } else if (g.epi == EPI_ADD_ROWS) {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (full || col0 + i < N) v[i] = __fadd_rn(v[i], g.bias[base + i]);
    } else if (g.epi == EPI_GATE_VEC || g.epi == EPI_GATE_TABLE) {
      const int64_t goff = (g.epi == EPI_GATE_TABLE) ? int64_t(g.gate_row_map[row]) * N : 0;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (full || col0 + i < N) {
          const float branch = bf16_round(v[i]);
          const float gate = bf16_load(g.gate, goff + col0 + i);
          const float res = bf16_load(g.residual, base + i);
          v[i] = __fmaf_rn(branch, gate, res);
        }
      }
    }
  }
  if (g.out_dtype == DT_F16) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
      pk[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      pk[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
  }
}

// ---------------------------------------------------------------- split-K
// With g.sk, CTA pair u works on tile u % T over k-blocks
// [s*nkb/S, (s+1)*nkb/S), s = u / T (T = g.sk_tiles, S = g.sk_splits): the S
// pairs of a tile share its K range, and pairs with the same s walk their
// k-blocks in step, so tiles that share operands read them together.
// Partial accumulators of pair u, CTA `rank` of the pair: 128 rows x BN INT32
// as [chunk][4 words][row] uint4, so the 32 lanes of a warp (32 rows) store
// and load 512 contiguous bytes.
template <int BN>
__device__ __forceinline__ uint4* sk_slot(const GemmArgs& g, int u, uint32_t rank) {
  constexpr int kSlotU4 = kBM * BN * 4 / 16;
  return g.sk_part + static_cast<size_t>(u * 2 + static_cast<int>(rank)) * kSlotU4;
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded spin of one thread until *word >= target (shared memory written by
// other warps of this CTA); records DEV_TIMEOUT_FIXUP and aborts on timeout.
__device__ __forceinline__ void spin_shared_at_least(volatile int* word, int target,
                                                     volatile int* abort, unsigned int* status) {
  if (*word >= target) return;
  const unsigned long long start = globaltimer_ns();
  while (*word < target) {
    if (*abort) return;
    if (globaltimer_ns() - start > kWaitLimitNs) {
      if (status) atomicOr(status, DEV_TIMEOUT_FIXUP);
      *abort = 1;
      return;
    }
  }
}

template <int KIND, int BN, bool QK, bool PAIR>
__global__ void __launch_bounds__(GemmCfg<BN, QK, PAIR>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                   const __grid_constant__ CUtensorMap tmap_b,
                   const __grid_constant__ CUtensorMap tmap_b_half,
                   const __grid_constant__ CUtensorMap tmap_out,
                   const __grid_constant__ CUtensorMap tmap_out_k,
                   const __grid_constant__ CUtensorMap tmap_out_v, const GemmArgs g) {
  using Cfg = GemmCfg<BN, QK, PAIR>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int K_ELEMS = KIND == KIND_TF32 ? 32 : (KIND == KIND_BF16 || KIND == KIND_F16) ? 64 : 128;
  constexpr uint32_t IDESC = make_idesc(KIND, Cfg::TILE_M, BN);
  constexpr uint32_t IDESC_HALF = make_idesc(KIND, Cfg::TILE_M, BN / 2);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint8_t* qk_stage = sB + STAGES * Cfg::B_BYTES;  // 1024-aligned epilogue staging
  uint64_t* full = reinterpret_cast<uint64_t*>(qk_stage + Cfg::QK_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* fix_bar = drain + 1;  // split-K: partner partial sums landed in shared memory
  uint64_t* recv_ready = fix_bar + 1;  // cluster split-K: the receiving CTA's ring is free
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_ready + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // split-K hand-offs between the epilogue warps of this CTA (see below)
  volatile int* sk_ticket = reinterpret_cast<volatile int*>(tmem_slot + 2);
  volatile int* sk_signal = reinterpret_cast<volatile int*>(tmem_slot + 3);
  int* sk_stored = reinterpret_cast<int*>(tmem_slot + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Clusters are one CTA pair, or two pairs (ranks 0-1 and 2-3) under the
  // cluster split-K schedule.
  const uint32_t crank = PAIR ? cluster_rank() : 0;  // rank in the cluster
  const uint32_t rank = crank & 1u;                   // position in the CTA pair
  const uint32_t pair_even = crank & ~1u;             // the pair's even CTA
  const uint16_t pair_mask = static_cast<uint16_t>(3u << pair_even);
  const bool leader = rank == 0;
  const int unit = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int units = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], (PAIR ? 2 : 1) * Cfg::EPI_WARPS);
    }
    mbar_init(drain, 1);
    mbar_init(fix_bar, 1);
    mbar_init(recv_ready, 1);
    *abort_flag = 0;
    *sk_ticket = 0;
    *sk_signal = 0;
    *sk_stored = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    if (g.num_units > g.num_full) tma_prefetch_desc(&tmap_b_half);
    if ((QK && g.qk_fast) || (!QK && g.tma_store)) tma_prefetch_desc(&tmap_out);
    if (QK && g.qk_fast && g.grouped) {
      tma_prefetch_desc(&tmap_out_k);
      tma_prefetch_desc(&tmap_out_v);
    }
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // every CTA's barriers exist before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int nkb = g.num_k_blocks;
  // Work items of this CTA (pair), walked identically by the producer, MMA
  // and epilogue roles:
  //   data-parallel: units t = unit, unit + units, ... -- whole tiles, then
  //     the N-halves of a split last wave -- each over all k-blocks;
  //   split-K (g.sk, PAIR only): one item, tile unit % T over the k-blocks
  //     of split unit / T.
  struct Work {
    int tile, m_blk, n_col, kb0, kb1;
    bool whole, first;
  };
  const bool sk = PAIR && g.sk;
  const long long work_start = unit;
  auto next_work = [&](long long& cur, Work& w) -> bool {
    int n_blk;
    if (sk) {  // one item: a tile and this pair's K range of it
      if (cur != unit) return false;
      // cluster split-K: the two pairs of cluster c take tile c, splits 0 / 1
      w.tile = g.sk_cluster ? unit >> 1 : unit % g.sk_tiles;
      const int split = g.sk_cluster ? unit & 1 : unit / g.sk_tiles;
      w.kb0 = split * nkb / g.sk_splits;
      w.kb1 = (split + 1) * nkb / g.sk_splits;
      w.first = true;
      cur = -1;
      tile_coords(w.tile, g, w.m_blk, n_blk);
      w.n_col = n_blk * BN;
      w.whole = true;
      return true;
    }
    if (cur >= g.num_units) return false;
    const int u = static_cast<int>(cur);
    if (u < g.num_full) {
      tile_coords(u, g, w.m_blk, n_blk);
      w.n_col = n_blk * BN;
      w.whole = true;
    } else {
      const int h = u - g.num_full;
      tile_coords(g.num_full + (h >> 1), g, w.m_blk, n_blk);
      w.n_col = n_blk * BN + (h & 1) * (BN / 2);
      w.whole = false;
    }
    w.tile = u;
    w.kb0 = 0;
    w.kb1 = nkb;
    w.first = true;
    cur += units;
    return true;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      // With programmatic dependent launch the set-up above overlapped the
      // previous kernel; the operands it may have written are read only now.
      grid_dependency_wait();
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      long long cur = work_start;
      Work w;
      // INT8 data-parallel tiles walk K forward and backward in turn, so a
      // tile starts on the k-slices its predecessor (and the other pairs of
      // the same wave) just left in L2: fewer operand re-reads from DRAM.
      // INT32 sums are exact in any order, so the result does not change;
      // FP32-accumulating kinds keep the forward order.  Both CTAs of a pair
      // walk the same work items, so they agree on the direction.
      int tiles_done = 0;
      while (!*abort_flag && next_work(cur, w)) {
        const bool backward = KIND == KIND_I8 && !sk && (tiles_done++ & 1);
        const int a_row = w.m_blk * Cfg::TILE_M + static_cast<int>(rank) * kBM;
        const int b_rows = w.whole ? Cfg::B_ROWS : Cfg::B_ROWS / 2;
        const int b_row = w.n_col + static_cast<int>(rank) * b_rows;
        const CUtensorMap* bmap = w.whole ? &tmap_b : &tmap_b_half;
        const uint32_t stage_bytes = Cfg::A_BYTES + b_rows * 128;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait_bounded(&empty[stage], phase ^ 1u, abort_flag, g.status,
                                 DEV_TIMEOUT_PRODUCER))
            break;
          const int kx = (backward ? w.kb1 - 1 - (kb - w.kb0) : kb) * K_ELEMS;
          if constexpr (PAIR) {
            // The even CTA expects both CTAs' bytes; each CTA loads its halves.
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * stage_bytes);
            tma_load_2d_pair(sA + stage * Cfg::A_BYTES, &tmap_a, &full[stage], kx, a_row);
            tma_load_2d_pair(sB + stage * Cfg::B_BYTES, bmap, &full[stage], kx, b_row);
          } else {
            mbar_arrive_expect_tx(&full[stage], stage_bytes);
            tma_load_2d(sA + stage * Cfg::A_BYTES, &tmap_a, &full[stage], kx, a_row);
            tma_load_2d(sB + stage * Cfg::B_BYTES, bmap, &full[stage], kx, b_row);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (*abort_flag && (!PAIR || leader)) {
        // Drain: wait (bounded) until the copies already issued into the
        // ring have landed, so no TMA write targets this CTA after it exits.
        // (In a pair the even CTA's barriers count both CTAs' copies; the
        // closing cluster barrier keeps the odd CTA alive until then.)
        int s = stage, ph = phase;
        for (int i = 0; i < STAGES && i < issued; ++i) {
          s = (s == 0) ? STAGES - 1 : s - 1;
          if (s == STAGES - 1) ph ^= 1;
          const unsigned long long t0 = globaltimer_ns();
          while (!mbar_try_wait(&full[s], ph)) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
              atomicOr(g.status, DEV_TIMEOUT_DRAIN);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if ((!PAIR || leader) && elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      long long cur = work_start;
      Work w;
      for (; ok && next_work(cur, w); ++local) {
        const uint32_t idesc = w.whole ? IDESC : IDESC_HALF;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait_bounded(&acc_empty[acc], acc_phase ^ 1u, abort_flag, g.status,
                               DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait_bounded(&full[stage], phase, abort_flag, g.status, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t accumulate = (kb != w.kb0 || k != 0) ? 1u : 0u;
            if constexpr (PAIR)
              tc_mma_pair<KIND>(d_tmem, smem_desc_k128(a_base + k * 32),
                                smem_desc_k128(b_base + k * 32), idesc, accumulate);
            else
              tc_mma<KIND>(d_tmem, smem_desc_k128(a_base + k * 32),
                           smem_desc_k128(b_base + k * 32), idesc, accumulate);
          }
          if constexpr (PAIR)
            tc_commit_pair(&empty[stage], pair_mask);
          else
            tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (PAIR)
          tc_commit_pair(&acc_full[acc], pair_mask);
        else
          tc_commit(&acc_full[acc]);
      }
      if (!ok) {
        // Aborted: let every MMA already issued retire before TMEM is freed.
        if constexpr (PAIR)
          tc_commit_pair(drain, pair_mask);
        else
          tc_commit(drain);
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(drain, 0)) {
          if (globaltimer_ns() - t0 > kWaitLimitNs) {
            atomicOr(g.status, DEV_TIMEOUT_DRAIN);
            break;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int ehalf = (warp - 2) >> 2;  // 8-warp Q/K epilogue: which head of the tile
    const int row_in_tile = static_cast<int>(rank) * kBM + quarter * 32 + lane;
    // acc_empty lives in the even CTA of a pair: the odd CTA arrives remotely.
    const uint32_t acc_empty_remote0 = PAIR ? map_to_rank(&acc_empty[0], pair_even) : 0u;
    const uint32_t acc_empty_remote1 = PAIR ? map_to_rank(&acc_empty[1], pair_even) : 0u;
    auto release_acc = [&](int acc) {
      if constexpr (PAIR)
        mbar_arrive_cluster(acc == 0 ? acc_empty_remote0 : acc_empty_remote1);
      else
        mbar_arrive(&acc_empty[acc]);
    };
    // plain epilogues: this warp's two staging buffers and their use count
    uint8_t* out_stage = qk_stage + (warp - 2) * 4096;
    const uint64_t out_policy = l2_policy_evict_first();
    uint32_t ostage = 0;
    int local = 0;
    long long cur = work_start;
    Work w;
    // Split-K hand-offs between this CTA's epilogue warps, all through
    // bounded spins on shared words (no hardware barrier a timed-out warp
    // could leave waiting): sk_signal counts the leader's announcements (the
    // arrival ticket is readable; the other pairs' partial sums are ready),
    // sk_stored counts warps whose partial stores are complete.  Every warp
    // walks the same work items, so all of them expect the same counts.
    int sig_expect = 0, stored_expect = 0;
    uint32_t fix_phase = 0;
    const bool sk_leader = threadIdx.x == 64;  // lane 0 of the first epilogue warp
    // scales, bias, gate, residual and the outputs are touched only after the
    // previous kernel in the stream has completed (programmatic launch)
    grid_dependency_wait();
    const int prow = quarter * 32 + lane;      // this thread's row within the CTA's 128
    for (; next_work(cur, w); ++local) {
      const int m_blk = w.m_blk, n_col = w.n_col;
      const bool whole = w.whole;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_bounded(&acc_full[acc], acc_phase, abort_flag, g.status,
                             DEV_TIMEOUT_EPILOGUE))
        break;
      __syncwarp();
      tc_fence_after();
      const int64_t row = int64_t(m_blk) * Cfg::TILE_M + row_in_tile;
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      const float sa = (g.quantized && row < g.M) ? __ldg(g.a_scales + row) : 1.0f;
      // Split-K: the S pairs of a tile each take an arrival ticket per CTA.
      // All but the last stage their INT32 partial sums in the (now idle)
      // operand ring, store them to their workspace slot with one bulk copy
      // and count them done.  The last waits (bounded) until the others are
      // done, resets the counters, and for each partner bulk-loads its slot
      // into the ring and adds it into its own TMEM accumulator; the ordinary
      // epilogue then reads complete sums.  (All of this CTA's MMAs have
      // retired once acc_full completed, so the ring's 192 KB are free.)
      if (sk && g.sk_cluster) {
        // Cluster split-K: this cluster's two pairs took the two K halves of
        // one tile.  The second pair (ranks 2-3) stages its partial sums in
        // its idle ring and bulk-copies them into the ring of its
        // counterpart in the first pair (rank - 2: the same 128 rows), once
        // that CTA has announced its own MMAs done (recv_ready, its ring is
        // then free) and armed its fix_bar for the bytes.  The first pair
        // adds them into its TMEM accumulator and runs the epilogue.
        uint4* ring = reinterpret_cast<uint4*>(smem);  // [chunk][4 words][row] uint4
        constexpr int kChunks = BN / 32;
        const int c_first = Cfg::EPI_WARPS == 8 ? ehalf * (kChunks / 2) : 0;
        const int c_end = Cfg::EPI_WARPS == 8 ? c_first + kChunks / 2 : kChunks;
        constexpr uint32_t kSlotBytes = kBM * BN * 4;
        if (crank >= 2) {  // sender
#pragma unroll 1
          for (int c = c_first; c < c_end; ++c) {
            uint32_t r[32];
            tmem_ld32(taddr + c * 32, r);
            tmem_wait_ld();
            if (c == c_end - 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) release_acc(acc);
            }
#pragma unroll
            for (int q = 0; q < 8; ++q)
              ring[(c * 8 + q) * kBM + prow] =
                  make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
          }
          fence_proxy_async_shared();  // the bulk copy (async proxy) reads these writes
          __syncwarp();
          stored_expect += Cfg::EPI_WARPS;
          if (lane == 0) atomicAdd(sk_stored, 1);
          if (sk_leader) {
            spin_shared_at_least(sk_stored, stored_expect, abort_flag, g.status);
            if (!*abort_flag &&
                mbar_wait_bounded(recv_ready, 0, abort_flag, g.status, DEV_TIMEOUT_FIXUP)) {
              const uint32_t dst = map_to_rank(ring, crank - 2);
              const uint32_t bar = map_to_rank(fix_bar, crank - 2);
              for (uint32_t off = 0; off < kSlotBytes; off += 16384)
                bulk_copy_s2cluster(dst + off, reinterpret_cast<const uint8_t*>(ring) + off, 16384,
                                    bar);
            }
          }
          __syncwarp();
          continue;  // (the kernel's closing cluster barrier keeps this ring alive until read)
        }
        if (sk_leader) {  // receiver: arm fix_bar, then let the sender copy
          mbar_arrive_expect_tx(fix_bar, kSlotBytes);
          mbar_arrive_cluster(map_to_rank(recv_ready, crank + 2));
        }
        if (!mbar_wait_bounded(fix_bar, fix_phase, abort_flag, g.status, DEV_TIMEOUT_FIXUP))
          break;
        fix_phase ^= 1u;
#pragma unroll 1
        for (int c = c_first; c < c_end; ++c) {
          uint32_t r[32];
          tmem_ld32(taddr + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const uint4 pv = ring[(c * 8 + q) * kBM + prow];
            r[4 * q] += pv.x;
            r[4 * q + 1] += pv.y;
            r[4 * q + 2] += pv.z;
            r[4 * q + 3] += pv.w;
          }
          tmem_st32(taddr + c * 32, r);
          tmem_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        tc_fence_after();
      } else if (sk) {
        const int others = g.sk_splits - 1;
        int* ctr = g.sk_ctr + (w.tile * 2 + static_cast<int>(rank)) * 2;
        uint4* ring = reinterpret_cast<uint4*>(smem);  // [chunk][4 words][row] uint4
        constexpr int kChunks = BN / 32;
        const int c_first = Cfg::EPI_WARPS == 8 ? ehalf * (kChunks / 2) : 0;
        const int c_end = Cfg::EPI_WARPS == 8 ? c_first + kChunks / 2 : kChunks;
        constexpr uint32_t kSlotBytes = kBM * BN * 4;
        ++sig_expect;
        if (sk_leader) {
          *sk_ticket = atomicAdd(ctr, 1);
          __threadfence_block();
          *sk_signal = sig_expect;
        }
        if (lane == 0) spin_shared_at_least(sk_signal, sig_expect, abort_flag, g.status);
        __syncwarp();
        const int ticket = *sk_ticket;
        if (ticket < others) {
#pragma unroll 1
          for (int c = c_first; c < c_end; ++c) {
            uint32_t r[32];
            tmem_ld32(taddr + c * 32, r);
            tmem_wait_ld();
            if (c == c_end - 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) release_acc(acc);
            }
#pragma unroll
            for (int q = 0; q < 8; ++q)
              ring[(c * 8 + q) * kBM + prow] =
                  make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
          }
          fence_proxy_async_shared();  // the bulk copy (async proxy) reads these writes
          __syncwarp();
          stored_expect += Cfg::EPI_WARPS;
          if (lane == 0) atomicAdd(sk_stored, 1);
          if (sk_leader) {
            spin_shared_at_least(sk_stored, stored_expect, abort_flag, g.status);
            bulk_store_s2g(sk_slot<BN>(g, unit, rank), ring, kSlotBytes);
            bulk_commit_group();
            bulk_wait_group0();        // the partial sums are in global memory
            fence_proxy_async_global();
            __threadfence();
            atomicAdd(ctr + 1, 1);
          }
          __syncwarp();
          continue;
        }
        ++sig_expect;
        if (sk_leader) {
          const unsigned long long start = globaltimer_ns();
          while (ld_acquire_gpu(ctr + 1) < others) {
            if (*abort_flag) break;
            if (globaltimer_ns() - start > kWaitLimitNs) {
              atomicOr(g.status, DEV_TIMEOUT_FIXUP);
              *abort_flag = 1;
              break;
            }
          }
          ctr[0] = 0;  // zero again for the next launch
          ctr[1] = 0;
          __threadfence();
          fence_proxy_async_global();  // the partners' slots are read by bulk copies
          *sk_signal = sig_expect;
        }
        if (lane == 0) spin_shared_at_least(sk_signal, sig_expect, abort_flag, g.status);
        __syncwarp();
        for (int s = 0; s < g.sk_splits; ++s) {
          const int v = w.tile + s * g.sk_tiles;
          if (v == unit) continue;
          if (sk_leader) {
            mbar_arrive_expect_tx(fix_bar, kSlotBytes);
            const uint8_t* src = reinterpret_cast<const uint8_t*>(sk_slot<BN>(g, v, rank));
            for (uint32_t off = 0; off < kSlotBytes; off += 16384)
              bulk_load_g2s(reinterpret_cast<uint8_t*>(ring) + off, src + off, 16384, fix_bar);
          }
          if (!mbar_wait_bounded(fix_bar, fix_phase, abort_flag, g.status, DEV_TIMEOUT_FIXUP))
            break;
          fix_phase ^= 1u;
#pragma unroll 1
          for (int c = c_first; c < c_end; ++c) {
            uint32_t r[32];
            tmem_ld32(taddr + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const uint4 pv = ring[(c * 8 + q) * kBM + prow];
              r[4 * q] += pv.x;
              r[4 * q + 1] += pv.y;
              r[4 * q + 2] += pv.z;
              r[4 * q + 3] += pv.w;
            }
            tmem_st32(taddr + c * 32, r);
            tmem_wait_st();
          }
          // every warp has read the ring before the next partner's copy lands
          __syncwarp();
          stored_expect += Cfg::EPI_WARPS;
          if (lane == 0) atomicAdd(sk_stored, 1);
          if (lane == 0) spin_shared_at_least(sk_stored, stored_expect, abort_flag, g.status);
          __syncwarp();
        }
        tc_fence_before();
        __syncwarp();
        tc_fence_after();
      }
      if constexpr (!QK) {
        // This warp's 32-column chunks: all of the tile's, or with 8 warps
        // the half matching ehalf.
        const int chunks = whole ? BN / 32 : BN / 64;
        const int c_first = Cfg::EPI_WARPS == 8 ? ehalf * (chunks / 2) : 0;
        const int c_end = Cfg::EPI_WARPS == 8 ? c_first + chunks / 2 : chunks;
        if (g.tma_store) {
          const int64_t row0 = row - lane;  // this warp's first row
#pragma unroll 1
          for (int c = c_first; c < c_end; ++c) {
            float sbc[32];
            load_col_scales(g, n_col + c * 32, sbc);
            uint32_t r[32];
            tmem_ld32(taddr + c * 32, r);
            tmem_wait_ld();
            if (c == c_end - 1) {  // the accumulator is drained: hand it back
              tc_fence_before();
              __syncwarp();
              if (lane == 0) release_acc(acc);
            }
            uint32_t pk[16];
            epilogue_pack16<KIND>(g, r, row, n_col + c * 32, sa, sbc, pk);
            uint8_t* buf = out_stage + (ostage & 1) * 2048;
            if (lane == 0) bulk_wait_group_read1();  // the store two chunks back has read buf
            __syncwarp();
            // row `lane` of a 32 x 64-byte box; 64-byte swizzle: 16-byte
            // chunk j sits at j ^ ((row >> 1) & 3)
            const int sw = (lane >> 1) & 3;
#pragma unroll
            for (int j = 0; j < 4; ++j)
              *reinterpret_cast<uint4*>(buf + lane * 64 + ((j ^ sw) << 4)) =
                  make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
            fence_proxy_async_shared();
            __syncwarp();
            if (lane == 0 && row0 < g.M && n_col + c * 32 < g.N) {
              // evict-first: the output is not read by this kernel, and its
              // write-back then overlaps the MMAs instead of the next kernel
              tma_store_2d_hint(&tmap_out, buf, g.col_off + n_col + c * 32,
                                static_cast<int32_t>(row0), out_policy);
              bulk_commit_group();
            }
            if (g.n_peers > 0 && ((c - c_first) & 1)) {
              // Column-parallel all-gather, after every second chunk: the two
              // staged 32 x 32 blocks (this chunk's buffer and the previous
              // one's) go to every peer rank's output over NVLink as 128-byte
              // row segments, eight lanes per row, 16-byte stores.  (Staging
              // reads are generic-proxy reads beside the TMA stores', both
              // only read; the previous buffer is refilled only after these.)
              // Every warp drains an even number of chunks per tile.
              const uint8_t* bufs[2] = {out_stage + ((ostage - 1) & 1) * 2048, buf};
              const int col_pair = n_col + (c - 1) * 32;
#pragma unroll
              for (int p = lane; p < 256; p += 32) {
                const int rr = p >> 3, h = (p >> 2) & 1, j = p & 3;
                const int col = col_pair + h * 32 + j * 8;
                if (row0 + rr < g.M && col < g.N) {
                  const uint4 v = *reinterpret_cast<const uint4*>(bufs[h] + rr * 64 +
                                                                  ((j ^ ((rr >> 1) & 3)) << 4));
                  const int64_t off = (row0 + rr) * g.ldo + g.col_off + col;  // elements
                  for (int q = 0; q < g.n_peers; ++q)
                    *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(g.peer_out[q]) + off) = v;
                }
              }
            }
            ++ostage;
          }
          if (c_first >= c_end) {  // no columns for this warp (cannot happen: chunks >= 2)
            tc_fence_before();
            __syncwarp();
            if (lane == 0) release_acc(acc);
          }
        } else {
#pragma unroll 1
          for (int c = c_first; c < c_end; ++c) {
            uint32_t r[32];
            tmem_ld32(taddr + c * 32, r);
            tmem_wait_ld();
            epilogue_chunk<KIND>(g, r, row, n_col + c * 32, sa);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release_acc(acc);
        }
      } else {
        // One or two 128-wide heads per unit.  Per head, pass 1: BF16
        // projection z, its square sum (sequential over the head's 128
        // channels) and a staged copy of this thread's row; pass 2: RMS,
        // gamma, split-half RoPE and the head-major store.
        //
        // Staging: each warp owns 32 rows x 128 channels (8 KB) as two
        // 64-channel halves of 32 rows x 128 bytes whose 16-byte chunks are
        // XOR-swizzled by (row & 7) -- the TMA 128-byte swizzle, so one
        // thread's row is read and written without bank conflicts and the
        // finished 32 x 128 head block leaves with two tiled TMA stores
        // (rows past M clipped by the tensor map).
        constexpr bool kHeadPerWarp = Cfg::EPI_WARPS == 8;
        uint8_t* wstage = qk_stage + (kHeadPerWarp ? ehalf * (kBM * 256) : 0) + quarter * 8192;
        auto chunk = [&](int ch) -> uint8_t* {  // channels 8*ch .. 8*ch+7 of this row
          return wstage + (ch >> 3) * 4096 + lane * 128 + (((ch & 7) ^ (lane & 7)) << 4);
        };
        const int heads_tile = whole ? BN / 128 : (BN / 2) / 128;
        const int heads_left = (g.N - n_col) / 128;  // N tail: a second head may not exist
        const int heads_here = heads_left < heads_tile ? (heads_left > 0 ? heads_left : 0)
                                                       : heads_tile;
        // this warp's heads: all of them, or with 8 warps the one matching ehalf
        const int h_first = kHeadPerWarp ? ehalf : 0;
        const int h_step = kHeadPerWarp ? BN / 128 : 1;
        int h_last = -1;
        for (int hh = h_first; hh < heads_here; hh += h_step) h_last = hh;
        if (h_last < 0) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release_acc(acc);
        }
        const int64_t row0 = row - lane;  // this warp's first row
#pragma unroll 1
        for (int hh = h_first; hh < heads_here; hh += h_step) {
          // 128-column block of the projection; grouped Q/K/V weights order
          // the blocks [head, stream], one output tensor per stream.
          const int hb = n_col / 128 + hh;
          const int head = g.grouped ? hb / 3 : hb;
          const int stream_id = g.grouped ? hb - 3 * head : 0;  // 0 Q, 1 K, 2 V
          const bool norm_rope = stream_id != 2;  // V: projection and layout only
          if (lane == 0) bulk_wait_group_read0();  // the previous store has read the staging
          __syncwarp();
          // This row's cos / sin chunks (16 bytes each, R % 8 == 0 path): issued
          // before the accumulator drain so the loads (one row per lane) are in
          // flight while pass 1 runs.
          uint4 cpre[8], spre[8];
          if (g.qk_fast && norm_rope && row < g.M) {
            const int RC = g.rope_half >> 3;
            const uint4* cs4 = reinterpret_cast<const uint4*>(
                reinterpret_cast<const __nv_bfloat16*>(g.cos) + row * g.rope_half);
            const uint4* sn4 = reinterpret_cast<const uint4*>(
                reinterpret_cast<const __nv_bfloat16*>(g.sin) + row * g.rope_half);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              if (q < RC) {
                cpre[q] = __ldg(cs4 + q);
                spre[q] = __ldg(sn4 + q);
              }
            }
          }
          float sumsq = 0.0f;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float sbc[32];
            load_col_scales(g, hb * 128 + c * 32, sbc);  // N % 128 == 0: whole chunks
            uint32_t r[32];
            tmem_ld32(taddr + hh * 128 + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint32_t pk[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int e = q * 8 + 2 * i;
                float2 z = make_float2(acc_value<KIND>(r[e]), acc_value<KIND>(r[e + 1]));
                if (g.quantized)
                  z = __fmul2_rn(__fmul2_rn(z, make_float2(sa, sa)),
                                 make_float2(sbc[e], sbc[e + 1]));
                const __nv_bfloat162 zz = __float22bfloat162_rn(z);
                const float f0 = __low2float(zz), f1 = __high2float(zz);
                sumsq = __fmaf_rn(f0, f0, sumsq);
                sumsq = __fmaf_rn(f1, f1, sumsq);
                pk[i] = *reinterpret_cast<const uint32_t*>(&zz);
              }
              *reinterpret_cast<uint4*>(chunk(c * 4 + q)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            }
          }
          if (hh == h_last) {
            // The accumulator is no longer needed: hand it back to the MMA warp.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) release_acc(acc);
          }
          const float inv =
              __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sumsq, 128.0f), g.eps)));
          const int R = g.rope_half;
          const __nv_bfloat16* gm =
              reinterpret_cast<const __nv_bfloat16*>(stream_id == 1 ? g.gamma_k : g.gamma);
          const CUtensorMap* omap =
              stream_id == 0 ? &tmap_out : (stream_id == 1 ? &tmap_out_k : &tmap_out_v);
          void* obase = stream_id == 0 ? g.out : (stream_id == 1 ? g.out_k : g.out_v);
          if (g.qk_fast) {
            // R % 8 == 0: channel a pairs with a + R, both whole 16-byte chunks.
            if (row < g.M && norm_rope) {
              const int RC = R >> 3;
              const uint4* gm4 = reinterpret_cast<const uint4*>(gm);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                if (q >= RC) break;
                uint4 zl = *reinterpret_cast<const uint4*>(chunk(q));
                uint4 zh = *reinterpret_cast<const uint4*>(chunk(q + RC));
                rope_chunk16(zl, zh, __ldg(gm4 + q), __ldg(gm4 + q + RC), cpre[q], spre[q], inv);
                *reinterpret_cast<uint4*>(chunk(q)) = zl;
                *reinterpret_cast<uint4*>(chunk(q + RC)) = zh;
              }
#pragma unroll 1
              for (int q = 2 * RC; q < 16; ++q)
                *reinterpret_cast<uint4*>(chunk(q)) =
                    norm_chunk16(*reinterpret_cast<const uint4*>(chunk(q)), __ldg(gm4 + q), inv);
            }
            fence_proxy_async_shared();
            __syncwarp();
            if (lane == 0 && row0 < g.M) {
              tma_store_3d(omap, wstage, 0, static_cast<int32_t>(row0), head);
              tma_store_3d(omap, wstage + 4096, 64, static_cast<int32_t>(row0), head);
              bulk_commit_group();
            }
          } else if (row < g.M) {
            // Any R in [1, 64]: element-wise from the staged row, direct stores.
            auto zat = [&](int j) -> float {
              return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(chunk(j >> 3) +
                                                                              (j & 7) * 2));
            };
            const __nv_bfloat16* cs = reinterpret_cast<const __nv_bfloat16*>(g.cos) + row * R;
            const __nv_bfloat16* sn = reinterpret_cast<const __nv_bfloat16*>(g.sin) + row * R;
            __nv_bfloat16* yrow =
                reinterpret_cast<__nv_bfloat16*>(obase) + (int64_t(head) * g.M + row) * 128;
#pragma unroll 1
            for (int j0 = 0; j0 < 128; j0 += 8) {
              uint4 pk;
              __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(&pk);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const int j = j0 + e;
                if (!norm_rope) {  // V stream: the BF16 projection itself
                  h[e] = __float2bfloat16_rn(zat(j));
                  continue;
                }
                const float uj = __fmul_rn(__fmul_rn(zat(j), inv), __bfloat162float(gm[j]));
                float out = uj;
                if (j < 2 * R) {
                  const int p = j < R ? j + R : j - R;
                  const int ang = j < R ? j : j - R;
                  const float up = __fmul_rn(__fmul_rn(zat(p), inv), __bfloat162float(gm[p]));
                  const float c = __bfloat162float(cs[ang]);
                  const float s = __bfloat162float(sn[ang]);
                  out = j < R ? __fsub_rn(__fmul_rn(uj, c), __fmul_rn(up, s))
                              : __fadd_rn(__fmul_rn(uj, c), __fmul_rn(up, s));
                }
                h[e] = __float2bfloat16_rn(out);
              }
              *reinterpret_cast<uint4*>(yrow + j0) = pk;
            }
          }
        }
      }
    }
    if (lane == 0) bulk_wait_group0();  // this warp's TMA stores are complete
    if (g.n_peers > 0) __threadfence_system();  // peer stores performed before the grid ends
    __syncwarp();
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the peer no longer touches this CTA
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

template <int KIND, int BN, bool QK, bool PAIR>
static cudaError_t launch_k(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tbh,
                            const CUtensorMap& to, const CUtensorMap& tok, const CUtensorMap& tov,
                            const GemmArgs& g, int grid, cudaStream_t stream) {
  using Cfg = GemmCfg<BN, QK, PAIR>;
  auto kern = gemm_tc_kernel<KIND, BN, QK, PAIR>;
  static std::atomic<long long> shape[kMaxLaunchDevices];
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e = launch_shape(reinterpret_cast<const void*>(kern), Cfg::THREADS, Cfg::SMEM_BYTES, shape,
                               &dev, &sms, &per_sm);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n_attr = 0;
  if (PAIR) {
    attr[n_attr].id = cudaLaunchAttributeClusterDimension;
    attr[n_attr].val.clusterDim.x = g.sk && g.sk_cluster ? 4 : 2;
    attr[n_attr].val.clusterDim.y = 1;
    attr[n_attr].val.clusterDim.z = 1;
    ++n_attr;
  }
  if (g.pdl) {  // programmatic dependent launch (see grid_dependency_wait)
    attr[n_attr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n_attr].val.programmaticStreamSerializationAllowed = 1;
    ++n_attr;
  }
  cfg.attrs = n_attr ? attr : nullptr;
  cfg.numAttrs = n_attr;
  e = cudaLaunchKernelEx(&cfg, kern, ta, tb, tbh, to, tok, tov, g);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

int gemm_block_n(const GemmArgs& g) { return g.N <= 128 ? 128 : 256; }

cudaError_t launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tbh,
                        const CUtensorMap& to, const CUtensorMap& tok, const CUtensorMap& tov,
                        const GemmArgs& g, int bn, int grid, bool pair, cudaStream_t stream) {
  const bool qk = g.epi == EPI_QK;
#define M5B_ARGS ta, tb, tbh, to, tok, tov, g, grid, stream
#define M5B_KIND_CASE(KIND_)                                                  \
  case KIND_:                                                                 \
    if (qk) return pair ? launch_k<KIND_, 256, true, true>(M5B_ARGS)          \
                        : launch_k<KIND_, 128, true, false>(M5B_ARGS);        \
    if (pair) return launch_k<KIND_, 256, false, true>(M5B_ARGS);             \
    if (bn == 128) return launch_k<KIND_, 128, false, false>(M5B_ARGS);       \
    return launch_k<KIND_, 256, false, false>(M5B_ARGS);
  switch (g.kind) {
    M5B_KIND_CASE(KIND_I8)
    M5B_KIND_CASE(KIND_F8)
    M5B_KIND_CASE(KIND_BF16)
    M5B_KIND_CASE(KIND_F16)
    case KIND_TF32:  // plain epilogues only (the FP32 GEMM mode)
      if (qk) return cudaErrorInvalidValue;
      if (pair) return launch_k<KIND_TF32, 256, false, true>(M5B_ARGS);
      if (bn == 128) return launch_k<KIND_TF32, 128, false, false>(M5B_ARGS);
      return launch_k<KIND_TF32, 256, false, false>(M5B_ARGS);
    default: return cudaErrorInvalidValue;
  }
#undef M5B_KIND_CASE
#undef M5B_ARGS
}

}  // namespace m5b
