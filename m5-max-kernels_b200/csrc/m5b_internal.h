// Launch-argument structs shared by the kernels (prep.cu, gemm.cu) and the
// C-ABI layer (api.cu).  Nothing in here is exported from the library.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace m5b {

// Launch shape of one kernel instance on one device, computed once: the
// dynamic shared-memory attribute is set and the occupancy query made on the
// first launch with a given shared-memory size, and reused afterwards (the
// host path of a launch then makes no attribute or occupancy calls).  `slot`
// is the instance's per-device cache entry; racing first launches both
// compute the same value.
constexpr int kMaxLaunchDevices = 64;
inline cudaError_t launch_shape(const void* kern, int threads, int smem,
                                std::atomic<long long>* slots, int* dev_out, int* sms_out,
                                int* per_sm_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxLaunchDevices) return cudaErrorInvalidDevice;
  *dev_out = dev;
  static std::atomic<int> sms_cache[kMaxLaunchDevices];
  int sms = sms_cache[dev].load(std::memory_order_relaxed);
  if (sms == 0) {
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    sms_cache[dev].store(sms, std::memory_order_relaxed);
  }
  *sms_out = sms;
  const long long key = static_cast<long long>(smem + 1) << 32;
  const long long v = slots[dev].load(std::memory_order_acquire);
  if (v != 0 && (v & ~0xFFFFFFFFll) == key) {
    *per_sm_out = static_cast<int>(v & 0xFFFFFFFFll);
    return cudaSuccess;
  }
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) per_sm = 1;
  slots[dev].store(key | per_sm, std::memory_order_release);
  *per_sm_out = per_sm;
  return cudaSuccess;
}

enum NormKind : int { NORM_NONE = 0, NORM_RMS = 1, NORM_LAYER = 2 };
// OUT_ROW: the (modulated) row itself in the input dtype, no rotation -- the
// staged norm + modulation comparator; OUT_F32 writes fp32 rows.
enum RowOut : int { OUT_INT8 = 0, OUT_E4M3 = 1, OUT_F32 = 2, OUT_ROW = 3 };
// RMS scale folding (codes from (X gamma) D H, inverse RMS in the row scale)
// and its direct counterpart (normalize first); both INT8 only.
enum RmsQuant : int { RMSQ_NONE = 0, RMSQ_FOLD = 1, RMSQ_DIRECT = 2 };

struct RowPrepArgs {
  const void* x;               // [rows, K] input (the residual R when gated)
  const void* branch;          // [rows, K] gated branch, or null
  const void* gate;            // [K] or [P, K] gate table, or null
  const int32_t* gate_row_map; // [rows] gate table index, or null
  int gate_dtype;
  const void* gamma;           // [K] (norm only)
  const void* scale;           // [K] or [P, K] AdaLN scale (norm only)
  const void* shift;           // [K] or [P, K] AdaLN shift (norm only)
  int gamma_dtype, scale_dtype, shift_dtype;
  const int32_t* row_map;      // [rows] modulation table index, or null
  const int8_t* signs;         // [K] +-1 Hadamard signs, or null (all +1)
  int64_t rows, K;
  int norm;                    // NormKind
  float eps;
  int round_output;            // round the modulated value through the input dtype
  int rms_quant;               // RmsQuant; gamma is then an fp32 [K] vector, no scale / shift
  float inv_sqrt_block;        // fp32(1/sqrt(block)) for the rotation
  int warps;                   // warps per CTA (row_prep_warps)
  int vec_ok;                  // 16-byte vector loads / stores of rows are aligned
  int params_vec;              // gamma / scale / shift / gate rows allow 16-byte loads
  void* q;                     // [rows, K] int8 or E4M3 codes
  float* s;                    // [rows] per-row scales
  float* y;                    // [rows, K] fp32 rotated values (OUT_F32), or input-dtype rows (OUT_ROW)
  void* r_out;                 // [rows, K] updated residual (gated)
  unsigned int* status;        // device status word (bounded-wait errors)
};

// TMA descriptors of the row-streamed inputs (x and, gated, branch).
struct RowMaps {
  CUtensorMap x;
  CUtensorMap b;
  int valid;      // rows are staged through shared memory with these maps
  int box_rows;   // 128-byte box rows per TMA load
};

// Record `msg` as this thread's m5b_last_error() text and return `code`.
int set_last_error(int code, const char* msg);

int row_prep_warps(int64_t K, int block);
bool quant_rows_applicable(const RowPrepArgs& a, int x_dtype, int block, int out);
cudaError_t launch_quant_rows(const RowPrepArgs& a, const RowMaps& m, int x_dtype, int out,
                              cudaStream_t stream);
cudaError_t launch_row_prep(const RowPrepArgs& a, const RowMaps& maps, int x_dtype, int block,
                            int out, cudaStream_t stream);
// Register-streamed kernel of rows16_impl.cuh (16-bit rows of 1024..8192).
bool rows16_applicable(const RowPrepArgs& a, int x_dtype, int block, int out);
cudaError_t launch_rows16(const RowPrepArgs& a, int x_dtype, int block, int out,
                          cudaStream_t stream);

// MXINT8 block quantization of n = rows * K values (K % 32 == 0; mxint8.cu).
cudaError_t launch_mxint8(const void* x, int x_dtype, int64_t n, void* q, uint8_t* e,
                          cudaStream_t stream);

// FP32 GEMM mode: out = [rows, chunks, 3, ck] parts (hi, hi|lo, hi|lo) of
// each ck-column chunk of x [rows, k] (zero past k) for the three-product
// TF32 GEMM; lo_part (1 or 2) names the part holding x - hi (tf32split.cu).
cudaError_t launch_tf32_split(const float* x, int64_t rows, int64_t k, int64_t chunks, int64_t ck,
                              float* out, int lo_part, cudaStream_t stream);
// Internal GEMM mode of the split parts (never a user mode): TF32 operands.
constexpr int kModeTf32Parts = 0x100;
// K chunking of the FP32 mode: chunks of at most kFp32ChunkK columns (a
// multiple of 4), each one TF32 GEMM over its 3 x CK split columns whose
// result is added to the previous chunks' with one IEEE add (the tensor
// core's FP32 accumulator loses up to about half an ulp per MMA step, so its
// error grows with K; chunks bound it).
constexpr long long kFp32ChunkK = 2048;
inline long long fp32_chunks(long long k) {
  const long long k4 = (k + 3) / 4 * 4;
  return (k4 + kFp32ChunkK - 1) / kFp32ChunkK;
}
inline long long fp32_chunk_k(long long k) {  // CK: columns per chunk
  const long long k4 = (k + 3) / 4 * 4, s = fp32_chunks(k);
  return ((k4 + s - 1) / s + 3) / 4 * 4;
}
// Bytes of one split operand ([rows, S chunks, 3 parts, CK] fp32, 256-byte rounded).
inline long long fp32_split_bytes(long long rows, long long k) {
  return (rows * fp32_chunks(k) * 3 * fp32_chunk_k(k) * 4 + 255) / 256 * 256;
}

// Staged comparators (staged.cu).
struct GatedAddArgs {
  const void* residual;        // [rows, K]
  const void* branch;          // [rows, K], the residual's dtype
  const void* gate;            // [K] or [P, K]
  int gate_dtype;
  const int32_t* gate_row_map; // [rows] gate table index, or null
  int64_t rows, K;
  int vec_ok;                  // K % 8 == 0 and every pointer 16-byte aligned
  void* out;                   // [rows, K] updated residual, the residual's dtype
};
cudaError_t launch_gated_add(const GatedAddArgs& a, int x_dtype, cudaStream_t stream);

struct QkNormArgs {
  const void* projected;       // [M, N] bf16, N % 128 == 0, 16-byte aligned
  int64_t M, N;
  const void* gamma;           // [128] bf16
  const void* cos;             // [M, rope_half] bf16
  const void* sin;             // [M, rope_half] bf16
  int rope_half;
  float eps;
  int fast;                    // rope_half % 8 == 0 and 16-byte aligned tables
  void* out;                   // [N / 128, M, 128] bf16, 16-byte aligned
};
cudaError_t launch_qk_norm_rope(const QkNormArgs& a, cudaStream_t stream);

// GEMM epilogues.  C[m, n] for the plain epilogues, [N/128, M, 128] for QK.
enum Epilogue : int {
  EPI_PLAIN = 0,       // out = acc (float GEMM) or (acc * sa[m]) * sb[n] (quantized)
  EPI_BIAS_VEC = 1,    // ... + bias[n]
  EPI_BIAS_TABLE = 2,  // ... + bias[bias_row_map[m], n]
  EPI_GATE_VEC = 3,    // out = R[m, n] + bf16(branch) * gate[n]
  EPI_GATE_TABLE = 4,  // out = R[m, n] + bf16(branch) * gate[gate_row_map[m], n]
  EPI_QK = 5,          // bf16 branch -> per-head RMSNorm * gamma -> split-half RoPE
  EPI_ADD_ROWS = 6,    // ... + bias[m, n]: an fp32 [M, N] partial (the FP32 mode's K chunks;
                       // plain loads, so bias may be the output itself)
};

struct GemmArgs {
  int M, N, K;
  int kind;                   // MmaKind
  int epi;                    // Epilogue
  int quantized;              // apply a_scales / b_scales
  const float* a_scales;      // [M]
  const float* b_scales;      // [N]
  int sb_vec;                 // b_scales 16-byte aligned: whole chunks load as float4
  void* out;                  // output
  int out_dtype;              // DT_BF16 / DT_F16 / DT_F32 (plain epilogues)
  const float* bias;          // [N] or [P, N]
  const int32_t* bias_row_map;
  const void* residual;       // [M, N] bf16
  const void* gate;           // [N] or [P, N] bf16
  const int32_t* gate_row_map;
  const void* gamma;          // [128] bf16 (QK)
  const void* cos;            // [M, R] bf16 (QK)
  const void* sin;            // [M, R] bf16 (QK)
  int rope_half;
  int qk_fast;                // QK: rope_half % 8 == 0 and 16-byte aligned tables (vector path)
  int grouped;                // QK: W rows are [head, stream (Q, K, V), 128]; three outputs
  const void* gamma_k;        // [128] bf16 K-stream gamma (grouped)
  void* out_k;                // grouped: K output [H, M, 128] bf16
  void* out_v;                // grouped: V output [H, M, 128] bf16 (projection only)
  int tma_store;              // plain / bias / gate epilogues: 16-bit output leaves through
                              // the output tensor map (32 x 32 boxes, 64-byte swizzle)
  // Column-parallel all-gather (tma_store path, bf16): this rank's N columns
  // are columns [col_off, col_off + N) of [M, ldo] outputs, written to the
  // local output (tensor map) and to every peer rank's output (peer_out,
  // NVLink peer stores).
  int col_off;
  int64_t ldo;
  int n_peers;
  void* peer_out[7];
  float eps;
  int num_m_blocks, num_n_blocks, num_k_blocks;
  int group_m;
  // Work units: units [0, num_full) are whole tiles; when a CTA-pair launch's
  // last wave would be at most half full, the remaining tiles are split into
  // two N-halves each (units [num_full, num_units)), which evens out the wave.
  int num_full;
  int num_units;
  int pdl;                    // launch with programmatic stream serialization
  // Split-K schedule (INT8 CTA-pair GEMMs whose tiles fill at most half of
  // the GPU's CTA pairs, see gemm.cu): CTA pair u works on tile u % sk_tiles
  // over the k-blocks of split u / sk_tiles (sk_splits equal K ranges); the
  // last pair of a tile to finish adds the others' INT32 partial
  // accumulators (sk_part) to its own.  sk_ctr holds two counters per (tile,
  // CTA of the pair): arrival tickets and finished partial stores; they start
  // at zero and the finishing pair resets them, so they are zero again after
  // every launch.
  int sk;                     // 1: split-K schedule
  // 1: cluster split-K -- the launch is clusters of four CTAs (two pairs),
  // one cluster per tile, S = 2; the second pair's partial sums move into
  // the first pair's shared memory by a bulk copy (no workspace, no tickets)
  int sk_cluster;
  int sk_splits;              // S >= 2 pairs per tile
  int sk_tiles;               // T tiles; the launch has T * S CTA pairs
  int* sk_ctr;                // [tiles][2 CTAs][ticket, done]
  uint4* sk_part;             // [T * S pairs][2 CTAs][128 x 256 INT32 partials]
  unsigned int* status;       // device status word (bounded-wait errors)
};

// Split-K workspace for a GPU with `pairs` CTA pairs: the partial
// accumulators of every pair (128 x 256 INT32 per CTA) and the counters of up
// to `pairs` tiles.
constexpr int kSplitKMaxSplits = 4;
constexpr int kSplitKMinBlocks = 8;        // k-blocks per split, at least
inline long long splitk_part_bytes(int pairs) { return (long long)pairs * 2 * 128 * 256 * 4; }
inline long long splitk_workspace_bytes(int pairs) {
  return splitk_part_bytes(pairs) + (long long)pairs * 2 * 2 * (long long)sizeof(int);
}

// `to`: the Q/K output map (3D {128, M, N/128} bf16, boxes {64, 32, 1}, 128-byte
// swizzle), or with g.tma_store the [M, N] output map of the other epilogues
// (2D {N, M} bf16 / fp16, boxes {32, 32}, 64-byte swizzle).
// `to_k`, `to_v`: the grouped Q/K/V path's K and V output maps (as `to`).
cudaError_t launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tb_half,
                        const CUtensorMap& to, const CUtensorMap& to_k, const CUtensorMap& to_v,
                        const GemmArgs& g, int bn, int grid, bool pair, cudaStream_t stream);
int gemm_block_n(const GemmArgs& g);

}  // namespace m5b
