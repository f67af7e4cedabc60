/*
 * m5b200 — C ABI of the B200 (sm_100a) quantized linear-projection kernels.
 *
 * Each entry point replaces one operator contract of the reference project
 * (9Tempest/m5-max-kernels, Python + Metal).  The reference's operators are
 * Python functions in src/m5kernels/*.py that build Metal kernels through
 * MLX; the functions below take plain device pointers, sizes and a CUDA
 * stream instead, so any host language can bind them (ctypes, cgo, JNI ...).
 *
 * Conventions
 *   - All tensor pointers are CUDA device pointers, row-major and contiguous.
 *   - Outputs are preallocated by the caller; inputs are never written.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are
 *     asynchronous: they enqueue kernels and return.
 *   - Return value: M5B_OK, or an error code; m5b_last_error() then describes
 *     the failure (thread-local, valid until the next call on this thread).
 *       M5B_EINVAL       contract violation     (the reference raises ValueError)
 *       M5B_EUNSUPPORTED unsupported shape/mode (the reference raises NotImplementedError)
 *       M5B_ECUDA        CUDA runtime/driver error
 *   - Value preconditions (finite inputs, +-1 signs, table-index bounds) are
 *     the caller's, as in the reference; they are not checked here.
 *   - Device-side waits are bounded; a wait that gives up records a bit in a
 *     per-device status word readable with m5b_device_status().
 */
#ifndef M5B200_H
#define M5B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define M5B_API __attribute__((visibility("default")))
#else
#define M5B_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define M5B_OK 0
#define M5B_EINVAL 1
#define M5B_EUNSUPPORTED 2
#define M5B_ECUDA 3

/* element types */
#define M5B_F32 0
#define M5B_F16 1
#define M5B_BF16 2
#define M5B_I8 3
#define M5B_U8 4
#define M5B_I32 5 /* raw INT32 GEMM accumulators (m5b_gemm, INT8 mode only) */

/* quantization / GEMM modes */
#define M5B_MODE_INT8 0 /* symmetric INT8, scale = amax/127 (INT32 accumulation) */
#define M5B_MODE_FP8 1  /* OCP E4M3 codes (uint8 bits), scale = amax/448 (FP32 accumulation) */
#define M5B_MODE_BF16 2 /* bf16 operands, FP32 accumulation (GEMM only) */
#define M5B_MODE_FP16 3 /* fp16 operands, FP32 accumulation (GEMM only) */
#define M5B_MODE_FP32 4 /* fp32 operands, FP32 accuracy from three TF32 tensor-core products
                           (GEMM only; needs the m5b_gemm_ex workspace) */

/* normalizations */
#define M5B_NORM_RMS 1
#define M5B_NORM_LAYER 2

/* Library version (major * 10000 + minor * 100 + patch). */
M5B_API int m5b_version(void);

/* Description of the last error on this thread ("" if none). */
M5B_API const char* m5b_last_error(void);

/* Device status word of the current device: bit 0 producer wait, bit 1 MMA
 * wait, bit 2 epilogue wait, bit 3 drain wait, bit 4 split-K partial-sum
 * wait gave up.  Synchronizes the
 * device.  If clear != 0 the word is reset to zero afterwards. */
M5B_API int m5b_device_status(unsigned int* status_out, int clear);

/* Per-token symmetric quantization of x[rows, k] (bf16 / fp16 / fp32).
 * mode INT8: q int8, scale = amax/127, q = clip(rint(x/scale), +-127).
 * mode FP8 : q = E4M3 bits (RNE, saturating), scale = amax/448.
 * All-zero rows get scale 1.
 * Replaces src/m5kernels/metal.py:27-44 (quantize) with the arithmetic of
 * src/m5kernels/numerics.py:29-46 (quantize_reference). */
M5B_API int m5b_quantize(const void* x, int x_dtype, int64_t rows, int64_t k, int mode, void* q,
                 float* scales, void* stream);

/* MXINT8 quantization of x[rows, k] (bf16 / fp16 / fp32), k % 32 == 0: per
 * 32-element block along a row, peak = max|x|,
 *   e = clip(floor(log2(peak)) - 6, -127, 127)   (0 for an all-zero block),
 *   q = clip(rint(x / 2^e), +-127)  int8 [rows, k],
 *   scale_bytes[rows, k / 32] = e + 127           (E8M0),
 * so x ~= q * 2^e (the S1.6 /64 of OCP MXINT8 folded into the scale plane).
 * floor(log2(peak)) is the exact binary exponent of the peak.  x 16-byte
 * aligned, q 8-byte aligned.
 * Replaces src/m5kernels/metal.py:27-44 (quantize, mode "mxint8") with the
 * arithmetic of src/m5kernels/numerics.py:32-40 (quantize_reference). */
M5B_API int m5b_quantize_mxint8(const void* x, int x_dtype, int64_t rows, int64_t k, int8_t* q,
                                uint8_t* scale_bytes, void* stream);

/* FP32 signed block Hadamard rotation y = x D H (H normalized Sylvester,
 * blocks of block_size along k, block_size in {32..1024}, k % block_size == 0).
 * signs: int8[k] of +-1, or NULL for D = I.
 * Replaces src/m5kernels/hadamard.py:33-77 (rotate). */
M5B_API int m5b_rotate(const void* x, int x_dtype, int64_t rows, int64_t k, int block_size,
               const int8_t* signs, float* y, void* stream);

/* quantize(rotate(x)) in one pass, bit-identical to the two-step path.
 * Replaces the online preparation of src/m5kernels/hadamard_gemm.py:65-66. */
M5B_API int m5b_hadamard_quantize(const void* x, int x_dtype, int64_t rows, int64_t k, int block_size,
                          const int8_t* signs, int mode, void* q, float* scales, void* stream);

/* Fused normalization + AdaLN modulation + rotation + quantization:
 *   y = norm(x) * gamma * (1 + scale[map]) + shift[map]   (FP32)
 *   y = round_through(x_dtype, y)  if round_output
 *   q, s = quantize(y D H, mode)
 * norm M5B_NORM_RMS (mean of squares) or M5B_NORM_LAYER (centered, population
 * variance); epsilon inside the square root.  scale/shift are [k] vectors when
 * row_map == NULL, else [table_rows, k] tables indexed by row_map[rows].
 * Replaces src/m5kernels/norm_hadamard.py:122-176
 * (fused_norm_hadamard_quantize), extended with an E4M3 output mode. */
M5B_API int m5b_fused_norm_hadamard_quantize(const void* x, int x_dtype, int64_t rows, int64_t k,
                                     const void* gamma, int gamma_dtype, const void* scale,
                                     int scale_dtype, const void* shift, int shift_dtype,
                                     const int32_t* row_map, int64_t table_rows,
                                     const int8_t* signs, int block_size, int norm,
                                     float epsilon, int round_output, int mode, void* q,
                                     float* scales, void* stream);

/* As above, on the updated residual R' = cast(R + branch * gate[gate_map])
 * (one FP32 fused multiply-add, then RNE to x_dtype), which is also written
 * to residual_out.  gate is [k] when gate_row_map == NULL, else
 * [gate_rows, k].  Replaces src/m5kernels/norm_hadamard.py:198-265
 * (fused_gated_residual_norm_hadamard_quantize). */
M5B_API int m5b_fused_gated_residual_norm_hadamard_quantize(
    const void* residual, const void* branch, int x_dtype, int64_t rows, int64_t k,
    const void* gate, int gate_dtype, const int32_t* gate_row_map, int64_t gate_rows,
    const void* gamma, int gamma_dtype, const void* scale, int scale_dtype, const void* shift,
    int shift_dtype, const int32_t* row_map, int64_t table_rows, const int8_t* signs,
    int block_size, int norm, float epsilon, int round_output, int mode, void* q, float* scales,
    void* residual_out, void* stream);

/* RMS preparation with the inverse RMS folded into the INT8 row scale:
 *   r = 1/sqrt(sum(x^2)/k + eps)            (x the ORIGINAL row, FP32)
 *   fold_scale 1: u = (x * gamma) D H,  scale = (peak(u) * r) / 127
 *   fold_scale 0: u = ((x * r) * gamma) D H, scale = peak(u) / 127
 *   q = clip(rint((u / peak(u)) * 127), +-127); a zero row of u gets q = 0,
 *   scale 1.  No additive shift, no rounding to the input dtype in between.
 * gamma: fp32[k]; signs: int8[k] of +-1 (required); block_size 1 (no
 * rotation, any k) or a power of two from 32 through 1024 dividing k.
 * Replaces src/m5kernels/rms_quant.py:41-117 (rms_quantize) with the
 * semantics of rms_quant_reference.py:24-89. */
M5B_API int m5b_rms_quantize(const void* x, int x_dtype, int64_t rows, int64_t k,
                             const float* gamma, const int8_t* signs, int block_size,
                             int fold_scale, float epsilon, int8_t* q, float* scales,
                             void* stream);

/* Staged comparators: one stage of the fused kernels on its own, with the same
 * FP32 operations in the same order, so that a staged pipeline reproduces the
 * fused result bit for bit (fusion-gain baselines and staged == fused checks).
 *
 * m5b_unfused_norm: y = norm(x) * gamma * (1 + scale[map]) + shift[map] with
 * the statistics and modulation of m5b_fused_norm_hadamard_quantize, no
 * signs, rotation or quantization.  y is [rows, k] in x_dtype when
 * round_output != 0 (fp32 when x is fp32), else fp32.
 * Replaces src/m5kernels/norm_hadamard.py:321-348 (unfused_norm). */
M5B_API int m5b_unfused_norm(const void* x, int x_dtype, int64_t rows, int64_t k,
                             const void* gamma, int gamma_dtype, const void* scale,
                             int scale_dtype, const void* shift, int shift_dtype,
                             const int32_t* row_map, int64_t table_rows, int norm, float epsilon,
                             int round_output, void* y, void* stream);

/* m5b_gated_residual_add: out = cast(R + branch * gate[gate_map]) (one FP32
 * fused multiply-add, then RNE to x_dtype), the residual_out of
 * m5b_fused_gated_residual_norm_hadamard_quantize.  residual, branch and out
 * share x_dtype; gate is [k], or [gate_rows, k] with gate_row_map[rows].
 * Replaces src/m5kernels/norm_hadamard.py:280-300 (gated_residual_add). */
M5B_API int m5b_gated_residual_add(const void* residual, const void* branch, int x_dtype,
                                   int64_t rows, int64_t k, const void* gate, int gate_dtype,
                                   const int32_t* gate_row_map, int64_t gate_rows, void* out,
                                   void* stream);

/* m5b_qk_norm_rope: the Q/K post-processing of m5b_projection_qk_rope applied
 * to a stored bf16 projection [m, n] (n % 128 == 0): per (row, head)
 * r = 1/sqrt(mean(z^2) + eps), u = z * r * gamma, split-half RoPE on j < 2R,
 * out bf16 [n/128, m, 128].  projected and out 16-byte aligned.
 * Replaces src/m5kernels/qk_rope.py:185-203 (qk_norm_rope). */
M5B_API int m5b_qk_norm_rope(const void* projected, int64_t m, int64_t n, const void* gamma,
                             const void* cos, const void* sin, int rope_half, float epsilon,
                             void* out, void* stream);

/* C[m, n] = epilogue(A[m, k] . B[n, k]^T) on tcgen05 tensor cores.
 *   mode INT8: int8 operands, INT32 accumulation; FP8: E4M3 operands, FP32
 *   accumulation (k % 128 == 0); BF16 / FP16: FP32 accumulation.
 *   Quantized modes require a_scales[m], b_scales[n]:
 *       v = (float(acc) * a_scales[m]) * b_scales[n]
 *   bias (INT8 only): v += bias[n] (bias_row_map == NULL) or
 *       bias[bias_row_map[m], n] (bias is [bias_rows, n]).
 *   gated residual (INT8 / BF16, bf16 output): out = R[m, n] + bf16(v) * gate,
 *       gate [n] or [gate_rows, n] with gate_row_map.
 *   out_dtype: M5B_BF16, M5B_F16 or M5B_F32; M5B_I32 (INT8 mode, no scales,
 *       bias or gate) stores the raw INT32 accumulators.
 * Replaces src/m5kernels/metal.py:158-269 (gemm). */
M5B_API int m5b_gemm(const void* a, const void* b, int64_t m, int64_t n, int64_t k, int mode,
             const float* a_scales, const float* b_scales, void* out, int out_dtype,
             const float* bias, const int32_t* bias_row_map, int64_t bias_rows,
             const void* residual, const void* gate, const int32_t* gate_row_map,
             int64_t gate_rows, void* stream);

/* Workspace bytes that let m5b_gemm_ex (and m5b_linear_ex,
 * m5b_projection_qk_rope_ex) run an m x n x k GEMM of `mode` on the current
 * device with the split-K schedule, or 0 when that shape keeps the
 * data-parallel schedule.  Split-K is taken by INT8 GEMMs whose 256 x 256
 * tiles would fill at most a quarter of the GPU's CTA pairs (very few rows
 * and columns): every tile runs on S >= 2 CTA pairs over equal K ranges, and
 * the last of them to finish adds the others' INT32 partial sums (exact) --
 * outputs are bit-identical to the data-parallel schedule.
 * The size depends only on the device's SM count (about 0.25 MB per CTA
 * pair).  M5B_MODE_FP32 always needs a workspace: the split operands
 * [m, 3 K4] and [n, 3 K4] fp32 (K4 = K rounded up to 4), 12 (m + n) K4 bytes
 * rounded to 256-byte parts.  It is scratch, left overwritten: never share it
 * with the split-K calls, whose workspace must stay zeroed. */
M5B_API int64_t m5b_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k, int mode);

/* GEMM schedule for the calling host thread, the B200 counterpart of the
 * reference's per-call Metal tile (src/m5kernels/metal.py:158-166 `tile`,
 * swept by `m5bench tune`, src/m5kernels/cli.py:66-151).  It changes how
 * the work is scheduled, never the result (outputs are bit-identical under
 * every schedule).  split_k: -1 the library's rule, 0 data-parallel,
 * 2 two CTA pairs per 256 x 256 tile in one 4-CTA cluster, the second
 * pair's INT32 partial sums moved into the first pair's shared memory (no
 * workspace; tiles filling at most half of the pairs), 3..4 that many CTA
 * pairs per tile over equal K ranges through the workspace -- taken by INT8
 * CTA-pair GEMMs given one when all tiles x splits fit on the GPU at once;
 * every split keeps >= 8 k-blocks, else data-parallel.
 * group_m: 0 the library's raster, else M-blocks walked per N-block group.
 * Every GEMM entry point called later from this thread uses it (also
 * m5b_gemm_workspace_bytes) until (-1, 0) restores the defaults.  No
 * counterpart in the reference's C-level API: its tile is a call argument. */
M5B_API int m5b_gemm_set_schedule(int split_k, int group_m);

/* m5b_gemm with a workspace for the split-K schedule (NULL / 0: data-
 * parallel only, exactly m5b_gemm).  The workspace must be 256-byte aligned
 * and all zero before its first use (cudaMemset once after allocating it);
 * every call leaves it zeroed again.  Calls that overlap on the GPU must not
 * share a workspace.  After a nonzero m5b_device_status (a timed-out wait)
 * zero it again.  Same replacement as m5b_gemm. */
M5B_API int m5b_gemm_ex(const void* a, const void* b, int64_t m, int64_t n, int64_t k, int mode,
                        const float* a_scales, const float* b_scales, void* out, int out_dtype,
                        const float* bias, const int32_t* bias_row_map, int64_t bias_rows,
                        const void* residual, const void* gate, const int32_t* gate_row_map,
                        int64_t gate_rows, void* workspace, int64_t workspace_bytes,
                        void* stream);

/* Column-parallel projection with the all-gather fused into the epilogue.
 * This rank holds n output channels of W (b [n, k], b_scales [n]); its
 * result columns are columns [col_offset, col_offset + n) of the [m, n_total]
 * bf16 output that every rank holds.  Each output tile is stored to `out`
 * (this GPU) and to each of the n_peers buffers in peer_outs (the other
 * ranks' outputs, mapped into this process with m5b_ipc_import) with NVLink
 * peer stores, so after every rank's call has completed (order the ranks
 * with a stream-ordered barrier, e.g. a one-element NCCL all-reduce) every
 * output holds all n_total columns.  mode INT8 / FP8 (with scales) or BF16;
 * n % 32 == 0, col_offset % 32 == 0, n_total % 8 == 0, n_peers <= 7.
 * Replaces the optional column-parallel FFN-up variant's GEMM +
 * all_gather_into_tensor (the reference itself is
 * single-GPU: metal.py:158-269 per rank). */
M5B_API int m5b_gemm_allgather(const void* a, const void* b, int64_t m, int64_t n, int64_t k,
                               int mode, const float* a_scales, const float* b_scales, void* out,
                               int64_t n_total, int64_t col_offset, void* const* peer_outs,
                               int n_peers, void* stream);

/* CUDA IPC of an output buffer (plain peer mapping, no multicast object).
 * m5b_ipc_export writes the 64-byte handle of the allocation holding `ptr`
 * and ptr's byte offset inside it; m5b_ipc_import maps another process's
 * handle and returns the buffer's address in this process; m5b_ipc_release
 * unmaps it.  Helpers of m5b_gemm_allgather; no counterpart in the
 * reference. */
M5B_API int m5b_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out);
M5B_API int m5b_ipc_import(const void* handle, int64_t offset, void** ptr_out);
M5B_API int m5b_ipc_release(void* ptr, int64_t offset);

/* Workspace bytes m5b_linear needs for activations [m, k]: the per-token
 * codes (m * k bytes, 256-byte aligned) followed by the fp32 scales. */
M5B_API int64_t m5b_linear_workspace_bytes(int64_t m, int64_t k);

/* One call for the online projection y = gemm(quantize([rotate](x)), wq):
 *   codes, scales = quantize(x D H) (block_size > 0, signs as in m5b_rotate)
 *                 or quantize(x)     (block_size == 0)
 *   y[m, n] = (float(acc) * scales[m]) * w_scales[n] -> out_dtype (bf16/f16/f32)
 * x: [m, k] bf16 / fp16 / fp32; wq: [n, k] codes prepared offline with the
 * same mode (and rotation); k % 16 == 0 (mode FP8: k % 128 == 0).  The codes
 * and scales live in the caller's workspace (m5b_linear_workspace_bytes).
 * Replaces the reference's online stage quantize -> gemm
 * (src/m5kernels/engine.py:180-182, hadamard_gemm.py:65-69). */
M5B_API int m5b_linear(const void* x, int x_dtype, int64_t m, int64_t k, int block_size,
                       const int8_t* signs, const void* wq, const float* w_scales, int64_t n,
                       int mode, void* out, int out_dtype, void* workspace,
                       int64_t workspace_bytes, void* stream);

/* m5b_linear whose GEMM may take the split-K schedule: gemm_workspace
 * (m5b_gemm_workspace_bytes(m, n, k, mode) bytes, separate from the codes /
 * scales workspace) follows the rules of m5b_gemm_ex's workspace.  Same
 * replacement as m5b_linear. */
M5B_API int m5b_linear_ex(const void* x, int x_dtype, int64_t m, int64_t k, int block_size,
                          const int8_t* signs, const void* wq, const float* w_scales, int64_t n,
                          int mode, void* out, int out_dtype, void* workspace,
                          int64_t workspace_bytes, void* gemm_workspace,
                          int64_t gemm_workspace_bytes, void* stream);

/* m5b_linear for callers that cannot allocate device memory (a host whose
 * device memory is already committed to its own pool, a plugin host that
 * forbids extension allocations, a hot path that must not take cudaMalloc's
 * device synchronisation).  Same arguments and result as m5b_linear minus the
 * workspace: the codes and scales live in a fixed 64 MiB + 64 KiB device array
 * inside the library, reserved on every GPU that loads it.  Limits:
 * m * k <= 67,108,864 and m <= 16,384 (else M5B_EINVAL).  Calls share that
 * array: calls whose kernels overlap on the GPU race and must be ordered.
 * The first call on a device looks the array's address up (make it before
 * any stream capture); the address is tied to the device's CUDA context, and
 * the first call after a cudaDeviceReset looks it up again (also before any
 * capture).  Allocates nothing.  No counterpart in the reference. */
M5B_API int m5b_linear_noalloc(const void* x, int x_dtype, int64_t m, int64_t k, int block_size,
                               const int8_t* signs, const void* wq, const float* w_scales,
                               int64_t n, int mode, void* out, int out_dtype, void* stream);

/* Q or K projection with per-head RMSNorm and split-half RoPE, head-major:
 *   z = bf16(v)  (v as in m5b_gemm), per (row, head): r = 1/sqrt(mean(z^2) + eps)
 *   u_j = z_j * r * gamma_j; for j < R: (u_j, u_{j+R}) rotated by
 *   (cos, sin)[row, j]; channels >= 2R unrotated; out bf16 [n/128, m, 128].
 * gamma bf16[128]; cos, sin bf16[m, rope_half], 1 <= rope_half <= 64.
 * mode INT8 (with scales) or BF16 (without).
 * Replaces src/m5kernels/qk_rope.py:120-182 (projection_qk_rope). */
M5B_API int m5b_projection_qk_rope(const void* a, const void* b, int64_t m, int64_t n, int64_t k,
                           int mode, const float* a_scales, const float* b_scales,
                           const void* gamma, const void* cos, const void* sin, int rope_half,
                           float epsilon, void* out, void* stream);

/* m5b_projection_qk_rope with a workspace for the split-K schedule of its
 * INT8 GEMM (m5b_gemm_workspace_bytes(m, n, k, mode) bytes; rules as for
 * m5b_gemm_ex).  The finishing CTA pair of a split tile adds the INT32
 * partial sums before the BF16 projection, so RMS and RoPE see the same
 * values as without the split.  Same replacement as m5b_projection_qk_rope. */
M5B_API int m5b_projection_qk_rope_ex(const void* a, const void* b, int64_t m, int64_t n,
                                      int64_t k, int mode, const float* a_scales,
                                      const float* b_scales, const void* gamma, const void* cos,
                                      const void* sin, int rope_half, float epsilon, void* out,
                                      void* workspace, int64_t workspace_bytes, void* stream);

/* Grouped Q/K/V projection: b is [heads, 3, 128, k] (rows in [head, stream,
 * channel] order, streams Q, K, V), b_scales [heads * 384].  One GEMM; per
 * 128-column block, z = bf16(v) as in m5b_projection_qk_rope, then
 *   Q: RMSNorm with gamma_q + split-half RoPE -> q_out [heads, m, 128]
 *   K: RMSNorm with gamma_k + split-half RoPE -> k_out [heads, m, 128]
 *   V: z unchanged (no RMS, no RoPE)          -> v_out [heads, m, 128]
 * all bf16 head-major.  Replaces the native grouped QKV projection of the
 * reference's H3 integration (integrations/h3/qkv-candidate.md:30-43, the
 * h3_gpu_m5_grouped_qkv_linear_rope_int8 API; per-stream contract of
 * integrations/h3/qkv_reference.h:15-36, layout docs/qk-rope-fusion.md:12). */
M5B_API int m5b_projection_qkv_rope(const void* a, const void* b, int64_t m, int64_t heads,
                                    int64_t k, int mode, const float* a_scales,
                                    const float* b_scales, const void* gamma_q,
                                    const void* gamma_k, const void* cos, const void* sin,
                                    int rope_half, float epsilon, void* q_out, void* k_out,
                                    void* v_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* M5B200_H */
