// C-ABI entry points of libm5b200.so (declared in include/m5b200.h).
//
// This layer checks the operator contracts that can be checked from sizes
// and pointers, builds TMA descriptors, picks launch shapes and enqueues the
// kernels of prep.cu / gemm.cu on the caller's stream.  It never allocates
// device memory.
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "m5b200.h"
#include "m5b_internal.h"

using namespace m5b;

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_err[0] = '\0';
  return M5B_OK;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(M5B_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

// ---------------------------------------------------------------- device state
__device__ unsigned int g_status_word;

constexpr int kMaxDevices = 64;
std::mutex g_dev_mutex;
unsigned int* g_status_ptr[kMaxDevices] = {};
int g_num_sms[kMaxDevices] = {};

int device_state(unsigned int** status, int* sms) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(M5B_ECUDA, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_dev_mutex);
  if (!g_status_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_status_word);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status)");
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    g_num_sms[dev] = n;
    g_status_ptr[dev] = static_cast<unsigned int*>(p);
  }
  if (status) *status = g_status_ptr[dev];
  if (sms) *sms = g_num_sms[dev];
  return M5B_OK;
}

// ---------------------------------------------------------------- TMA maps
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return fail(M5B_ECUDA, "cuTensorMapEncodeTiled is unavailable");
  return M5B_OK;
}

// K-major [rows, k] operand, boxes of 128 bytes x box_rows, 128-byte swizzle.
int make_kmajor_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t k, int elem_bytes,
                    int box_rows, int64_t ld) {
  const CUtensorMapDataType dt = elem_bytes == 1   ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                 : elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                   : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>((ld > 0 ? ld : k) * elem_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / elem_bytes), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(M5B_ECUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return M5B_OK;
}

// ---------------------------------------------------------------- helpers
bool float_dtype(int dt) { return dt == M5B_F32 || dt == M5B_F16 || dt == M5B_BF16; }
int dtype_bytes(int dt) { return dt == M5B_F32 ? 4 : (dt == M5B_I8 || dt == M5B_U8) ? 1 : 2; }
bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_block(int block, int64_t k) {
  if (block <= 0 || (block & (block - 1)))
    return fail(M5B_EINVAL, "block_size must be a positive integer power of two");
  if (block < 32 || block > 1024)
    return fail(M5B_EUNSUPPORTED, "supported block sizes are powers of two from 32 through 1024");
  if (k % block)
    return fail(M5B_EUNSUPPORTED, "K must be divisible by block_size; padding is not implicit");
  return M5B_OK;
}

int check_rows(int64_t rows, int64_t k) {
  if (rows <= 0 || k <= 0) return fail(M5B_EINVAL, "input must have nonempty shape [rows, K]");
  if (rows > 0x7fffffffLL) return fail(M5B_EUNSUPPORTED, "rows exceed the launch grid limit");
  return M5B_OK;
}

// 3D view {E, K/E, rows} of a row-major [rows, K] input (E = 128 / elem_bytes
// elements per 128-byte box row), loaded whole rows at a time with the
// 128-byte swizzle.  Returns false when the rows cannot be staged this way.
bool make_row_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t k, int eb,
                  int* box_rows) {
  if (!ptr || !aligned(ptr, 16) || (k % 64) != 0) return false;
  const int64_t e = 128 / eb;
  const int64_t nbr = k / e;  // box rows per input row
  const int64_t nb = nbr < 256 ? nbr : 256;
  if (nbr % nb) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(e), static_cast<cuuint64_t>(nbr),
                        static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {128, static_cast<cuuint64_t>(k * eb)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(e), static_cast<cuuint32_t>(nb), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt =
      eb == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16;
  CUresult r = g_encode(map, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  *box_rows = static_cast<int>(nb);
  return true;
}

int run_row_prep(RowPrepArgs& a, int x_dtype, int block, int out, void* stream) {
  a.warps = row_prep_warps(a.K, block);
  if (a.warps > 16)
    return fail(M5B_EUNSUPPORTED, "row width K=%lld exceeds the register-resident limit (32768)",
                static_cast<long long>(a.K));
  a.inv_sqrt_block = block > 0 ? static_cast<float>(1.0 / std::sqrt(static_cast<double>(block)))
                               : 1.0f;
  const bool vec = (a.K % 8) == 0 && aligned(a.x, 16) && (!a.branch || aligned(a.branch, 16)) &&
                   (!a.r_out || aligned(a.r_out, 16)) && (!a.q || aligned(a.q, 16)) &&
                   (!a.y || aligned(a.y, 16));
  a.vec_ok = vec ? 1 : 0;
  const bool pvec = (a.K % 8) == 0 && (!a.gamma || aligned(a.gamma, 16)) &&
                    (!a.scale || aligned(a.scale, 16)) && (!a.shift || aligned(a.shift, 16)) &&
                    (!a.gate || aligned(a.gate, 16)) && (!a.signs || aligned(a.signs, 16));
  a.params_vec = pvec ? 1 : 0;
  unsigned int* status = nullptr;
  int rc = device_state(&status, nullptr);
  if (rc) return rc;
  a.status = status;
  RowMaps maps{};
  rc = get_encode();
  if (rc) return rc;
  const int eb = dtype_bytes(x_dtype);
  int box_rows = 0, box_rows_b = 0;
  bool staged = vec && make_row_map(&maps.x, a.x, a.rows, a.K, eb, &box_rows);
  if (staged && a.branch) staged = make_row_map(&maps.b, a.branch, a.rows, a.K, eb, &box_rows_b);
  maps.valid = staged ? 1 : 0;
  maps.box_rows = box_rows;
  cudaError_t e = launch_row_prep(a, maps, x_dtype, block, out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "row preparation launch");
  return ok();
}

int prep_common(RowPrepArgs& a, const void* x, int x_dtype, int64_t rows, int64_t k) {
  int rc = check_rows(rows, k);
  if (rc) return rc;
  if (!float_dtype(x_dtype)) return fail(M5B_EINVAL, "input dtype must be float16, bfloat16 or float32");
  if (!x) return fail(M5B_EINVAL, "input pointer is NULL");
  a = RowPrepArgs{};
  a.x = x;
  a.rows = rows;
  a.K = k;
  return M5B_OK;
}

int out_kind(int mode) {
  if (mode == M5B_MODE_INT8) return OUT_INT8;
  if (mode == M5B_MODE_FP8) return OUT_E4M3;
  return -1;
}

int norm_setup(RowPrepArgs& a, const void* gamma, int gamma_dtype, const void* scale,
               int scale_dtype, const void* shift, int shift_dtype, const int32_t* row_map,
               int64_t table_rows, int norm, float epsilon, int round_output) {
  if (norm != M5B_NORM_RMS && norm != M5B_NORM_LAYER)
    return fail(M5B_EINVAL, "norm must be 'rms' or 'layer'");
  if (!(epsilon > 0.0f) || !std::isfinite(epsilon))
    return fail(M5B_EINVAL, "epsilon must be a positive finite real scalar");
  if (!gamma || !scale || !shift) return fail(M5B_EINVAL, "gamma, scale and shift are required");
  if (!float_dtype(gamma_dtype) || !float_dtype(scale_dtype) || !float_dtype(shift_dtype))
    return fail(M5B_EINVAL, "gamma, scale and shift must have floating dtype");
  if (row_map && table_rows <= 0)
    return fail(M5B_EINVAL, "mapped scale and shift must have matching nonempty shape [P,K]");
  a.gamma = gamma;
  a.scale = scale;
  a.shift = shift;
  a.gamma_dtype = gamma_dtype;
  a.scale_dtype = scale_dtype;
  a.shift_dtype = shift_dtype;
  a.row_map = row_map;
  a.norm = norm == M5B_NORM_RMS ? NORM_RMS : NORM_LAYER;
  a.eps = epsilon;
  a.round_output = round_output ? 1 : 0;
  return M5B_OK;
}

}  // namespace

int m5b::set_last_error(int code, const char* msg) { return fail(code, "%s", msg); }

extern "C" {

int m5b_version(void) { return 100; }

const char* m5b_last_error(void) { return g_err; }

int m5b_device_status(unsigned int* status_out, int clear) {
  unsigned int* p = nullptr;
  int rc = device_state(&p, nullptr);
  if (rc) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  unsigned int v = 0;
  e = cudaMemcpy(&v, p, sizeof(v), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device status word");
  if (clear) {
    e = cudaMemset(p, 0, sizeof(unsigned int));
    if (e != cudaSuccess) return cuda_fail(e, "clearing the device status word");
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  }
  if (status_out) *status_out = v;
  return ok();
}

int m5b_quantize(const void* x, int x_dtype, int64_t rows, int64_t k, int mode, void* q,
                 float* scales, void* stream) {
  RowPrepArgs a;
  int rc = prep_common(a, x, x_dtype, rows, k);
  if (rc) return rc;
  const int out = out_kind(mode);
  if (out < 0) return fail(M5B_EUNSUPPORTED, "quantize supports int8 and fp8 (E4M3)");
  if (!q || !scales) return fail(M5B_EINVAL, "output pointers are NULL");
  a.q = q;
  a.s = scales;
  return run_row_prep(a, x_dtype, 0, out, stream);
}

int m5b_quantize_mxint8(const void* x, int x_dtype, int64_t rows, int64_t k, int8_t* q,
                        uint8_t* scale_bytes, void* stream) {
  int rc = check_rows(rows, k);
  if (rc) return rc;
  if (k % 32) return fail(M5B_EINVAL, "MXINT8 requires K divisible by 32");
  if (!float_dtype(x_dtype)) return fail(M5B_EINVAL, "input dtype must be float16, bfloat16 or float32");
  if (!x || !q || !scale_bytes) return fail(M5B_EINVAL, "input or output pointer is NULL");
  if (!aligned(x, 16) || !aligned(q, 8))
    return fail(M5B_EINVAL, "input must be 16-byte and codes 8-byte aligned");
  if (rows > (int64_t(1) << 40) / k) return fail(M5B_EUNSUPPORTED, "tensor too large");
  cudaError_t e = launch_mxint8(x, x_dtype, rows * k, q, scale_bytes,
                                static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "MXINT8 quantization launch");
  return ok();
}

int m5b_rotate(const void* x, int x_dtype, int64_t rows, int64_t k, int block_size,
               const int8_t* signs, float* y, void* stream) {
  RowPrepArgs a;
  int rc = prep_common(a, x, x_dtype, rows, k);
  if (rc) return rc;
  rc = check_block(block_size, k);
  if (rc) return rc;
  if (!y) return fail(M5B_EINVAL, "output pointer is NULL");
  a.signs = signs;
  a.y = y;
  return run_row_prep(a, x_dtype, block_size, OUT_F32, stream);
}

int m5b_hadamard_quantize(const void* x, int x_dtype, int64_t rows, int64_t k, int block_size,
                          const int8_t* signs, int mode, void* q, float* scales, void* stream) {
  RowPrepArgs a;
  int rc = prep_common(a, x, x_dtype, rows, k);
  if (rc) return rc;
  rc = check_block(block_size, k);
  if (rc) return rc;
  const int out = out_kind(mode);
  if (out < 0) return fail(M5B_EUNSUPPORTED, "quantize supports int8 and fp8 (E4M3)");
  if (!q || !scales) return fail(M5B_EINVAL, "output pointers are NULL");
  a.signs = signs;
  a.q = q;
  a.s = scales;
  return run_row_prep(a, x_dtype, block_size, out, stream);
}

int m5b_fused_norm_hadamard_quantize(const void* x, int x_dtype, int64_t rows, int64_t k,
                                     const void* gamma, int gamma_dtype, const void* scale,
                                     int scale_dtype, const void* shift, int shift_dtype,
                                     const int32_t* row_map, int64_t table_rows,
                                     const int8_t* signs, int block_size, int norm,
                                     float epsilon, int round_output, int mode, void* q,
                                     float* scales, void* stream) {
  RowPrepArgs a;
  int rc = prep_common(a, x, x_dtype, rows, k);
  if (rc) return rc;
  rc = norm_setup(a, gamma, gamma_dtype, scale, scale_dtype, shift, shift_dtype, row_map,
                  table_rows, norm, epsilon, round_output);
  if (rc) return rc;
  rc = check_block(block_size, k);
  if (rc) return rc;
  const int out = out_kind(mode);
  if (out < 0) return fail(M5B_EUNSUPPORTED, "the fused preparation emits int8 or fp8 (E4M3)");
  if (!q || !scales) return fail(M5B_EINVAL, "output pointers are NULL");
  a.signs = signs;
  a.q = q;
  a.s = scales;
  return run_row_prep(a, x_dtype, block_size, out, stream);
}

int m5b_fused_gated_residual_norm_hadamard_quantize(
    const void* residual, const void* branch, int x_dtype, int64_t rows, int64_t k,
    const void* gate, int gate_dtype, const int32_t* gate_row_map, int64_t gate_rows,
    const void* gamma, int gamma_dtype, const void* scale, int scale_dtype, const void* shift,
    int shift_dtype, const int32_t* row_map, int64_t table_rows, const int8_t* signs,
    int block_size, int norm, float epsilon, int round_output, int mode, void* q, float* scales,
    void* residual_out, void* stream) {
  RowPrepArgs a;
  int rc = prep_common(a, residual, x_dtype, rows, k);
  if (rc) return rc;
  if (!branch || !gate || !residual_out)
    return fail(M5B_EINVAL, "branch, gate and residual_out are required");
  if (!float_dtype(gate_dtype)) return fail(M5B_EINVAL, "gate must have floating dtype");
  if (gate_row_map && gate_rows <= 0)
    return fail(M5B_EINVAL, "mapped gate must have nonempty shape [P,K]");
  rc = norm_setup(a, gamma, gamma_dtype, scale, scale_dtype, shift, shift_dtype, row_map,
                  table_rows, norm, epsilon, round_output);
  if (rc) return rc;
  rc = check_block(block_size, k);
  if (rc) return rc;
  const int out = out_kind(mode);
  if (out < 0) return fail(M5B_EUNSUPPORTED, "the fused preparation emits int8 or fp8 (E4M3)");
  if (!q || !scales) return fail(M5B_EINVAL, "output pointers are NULL");
  a.branch = branch;
  a.gate = gate;
  a.gate_dtype = gate_dtype;
  a.gate_row_map = gate_row_map;
  a.signs = signs;
  a.q = q;
  a.s = scales;
  a.r_out = residual_out;
  return run_row_prep(a, x_dtype, block_size, out, stream);
}

int m5b_rms_quantize(const void* x, int x_dtype, int64_t rows, int64_t k, const float* gamma,
                     const int8_t* signs, int block_size, int fold_scale, float epsilon,
                     int8_t* q, float* scales, void* stream) {
  RowPrepArgs a;
  int rc = prep_common(a, x, x_dtype, rows, k);
  if (rc) return rc;
  if (!gamma) return fail(M5B_EINVAL, "gamma must be a float32 vector of length K");
  if (!signs) return fail(M5B_EINVAL, "signs must be an int8 vector of length K containing only +/-1");
  if (block_size != 1) {
    rc = check_block(block_size, k);
    if (rc) return rc;
  }
  if (fold_scale != 0 && fold_scale != 1) return fail(M5B_EINVAL, "fold_scale must be a boolean");
  if (!(epsilon > 0.0f) || !std::isfinite(epsilon))
    return fail(M5B_EINVAL, "epsilon must remain finite and positive in float32");
  if (!q || !scales) return fail(M5B_EINVAL, "output pointers are NULL");
  a.gamma = gamma;
  a.gamma_dtype = DT_F32;
  a.signs = signs;
  a.eps = epsilon;
  a.rms_quant = fold_scale ? RMSQ_FOLD : RMSQ_DIRECT;
  a.q = q;
  a.s = scales;
  return run_row_prep(a, x_dtype, block_size == 1 ? 0 : block_size, OUT_INT8, stream);
}

int m5b_unfused_norm(const void* x, int x_dtype, int64_t rows, int64_t k, const void* gamma,
                     int gamma_dtype, const void* scale, int scale_dtype, const void* shift,
                     int shift_dtype, const int32_t* row_map, int64_t table_rows, int norm,
                     float epsilon, int round_output, void* y, void* stream) {
  RowPrepArgs a;
  int rc = prep_common(a, x, x_dtype, rows, k);
  if (rc) return rc;
  rc = norm_setup(a, gamma, gamma_dtype, scale, scale_dtype, shift, shift_dtype, row_map,
                  table_rows, norm, epsilon, round_output);
  if (rc) return rc;
  if (!y) return fail(M5B_EINVAL, "output pointer is NULL");
  a.y = static_cast<float*>(y);
  // rounded rows of a 16-bit input leave in that dtype, everything else as fp32
  const int out = (round_output && x_dtype != M5B_F32) ? OUT_ROW : OUT_F32;
  return run_row_prep(a, x_dtype, 0, out, stream);
}

int m5b_gated_residual_add(const void* residual, const void* branch, int x_dtype, int64_t rows,
                           int64_t k, const void* gate, int gate_dtype,
                           const int32_t* gate_row_map, int64_t gate_rows, void* out,
                           void* stream) {
  int rc = check_rows(rows, k);
  if (rc) return rc;
  if (!float_dtype(x_dtype)) return fail(M5B_EINVAL, "residual must have floating dtype");
  if (!residual || !branch || !gate || !out)
    return fail(M5B_EINVAL, "residual, branch, gate and out are required");
  if (!float_dtype(gate_dtype)) return fail(M5B_EINVAL, "gate must have floating dtype");
  if (gate_row_map && gate_rows <= 0)
    return fail(M5B_EINVAL, "mapped gate must have nonempty shape [P,K]");
  GatedAddArgs g{};
  g.residual = residual;
  g.branch = branch;
  g.gate = gate;
  g.gate_dtype = gate_dtype;
  g.gate_row_map = gate_row_map;
  g.rows = rows;
  g.K = k;
  g.out = out;
  g.vec_ok = (k % 8) == 0 && aligned(residual, 16) && aligned(branch, 16) && aligned(gate, 16) &&
             aligned(out, 16);
  cudaError_t e = launch_gated_add(g, x_dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gated residual launch");
  return ok();
}

int m5b_qk_norm_rope(const void* projected, int64_t m, int64_t n, const void* gamma,
                     const void* cos, const void* sin, int rope_half, float epsilon, void* out,
                     void* stream) {
  if (m <= 0 || n <= 0 || n % 128)
    return fail(M5B_EINVAL, "projection must have nonempty [M,N] shape with whole 128-wide heads");
  if (m > 0x7fffffffLL || n > 0x7fffffffLL)
    return fail(M5B_EUNSUPPORTED, "matrix dimensions exceed 2^31-1");
  if (rope_half < 1 || rope_half > 64)
    return fail(M5B_EINVAL, "cos must have shape [M,rope_half] with rope_half in [1,64]");
  if (!(epsilon > 0.0f) || !std::isfinite(epsilon))
    return fail(M5B_EINVAL, "epsilon must be a positive finite real scalar");
  if (!projected || !gamma || !cos || !sin || !out)
    return fail(M5B_EINVAL, "projected, gamma, cos, sin and out are required");
  if (!aligned(projected, 16) || !aligned(out, 16))
    return fail(M5B_EINVAL, "projection and output base addresses must be 16-byte aligned");
  QkNormArgs q{};
  q.projected = projected;
  q.M = m;
  q.N = n;
  q.gamma = gamma;
  q.cos = cos;
  q.sin = sin;
  q.rope_half = rope_half;
  q.eps = epsilon;
  q.out = out;
  q.fast = rope_half % 8 == 0 && aligned(gamma, 16) && aligned(cos, 16) && aligned(sin, 16);
  cudaError_t e = launch_qk_norm_rope(q, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "Q/K normalization launch");
  return ok();
}

// A CTA pair (cta_group::2, 256 x 256 tiles) when the problem has at least
// one full pair tile of rows and more than 128 output columns.
static bool use_pair(int epi, int64_t m, int64_t n) {
  return m >= 256 && (epi == EPI_QK ? n >= 256 : n > 128);
}

// GEMM schedule of the calling host thread (m5b_gemm_set_schedule): split_k
// -1 = the library's rule, 0 = data-parallel, 2..kSplitKMaxSplits = that
// split-K factor where it applies; group_m 0 = the library's raster group,
// else M-blocks per group.
struct ScheduleOverride {
  int split_k = -1;
  int group_m = 0;
};
static thread_local ScheduleOverride tl_schedule;

// ld: row stride of A and B in elements (0: k).
static int gemm_common(GemmArgs& g, CUtensorMap& ta, CUtensorMap& tb, CUtensorMap& tbh,
                       const void* a, const void* b, int64_t m, int64_t n, int64_t k, int mode,
                       int bn, bool pair, int64_t ld = 0) {
  if (m <= 0 || n <= 0 || k <= 0) return fail(M5B_EINVAL, "A and B must be nonempty matrices");
  if (m > 0x7fffffffLL || n > 0x7fffffffLL || k > 0x7fffffffLL)
    return fail(M5B_EUNSUPPORTED, "matrix dimensions exceed 2^31-1");
  if (!a || !b) return fail(M5B_EINVAL, "operand pointer is NULL");
  int kind;
  switch (mode) {
    case M5B_MODE_INT8: kind = KIND_I8; break;
    case M5B_MODE_FP8: kind = KIND_F8; break;
    case M5B_MODE_BF16: kind = KIND_BF16; break;
    case M5B_MODE_FP16: kind = KIND_F16; break;
    case kModeTf32Parts: kind = KIND_TF32; break;  // the FP32 mode's split [., 3 K4] parts
    default: return fail(M5B_EUNSUPPORTED, "GEMM modes are int8, fp8, bf16, fp16 and fp32");
  }
  const int eb = kind == KIND_TF32 ? 4 : (kind == KIND_BF16 || kind == KIND_F16) ? 2 : 1;
  if (mode == M5B_MODE_FP8 && k % 128)
    return fail(M5B_EUNSUPPORTED,
                "FP8 requires K/row stride divisible by 128; padding is not implicit");
  if (mode == M5B_MODE_INT8 && k > 133144)
    return fail(M5B_EUNSUPPORTED, "INT32 worst-case overflow bound exceeded");
  if ((k * eb) % 16)
    return fail(M5B_EUNSUPPORTED, "row stride K*%d bytes must be a multiple of 16 for TMA", eb);
  if (!aligned(a, 16) || !aligned(b, 16))
    return fail(M5B_EINVAL, "operand base addresses must be 16-byte aligned");
  int rc = get_encode();
  if (rc) return rc;
  if (ld > 0 && (ld < k || (ld * eb) % 16)) return fail(M5B_EINVAL, "bad operand row stride");
  rc = make_kmajor_map(&ta, a, m, k, eb, 128, ld);
  if (rc) return rc;
  rc = make_kmajor_map(&tb, b, n, k, eb, pair ? bn / 2 : bn, ld);
  if (rc) return rc;
  tbh = tb;
  if (pair) {  // half-height B boxes for split tail tiles
    rc = make_kmajor_map(&tbh, b, n, k, eb, bn / 4, ld);
    if (rc) return rc;
  }
  g.M = static_cast<int>(m);
  g.N = static_cast<int>(n);
  g.K = static_cast<int>(k);
  g.kind = kind;
  const int k_elems = 128 / eb;
  const int tile_m = pair ? 256 : 128;
  g.num_m_blocks = static_cast<int>((m + tile_m - 1) / tile_m);
  g.num_n_blocks = static_cast<int>((n + bn - 1) / bn);
  g.num_k_blocks = static_cast<int>((k + k_elems - 1) / k_elems);
  // Grouped-M raster: consecutive tiles walk the M-blocks of a group before
  // the next N-block, so a group's A rows are re-read from L2 while B streams.
  // A group's A footprint is capped near 48 MB (a little over a third of L2).
  // M5B_GEMM_GROUP_M overrides the choice (tuning experiments).
  const int64_t a_block_bytes = int64_t(tile_m) * k * eb;
  int64_t group = (48ll << 20) / (a_block_bytes > 0 ? a_block_bytes : 1);
  if (const char* env = std::getenv("M5B_GEMM_GROUP_M")) group = std::atoi(env);
  if (tl_schedule.group_m > 0) group = tl_schedule.group_m;
  if (group < 1) group = 1;
  if (group > g.num_m_blocks) group = g.num_m_blocks;
  g.group_m = static_cast<int>(group);
  return M5B_OK;
}

// Row-major [m, n] 16-bit output as a 2D map {n, m}: 32 x 32 boxes, 64-byte swizzle.
static int output_map(CUtensorMap* map, void* out, int out_dtype, int64_t m, int64_t n) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(m)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(n) * 2};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      out_dtype == M5B_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = g_encode(map, dt, 2, out, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(M5B_ECUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return M5B_OK;
}

// Split-K factor of a CTA-pair GEMM with `tiles` 256 x 256 tiles of nkb
// k-blocks on `slots` CTA pairs, or 0 for the data-parallel schedule.  An
// INT8 GEMM whose tiles fill at most a quarter of the pairs (even as N-halves
// they would leave half of the GPU idle) runs every tile as S >= 2 pairs over
// equal K ranges, up to S = 4; INT32 partial sums add exactly, so the result
// is the data-parallel one bit for bit.  Larger GEMMs keep the data-parallel
// schedule with its N-halves: at 32 tiles on 74 pairs (512 rows of FFN-down)
// two pairs per full tile finish their MMAs at 22 us against 29 us for one
// pair per N-half, but moving a 128 KB partial through global memory and
// adding it costs ~14 us of tail (37.7 against 35.3 us per GEMM); at 16
// tiles (256 rows) four pairs per tile measured 33.8 against 35.4 us.
// M5B_GEMM_SPLITK=0 turns it off, =2 extends it to half-filling tile counts
// (tuning and tests).
// A factor set by m5b_gemm_set_schedule applies when all T x S units are
// resident at once (T x S <= slots) and every split keeps kSplitKMinBlocks
// k-blocks; otherwise the GEMM runs data-parallel.
static int splitk_factor(int tiles, int nkb, int slots) {
  if (tl_schedule.split_k == 0 || tl_schedule.split_k == 2) return 0;  // (2: cluster split-K)
  if (tl_schedule.split_k >= 3) {
    const int s = tl_schedule.split_k;
    if (tiles <= 0 || int64_t(tiles) * s > slots || nkb / s < kSplitKMinBlocks) return 0;
    return s;
  }
  int fill = 4;  // tiles fill at most 1/fill of the pairs
  if (const char* force = std::getenv("M5B_GEMM_SPLITK")) {
    if (force[0] == '0') return 0;
    if (force[0] == '2') fill = 2;  // also up to half of the pairs (tuning)
  }
  if (tiles <= 0 || fill * tiles > slots) return 0;
  int s = slots / tiles;
  if (s > kSplitKMaxSplits) s = kSplitKMaxSplits;
  while (s >= 2 && nkb / s < kSplitKMinBlocks) --s;
  return s >= 2 ? s : 0;
}

// Cluster split-K (two pairs per tile in one 4-CTA cluster, partial sums
// through shared memory, no workspace), on request (m5b_gemm_set_schedule
// split_k = 2): INT8 CTA-pair GEMMs whose 256 x 256 tiles fill at most half
// of the pairs, with >= kSplitKMinBlocks k-blocks per half.  Whole tiles on
// two pairs move 2/3 of the operand bytes of the 64 N-halves they replace at
// 512 rows of FFN-down, but measured the same step (44.5-45.0 against 44.6
// us; GEMM 41.4 against 42.4 us between events), so the library's own rule
// keeps the data-parallel halves there.
static bool cluster_splitk(int tiles, int nkb, int slots) {
  if (tl_schedule.split_k != 2) return false;
  return tiles > 0 && 2 * tiles <= slots && nkb / 2 >= kSplitKMinBlocks;
}

static int gemm_launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tbh,
                       GemmArgs& g, int bn, bool pair, void* stream,
                       const CUtensorMap* to = nullptr, const CUtensorMap* to_k = nullptr,
                       const CUtensorMap* to_v = nullptr, void* sk_ws = nullptr,
                       int64_t sk_ws_bytes = 0) {
  unsigned int* status = nullptr;
  int sms = 0;
  int rc = device_state(&status, &sms);
  if (rc) return rc;
  g.status = status;
  g.sb_vec = (g.b_scales && aligned(g.b_scales, 16)) ? 1 : 0;
  const int tiles = g.num_m_blocks * g.num_n_blocks;
  const int slots = pair ? sms / 2 : sms;  // persistent CTAs (pairs)
  g.num_full = tiles;
  g.num_units = tiles;
  g.sk = 0;
  g.sk_cluster = 0;
  const int rem = tiles % slots;
  if (pair && tiles > slots && rem > 0 && 2 * rem <= slots) {
    g.num_full = tiles - rem;
    g.num_units = g.num_full + 2 * rem;
  } else if (pair && 2 * tiles <= slots) {  // under half a wave: every tile as two N-halves
    g.num_full = 0;
    g.num_units = 2 * tiles;
  }
  int grid = (g.num_units < slots ? g.num_units : slots) * (pair ? 2 : 1);
  // Programmatic dependent launch: the GEMM's set-up (barriers, TMEM,
  // descriptor prefetch) overlaps the end of the previous kernel in the
  // stream; every read of operands, scales and epilogue inputs, and every
  // write, waits for that kernel to complete (grid_dependency_wait).  Measured
  // after the quantization: 512 rows x K16384 -> N4096 step 50.2 -> 47.8 us,
  // 4096 rows unchanged.  M5B_GEMM_PDL=0 turns it off (tuning).
  g.pdl = 1;
  if (const char* env = std::getenv("M5B_GEMM_PDL")) g.pdl = env[0] == '0' ? 0 : 1;
  if (pair && bn == 256 && g.kind == KIND_I8 && sk_ws &&
      sk_ws_bytes >= splitk_workspace_bytes(slots) && aligned(sk_ws, 256)) {
    const int splits = splitk_factor(tiles, g.num_k_blocks, slots);
    if (splits > 0) {
      g.sk = 1;
      g.sk_splits = splits;
      g.sk_tiles = tiles;
      g.sk_part = static_cast<uint4*>(sk_ws);
      g.sk_ctr = reinterpret_cast<int*>(static_cast<uint8_t*>(sk_ws) + splitk_part_bytes(slots));
      g.num_full = tiles;
      g.num_units = tiles;
      grid = 2 * tiles * splits;
    }
  }
  if (!g.sk && pair && bn == 256 && g.kind == KIND_I8 && g.n_peers == 0 &&
      cluster_splitk(tiles, g.num_k_blocks, slots)) {
    g.sk = 1;
    g.sk_cluster = 1;
    g.sk_splits = 2;
    g.sk_tiles = tiles;
    g.num_full = tiles;
    g.num_units = tiles;
    grid = 4 * tiles;  // clusters of two pairs, one per tile
  }
  const CUtensorMap& o = to ? *to : tbh;
  cudaError_t e = launch_gemm(ta, tb, tbh, o, to_k ? *to_k : o, to_v ? *to_v : o, g, bn, grid,
                              pair, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "GEMM launch");
  return ok();
}

int m5b_gemm_set_schedule(int split_k, int group_m) {
  if (split_k < -1 || split_k == 1 || split_k > kSplitKMaxSplits)
    return fail(M5B_EINVAL, "split_k must be -1 (library rule), 0 or 2..%d", kSplitKMaxSplits);
  if (group_m < 0) return fail(M5B_EINVAL, "group_m must be >= 0");
  tl_schedule.split_k = split_k;
  tl_schedule.group_m = group_m;
  return ok();
}

int64_t m5b_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k, int mode) {
  if (mode == M5B_MODE_FP32) {  // the split parts, and the chunks' running sum
    if (m <= 0 || n <= 0 || k <= 0 || m > 0x7fffffffLL || n > 0x7fffffffLL || k > 0x7fffffffLL)
      return 0;
    return fp32_split_bytes(m, k) + fp32_split_bytes(n, k) +
           (fp32_chunks(k) > 1 ? (m * n * 4 + 255) / 256 * 256 : 0);
  }
  if (mode != M5B_MODE_INT8 || m <= 0 || n <= 0 || k <= 0 || !use_pair(EPI_PLAIN, m, n))
    return 0;
  if (m > 0x7fffffffLL || n > 0x7fffffffLL || k > 0x7fffffffLL) return 0;
  int sms = 0;
  unsigned int* status = nullptr;
  if (device_state(&status, &sms) != M5B_OK || sms < 4) return 0;
  const int64_t tiles = ((m + 255) / 256) * ((n + 255) / 256);
  if (tiles > 0x7fffffffLL) return 0;
  const int splits =
      splitk_factor(static_cast<int>(tiles), static_cast<int>((k + 127) / 128), sms / 2);
  return splits > 0 ? splitk_workspace_bytes(sms / 2) : 0;
}

static int gemm_impl(const void* a, const void* b, int64_t m, int64_t n, int64_t k, int mode,
                     const float* a_scales, const float* b_scales, void* out, int out_dtype,
                     const float* bias, const int32_t* bias_row_map, int64_t bias_rows,
                     const void* residual, const void* gate, const int32_t* gate_row_map,
                     int64_t gate_rows, void* workspace, int64_t workspace_bytes, void* stream);

// FP32 operands (src/m5kernels/metal.py:158-269, mode "fp32"): both operands
// are split into TF32 parts in the workspace (tf32split.cu), then one TF32
// GEMM per K chunk of <= kFp32ChunkK columns forms A_hi B_hi + A_hi B_lo +
// A_lo B_hi over the chunk with FP32 accumulation, each chunk after the first
// adding the running fp32 result (EPI_ADD_ROWS) -- the accuracy of an FP32
// GEMM, relative error ~1e-5 at any K.
static int gemm_fp32(const void* a, const void* b, int64_t m, int64_t n, int64_t k,
                     const float* a_scales, const float* b_scales, void* out, int out_dtype,
                     const float* bias, const int32_t* bias_row_map, const void* residual,
                     const void* gate, const int32_t* gate_row_map, void* workspace,
                     int64_t workspace_bytes, void* stream) {
  if (m <= 0 || n <= 0 || k <= 0) return fail(M5B_EINVAL, "A and B must be nonempty matrices");
  if (m > 0x7fffffffLL || n > 0x7fffffffLL || k > 0x7fffffffLL / 3)
    return fail(M5B_EUNSUPPORTED, "matrix dimensions exceed 2^31-1");
  if (!a || !b) return fail(M5B_EINVAL, "operand pointer is NULL");
  if (a_scales || b_scales)
    return fail(M5B_EINVAL, "float GEMM modes do not accept quantization scales");
  if (residual || gate || gate_row_map)
    return fail(M5B_EUNSUPPORTED, "gated GEMM supports INT8 and BF16 only");
  if (bias || bias_row_map)
    return fail(M5B_EUNSUPPORTED, "optional GEMM bias currently supports INT8 only");
  if (out_dtype == M5B_I32)
    return fail(M5B_EUNSUPPORTED, "int32 accumulator output requires INT8 operands");
  if (out_dtype != M5B_BF16 && out_dtype != M5B_F16 && out_dtype != M5B_F32)
    return fail(M5B_EUNSUPPORTED, "output dtype must be bfloat16, float16 or float32");
  if (!out) return fail(M5B_EINVAL, "output pointer is NULL");
  if (!aligned(a, 4) || !aligned(b, 4) || !aligned(out, 4))
    return fail(M5B_EINVAL, "fp32 operands and output must be 4-byte aligned");
  const long long a_bytes = fp32_split_bytes(m, k), b_bytes = fp32_split_bytes(n, k);
  const long long chunks = fp32_chunks(k), ck = fp32_chunk_k(k);
  // running sum of the chunks: the output itself when it is fp32, else scratch
  const long long part_bytes =
      (chunks > 1 && out_dtype != M5B_F32) ? (m * n * 4 + 255) / 256 * 256 : 0;
  const long long need = a_bytes + b_bytes + part_bytes;
  if (!workspace || workspace_bytes < need)
    return fail(M5B_EINVAL,
                "the fp32 GEMM needs m5b_gemm_workspace_bytes(m, n, k, M5B_MODE_FP32) = %lld bytes "
                "of workspace (m5b_gemm_ex)", need);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  float* a3 = reinterpret_cast<float*>(ws);
  float* b3 = reinterpret_cast<float*>(ws + a_bytes);
  float* partial = part_bytes ? reinterpret_cast<float*>(ws + a_bytes + b_bytes)
                              : static_cast<float*>(out);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_tf32_split(static_cast<const float*>(a), m, k, chunks, ck, a3, 2, st);
  if (e == cudaSuccess) e = launch_tf32_split(static_cast<const float*>(b), n, k, chunks, ck, b3, 1, st);
  if (e != cudaSuccess) return cuda_fail(e, "fp32 operand split launch");
  for (long long c = 0; c < chunks; ++c) {
    const bool last = c + 1 == chunks;
    GemmArgs g{};
    g.epi = c == 0 ? EPI_PLAIN : EPI_ADD_ROWS;
    g.N = static_cast<int>(n);
    const int bn = gemm_block_n(g);
    const bool pair = use_pair(EPI_PLAIN, m, n);
    CUtensorMap ta, tb, tbh;
    int rc = gemm_common(g, ta, tb, tbh, a3 + c * 3 * ck, b3 + c * 3 * ck, m, n, 3 * ck,
                         kModeTf32Parts, bn, pair, 3 * chunks * ck);
    if (rc) return rc;
    g.quantized = 0;
    g.bias = c == 0 ? nullptr : partial;
    g.out = last ? out : partial;
    g.out_dtype = last ? out_dtype : M5B_F32;
    CUtensorMap to{};
    if (last && (out_dtype == M5B_BF16 || out_dtype == M5B_F16) && n % 8 == 0 &&
        aligned(out, 16)) {
      rc = output_map(&to, out, out_dtype, m, n);
      if (rc) return rc;
      g.tma_store = 1;
      g.ldo = n;
      rc = gemm_launch(ta, tb, tbh, g, bn, pair, stream, &to);
    } else {
      rc = gemm_launch(ta, tb, tbh, g, bn, pair, stream);
    }
    if (rc) return rc;
  }
  return M5B_OK;
}

static int gemm_impl(const void* a, const void* b, int64_t m, int64_t n, int64_t k, int mode,
                     const float* a_scales, const float* b_scales, void* out, int out_dtype,
                     const float* bias, const int32_t* bias_row_map, int64_t bias_rows,
                     const void* residual, const void* gate, const int32_t* gate_row_map,
                     int64_t gate_rows, void* workspace, int64_t workspace_bytes, void* stream) {
  if (workspace_bytes < 0 || (workspace_bytes > 0 && !workspace))
    return fail(M5B_EINVAL, "workspace pointer is NULL");
  if (workspace && !aligned(workspace, 256))
    return fail(M5B_EINVAL, "workspace must be 256-byte aligned");
  if (mode == M5B_MODE_FP32)  // split the operands first
    return gemm_fp32(a, b, m, n, k, a_scales, b_scales, out, out_dtype, bias, bias_row_map,
                     residual, gate, gate_row_map, workspace, workspace_bytes, stream);
  GemmArgs g{};
  g.epi = EPI_PLAIN;
  g.N = static_cast<int>(n);
  const int bn = gemm_block_n(g);
  const bool pair = use_pair(EPI_PLAIN, m, n);
  CUtensorMap ta, tb, tbh;
  int rc = gemm_common(g, ta, tb, tbh, a, b, m, n, k, mode, bn, pair);
  if (rc) return rc;
  if (out_dtype == M5B_I32) {
    // Raw INT32 accumulators: INT8 operands, no scales and no epilogue.
    if (mode != M5B_MODE_INT8)
      return fail(M5B_EUNSUPPORTED, "int32 accumulator output requires INT8 operands");
    if (a_scales || b_scales || bias || bias_row_map || residual || gate || gate_row_map)
      return fail(M5B_EINVAL, "int32 accumulator output takes no scales, bias or gate");
    if (!out) return fail(M5B_EINVAL, "output pointer is NULL");
    g.out = out;
    g.out_dtype = DT_I32;
    return gemm_launch(ta, tb, tbh, g, bn, pair, stream, nullptr, nullptr, nullptr, workspace,
                       workspace_bytes);
  }
  const bool quant = (mode == M5B_MODE_INT8 || mode == M5B_MODE_FP8);
  if (quant && (!a_scales || !b_scales)) return fail(M5B_EINVAL, "scales required");
  if (!quant && (a_scales || b_scales))
    return fail(M5B_EINVAL, "float GEMM modes do not accept quantization scales");
  if (!out) return fail(M5B_EINVAL, "output pointer is NULL");
  if (out_dtype != M5B_BF16 && out_dtype != M5B_F16 && out_dtype != M5B_F32)
    return fail(M5B_EUNSUPPORTED, "output dtype must be bfloat16, float16 or float32");
  g.quantized = quant ? 1 : 0;
  g.a_scales = a_scales;
  g.b_scales = b_scales;
  g.out = out;
  g.out_dtype = out_dtype;
  const bool gated = residual || gate || gate_row_map;
  if (gated) {
    if (!residual || !gate) return fail(M5B_EINVAL, "gated GEMM requires both residual and gate");
    if (mode != M5B_MODE_INT8 && mode != M5B_MODE_BF16)
      return fail(M5B_EUNSUPPORTED, "gated GEMM supports INT8 and BF16 only");
    if (out_dtype != M5B_BF16)
      return fail(M5B_EUNSUPPORTED, "gated GEMM requires explicit BF16 output_dtype");
    if (bias || bias_row_map)
      return fail(M5B_EUNSUPPORTED, "combining GEMM bias and gated residual is unsupported");
    if (gate_row_map && gate_rows <= 0)
      return fail(M5B_EINVAL, "mapped gate must have nonempty shape [P,N]");
    g.epi = gate_row_map ? EPI_GATE_TABLE : EPI_GATE_VEC;
    g.residual = residual;
    g.gate = gate;
    g.gate_row_map = gate_row_map;
  } else if (bias || bias_row_map) {
    if (!bias) return fail(M5B_EINVAL, "bias_row_map requires a bias table");
    if (mode != M5B_MODE_INT8)
      return fail(M5B_EUNSUPPORTED, "optional GEMM bias currently supports INT8 only");
    if (bias_row_map && bias_rows <= 0)
      return fail(M5B_EINVAL, "mapped bias must have nonempty shape [P,N]");
    g.epi = bias_row_map ? EPI_BIAS_TABLE : EPI_BIAS_VEC;
    g.bias = bias;
    g.bias_row_map = bias_row_map;
  }
  // 16-bit outputs leave through a tensor map: 32 x 32 boxes staged per
  // epilogue warp with the 64-byte swizzle; the map clips the M and N tails.
  CUtensorMap to{};
  if ((out_dtype == M5B_BF16 || out_dtype == M5B_F16) && n % 8 == 0 && aligned(out, 16)) {
    rc = output_map(&to, out, out_dtype, m, n);
    if (rc) return rc;
    g.tma_store = 1;
    g.ldo = n;
    return gemm_launch(ta, tb, tbh, g, bn, pair, stream, &to, nullptr, nullptr, workspace,
                       workspace_bytes);
  }
  return gemm_launch(ta, tb, tbh, g, bn, pair, stream, nullptr, nullptr, nullptr, workspace,
                     workspace_bytes);
}

int m5b_gemm(const void* a, const void* b, int64_t m, int64_t n, int64_t k, int mode,
             const float* a_scales, const float* b_scales, void* out, int out_dtype,
             const float* bias, const int32_t* bias_row_map, int64_t bias_rows,
             const void* residual, const void* gate, const int32_t* gate_row_map,
             int64_t gate_rows, void* stream) {
  return gemm_impl(a, b, m, n, k, mode, a_scales, b_scales, out, out_dtype, bias, bias_row_map,
                   bias_rows, residual, gate, gate_row_map, gate_rows, nullptr, 0, stream);
}

int m5b_gemm_ex(const void* a, const void* b, int64_t m, int64_t n, int64_t k, int mode,
                const float* a_scales, const float* b_scales, void* out, int out_dtype,
                const float* bias, const int32_t* bias_row_map, int64_t bias_rows,
                const void* residual, const void* gate, const int32_t* gate_row_map,
                int64_t gate_rows, void* workspace, int64_t workspace_bytes, void* stream) {
  return gemm_impl(a, b, m, n, k, mode, a_scales, b_scales, out, out_dtype, bias, bias_row_map,
                   bias_rows, residual, gate, gate_row_map, gate_rows, workspace, workspace_bytes,
                   stream);
}

int m5b_gemm_allgather(const void* a, const void* b, int64_t m, int64_t n, int64_t k, int mode,
                       const float* a_scales, const float* b_scales, void* out, int64_t n_total,
                       int64_t col_offset, void* const* peer_outs, int n_peers, void* stream) {
  if (mode != M5B_MODE_INT8 && mode != M5B_MODE_FP8 && mode != M5B_MODE_BF16)
    return fail(M5B_EUNSUPPORTED, "the all-gather GEMM supports int8, fp8 and bf16 operands");
  if (m <= 0 || n <= 0 || n_total <= 0) return fail(M5B_EINVAL, "A and B must be nonempty matrices");
  if (n % 32 || col_offset % 32 || col_offset < 0 || col_offset + n > n_total || n_total % 8)
    return fail(M5B_EUNSUPPORTED,
                "column shards must be multiples of 32 columns inside a row of n_total %% 8 == 0");
  if (n_total > 0x7fffffffLL) return fail(M5B_EUNSUPPORTED, "n_total exceeds 2^31-1");
  if (n_peers < 0 || n_peers > 7) return fail(M5B_EUNSUPPORTED, "at most 7 peer outputs (8 ranks)");
  if (n_peers > 0 && !peer_outs) return fail(M5B_EINVAL, "peer output pointers are NULL");
  if (!out || !aligned(out, 16)) return fail(M5B_EINVAL, "output base address must be 16-byte aligned");
  for (int q = 0; q < n_peers; ++q)
    if (!peer_outs[q] || !aligned(peer_outs[q], 16))
      return fail(M5B_EINVAL, "peer output base addresses must be 16-byte aligned");
  const bool quant = mode != M5B_MODE_BF16;
  if (quant && (!a_scales || !b_scales)) return fail(M5B_EINVAL, "scales required");
  if (!quant && (a_scales || b_scales))
    return fail(M5B_EINVAL, "float GEMM modes do not accept quantization scales");
  GemmArgs g{};
  g.epi = EPI_PLAIN;
  g.N = static_cast<int>(n);
  const int bn = gemm_block_n(g);
  const bool pair = use_pair(EPI_PLAIN, m, n);
  CUtensorMap ta, tb, tbh;
  int rc = gemm_common(g, ta, tb, tbh, a, b, m, n, k, mode, bn, pair);
  if (rc) return rc;
  g.quantized = quant ? 1 : 0;
  g.a_scales = a_scales;
  g.b_scales = b_scales;
  g.out = out;
  g.out_dtype = M5B_BF16;
  CUtensorMap to{};
  rc = output_map(&to, out, M5B_BF16, m, n_total);
  if (rc) return rc;
  g.tma_store = 1;
  g.ldo = n_total;
  g.col_off = static_cast<int>(col_offset);
  g.n_peers = n_peers;
  for (int q = 0; q < n_peers; ++q) g.peer_out[q] = peer_outs[q];
  return gemm_launch(ta, tb, tbh, g, bn, pair, stream, &to);
}

// ---------------------------------------------------------------- CUDA IPC
// Peer ranks' output buffers are mapped with CUDA IPC (no multicast object).
// A handle names the whole cudaMalloc allocation; offset locates the buffer
// inside it (caching allocators hand out sub-blocks of larger segments).
static PFN_cuMemGetAddressRange_v3020 g_addr_range = nullptr;
static std::once_flag g_addr_range_once;

int m5b_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return fail(M5B_EINVAL, "pointer arguments are NULL");
  std::call_once(g_addr_range_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_addr_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  });
  if (!g_addr_range) return fail(M5B_ECUDA, "cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = g_addr_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) return fail(M5B_ECUDA, "cuMemGetAddressRange failed (%d)", int(r));
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return ok();
}

int m5b_ipc_import(const void* handle, int64_t offset, void** ptr_out) {
  if (!handle || !ptr_out || offset < 0) return fail(M5B_EINVAL, "invalid IPC import arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  *ptr_out = static_cast<uint8_t*>(base) + offset;
  return ok();
}

int m5b_ipc_release(void* ptr, int64_t offset) {
  if (!ptr || offset < 0) return fail(M5B_EINVAL, "invalid IPC release arguments");
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return ok();
}

// Head-major output map [heads, M, 128] bf16 as a 3D {128, M, heads} map; boxes
// of 64 channels x 32 rows (one epilogue warp's rows), 128-byte swizzle; rows
// past M clipped.
static int head_major_map(CUtensorMap* map, void* out, int64_t m, int64_t heads) {
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(m), static_cast<cuuint64_t>(heads)};
  cuuint64_t strides[2] = {256, static_cast<cuuint64_t>(m) * 256};
  cuuint32_t box[3] = {64, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, out, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(M5B_ECUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return M5B_OK;
}

// Shared body of the Q/K and grouped Q/K/V projections.  n = projection
// columns (heads * 128, or heads * 3 * 128 grouped).
static int qk_projection(const void* a, const void* b, int64_t m, int64_t n, int64_t k, int mode,
                         const float* a_scales, const float* b_scales, const void* gamma,
                         const void* gamma_k, const void* cos, const void* sin, int rope_half,
                         float epsilon, void* out, void* out_k, void* out_v, bool grouped,
                         void* workspace, int64_t workspace_bytes, void* stream) {
  if (workspace_bytes < 0 || (workspace_bytes > 0 && !workspace))
    return fail(M5B_EINVAL, "workspace pointer is NULL");
  if (workspace && !aligned(workspace, 256))
    return fail(M5B_EINVAL, "workspace must be 256-byte aligned");
  if (mode != M5B_MODE_INT8 && mode != M5B_MODE_BF16)
    return fail(M5B_EUNSUPPORTED, "Q/K projection fusion supports INT8 or BF16 only");
  if (m <= 0 || n <= 0 || n % 128)
    return fail(M5B_EINVAL, "projection must have nonempty [M,N] shape with whole 128-wide heads");
  if (mode == M5B_MODE_INT8 && k > 131071)
    return fail(M5B_EUNSUPPORTED, "INT32 worst-case overflow bound exceeded for signed INT8");
  if (rope_half < 1 || rope_half > 64)
    return fail(M5B_EINVAL, "cos must have shape [M,rope_half] with rope_half in [1,64]");
  if (!(epsilon > 0.0f) || !std::isfinite(epsilon))
    return fail(M5B_EINVAL, "epsilon must be a positive finite real scalar");
  if (!gamma || !cos || !sin || !out) return fail(M5B_EINVAL, "gamma, cos, sin and out are required");
  if (grouped && (!gamma_k || !out_k || !out_v))
    return fail(M5B_EINVAL, "grouped Q/K/V requires gamma_k and the K and V outputs");
  const bool quant = mode == M5B_MODE_INT8;
  if (quant && (!a_scales || !b_scales))
    return fail(M5B_EINVAL, "INT8 requires float32 a_scales[M] and b_scales[N]");
  if (!quant && (a_scales || b_scales))
    return fail(M5B_EINVAL, "BF16 projection does not accept quantization scales");
  if (!aligned(out, 16) || (grouped && (!aligned(out_k, 16) || !aligned(out_v, 16))))
    return fail(M5B_EINVAL, "output base address must be 16-byte aligned");
  GemmArgs g{};
  g.epi = EPI_QK;
  const bool pair = use_pair(EPI_QK, m, n);
  const int bn = pair ? 256 : 128;  // one or two 128-wide column blocks per tile
  CUtensorMap ta, tb, tbh;
  int rc = gemm_common(g, ta, tb, tbh, a, b, m, n, k, mode, bn, pair);
  if (rc) return rc;
  g.quantized = quant ? 1 : 0;
  g.a_scales = a_scales;
  g.b_scales = b_scales;
  g.out = out;
  g.out_dtype = M5B_BF16;
  g.gamma = gamma;
  g.cos = cos;
  g.sin = sin;
  g.rope_half = rope_half;
  g.eps = epsilon;
  g.grouped = grouped ? 1 : 0;
  g.gamma_k = gamma_k;
  g.out_k = out_k;
  g.out_v = out_v;
  // Vector path with TMA head-block stores: channel pairs (a, a + R) in whole
  // 16-byte chunks and 16-byte aligned tables.
  g.qk_fast = rope_half % 8 == 0 && aligned(gamma, 16) && aligned(cos, 16) && aligned(sin, 16) &&
              (!grouped || aligned(gamma_k, 16));
  const int64_t heads = grouped ? n / 384 : n / 128;
  CUtensorMap to{}, to_k{}, to_v{};
  if (g.qk_fast) {
    rc = head_major_map(&to, out, m, heads);
    if (!rc && grouped) rc = head_major_map(&to_k, out_k, m, heads);
    if (!rc && grouped) rc = head_major_map(&to_v, out_v, m, heads);
    if (rc) return rc;
  }
  return gemm_launch(ta, tb, tbh, g, bn, pair, stream, &to, grouped ? &to_k : nullptr,
                     grouped ? &to_v : nullptr, workspace, workspace_bytes);
}

int m5b_projection_qk_rope(const void* a, const void* b, int64_t m, int64_t n, int64_t k,
                           int mode, const float* a_scales, const float* b_scales,
                           const void* gamma, const void* cos, const void* sin, int rope_half,
                           float epsilon, void* out, void* stream) {
  return qk_projection(a, b, m, n, k, mode, a_scales, b_scales, gamma, nullptr, cos, sin,
                       rope_half, epsilon, out, nullptr, nullptr, false, nullptr, 0, stream);
}

int m5b_projection_qk_rope_ex(const void* a, const void* b, int64_t m, int64_t n, int64_t k,
                              int mode, const float* a_scales, const float* b_scales,
                              const void* gamma, const void* cos, const void* sin, int rope_half,
                              float epsilon, void* out, void* workspace, int64_t workspace_bytes,
                              void* stream) {
  return qk_projection(a, b, m, n, k, mode, a_scales, b_scales, gamma, nullptr, cos, sin,
                       rope_half, epsilon, out, nullptr, nullptr, false, workspace,
                       workspace_bytes, stream);
}

int m5b_projection_qkv_rope(const void* a, const void* b, int64_t m, int64_t heads, int64_t k,
                            int mode, const float* a_scales, const float* b_scales,
                            const void* gamma_q, const void* gamma_k, const void* cos,
                            const void* sin, int rope_half, float epsilon, void* q_out,
                            void* k_out, void* v_out, void* stream) {
  if (heads <= 0 || heads > (int64_t(1) << 20))
    return fail(M5B_EINVAL, "heads must be a positive count of 128-wide heads");
  return qk_projection(a, b, m, heads * 384, k, mode, a_scales, b_scales, gamma_q, gamma_k, cos,
                       sin, rope_half, epsilon, q_out, k_out, v_out, true, nullptr, 0, stream);
}

int64_t m5b_linear_workspace_bytes(int64_t m, int64_t k) {
  if (m <= 0 || k <= 0) return 0;
  const int64_t codes = (m * k + 255) & ~int64_t(255);
  return codes + m * int64_t(sizeof(float));
}


static int linear_impl(const void* x, int x_dtype, int64_t m, int64_t k, int block_size,
                       const int8_t* signs, const void* wq, const float* w_scales, int64_t n,
                       int mode, void* out, int out_dtype, void* workspace,
                       int64_t workspace_bytes, void* gemm_workspace,
                       int64_t gemm_workspace_bytes, void* stream) {
  if (mode != M5B_MODE_INT8 && mode != M5B_MODE_FP8)
    return fail(M5B_EUNSUPPORTED, "the online projection supports int8 and fp8 (E4M3)");
  if (m <= 0 || k <= 0 || n <= 0) return fail(M5B_EINVAL, "A and B must be nonempty matrices");
  if (k % 16)
    return fail(M5B_EUNSUPPORTED, "the online projection needs K %% 16 == 0 (16-byte code rows)");
  const int64_t need = m5b_linear_workspace_bytes(m, k);
  if (!workspace || workspace_bytes < need)
    return fail(M5B_EINVAL, "workspace of %lld bytes required", static_cast<long long>(need));
  if (!aligned(workspace, 256)) return fail(M5B_EINVAL, "workspace must be 256-byte aligned");
  uint8_t* codes = static_cast<uint8_t*>(workspace);
  float* scales = reinterpret_cast<float*>(codes + ((m * k + 255) & ~int64_t(255)));
  int rc = block_size > 0
               ? m5b_hadamard_quantize(x, x_dtype, m, k, block_size, signs, mode, codes, scales,
                                       stream)
               : m5b_quantize(x, x_dtype, m, k, mode, codes, scales, stream);
  if (rc) return rc;
  return gemm_impl(codes, wq, m, n, k, mode, scales, w_scales, out, out_dtype, nullptr, nullptr, 0,
                   nullptr, nullptr, nullptr, 0, gemm_workspace, gemm_workspace_bytes, stream);
}

int m5b_linear(const void* x, int x_dtype, int64_t m, int64_t k, int block_size,
               const int8_t* signs, const void* wq, const float* w_scales, int64_t n, int mode,
               void* out, int out_dtype, void* workspace, int64_t workspace_bytes, void* stream) {
  return linear_impl(x, x_dtype, m, k, block_size, signs, wq, w_scales, n, mode, out, out_dtype,
                     workspace, workspace_bytes, nullptr, 0, stream);
}

int m5b_linear_ex(const void* x, int x_dtype, int64_t m, int64_t k, int block_size,
                  const int8_t* signs, const void* wq, const float* w_scales, int64_t n, int mode,
                  void* out, int out_dtype, void* workspace, int64_t workspace_bytes,
                  void* gemm_workspace, int64_t gemm_workspace_bytes, void* stream) {
  return linear_impl(x, x_dtype, m, k, block_size, signs, wq, w_scales, n, mode, out, out_dtype,
                     workspace, workspace_bytes, gemm_workspace, gemm_workspace_bytes, stream);
}

}  // extern "C"
