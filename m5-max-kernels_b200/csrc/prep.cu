// Row-preparation dispatch: launch-shape rule and input-dtype switch.
// The kernel template lives in prep_impl.cuh; prep_{bf16,f16,f32}.cu hold its
// instantiations so they compile in parallel.
#include "common.cuh"
#include "m5b_internal.h"

namespace m5b {

cudaError_t launch_row_prep_bf16(const RowPrepArgs& a, const RowMaps& m, int block, int out,
                                 cudaStream_t stream);
cudaError_t launch_row_prep_f16(const RowPrepArgs& a, const RowMaps& m, int block, int out,
                                cudaStream_t stream);
cudaError_t launch_row_prep_f32(const RowPrepArgs& a, const RowMaps& m, int block, int out,
                                cudaStream_t stream);

// Warps per CTA for a row of width K: one thread per 64-element chunk, whole
// warps, so W = ceil(K / 2048).  The oracle uses the same rule (it fixes the
// reduction tree).
int row_prep_warps(int64_t K, int /*block*/) {
  const int64_t w = (K + 2047) / 2048;
  return w < 1 ? 1 : (w > 1024 ? 1024 : static_cast<int>(w));
}

cudaError_t launch_row_prep(const RowPrepArgs& a, const RowMaps& m, int x_dtype, int block,
                            int out, cudaStream_t stream) {
  // Plain per-token quantization needs no register-resident row: two
  // streaming passes (quant.cu) keep many more rows in flight per SM.
  if (quant_rows_applicable(a, x_dtype, block, out)) return launch_quant_rows(a, m, x_dtype, out, stream);
  // Rows of 1024..8192 16-bit elements: one row per CTA, 16 elements per
  // thread streamed through registers (rows16_impl.cuh).
  if (rows16_applicable(a, x_dtype, block, out)) return launch_rows16(a, x_dtype, block, out, stream);
  switch (x_dtype) {
    case DT_BF16: return launch_row_prep_bf16(a, m, block, out, stream);
    case DT_F16: return launch_row_prep_f16(a, m, block, out, stream);
    case DT_F32: return launch_row_prep_f32(a, m, block, out, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace m5b
