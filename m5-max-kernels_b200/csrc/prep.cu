// Row-preparation dispatch: launch-shape rule and input-dtype switch.
// The kernel template lives in prep_impl.cuh; prep_{bf16,f16,f32}.cu hold its
// instantiations so they compile in parallel.
#include "common.cuh"
#include "m5b_internal.h"

namespace m5b {

cudaError_t launch_row_prep_bf16(const RowPrepArgs& a, int block, int out, cudaStream_t stream);
cudaError_t launch_row_prep_f16(const RowPrepArgs& a, int block, int out, cudaStream_t stream);
cudaError_t launch_row_prep_f32(const RowPrepArgs& a, int block, int out, cudaStream_t stream);

constexpr int kMaxValuesPerThread = 64;  // must equal kMaxValues in prep_impl.cuh

// Warps per CTA for a row of width K: as few as possible (each thread keeps
// up to 64 FP32 values in registers).  The oracle uses the same rule.
int row_prep_warps(int64_t K, int block) {
  const int unit = block > 256 ? block : 256;
  const int vpu = unit / 256;
  const int slots = kMaxValuesPerThread / (8 * vpu);
  const int64_t units = (K + unit - 1) / unit;
  int64_t w = (units + slots - 1) / slots;
  if (w < 1) w = 1;
  return w > 1024 ? 1024 : static_cast<int>(w);
}

cudaError_t launch_row_prep(const RowPrepArgs& a, int x_dtype, int block, int out,
                            cudaStream_t stream) {
  switch (x_dtype) {
    case DT_BF16: return launch_row_prep_bf16(a, block, out, stream);
    case DT_F16: return launch_row_prep_f16(a, block, out, stream);
    case DT_F32: return launch_row_prep_f32(a, block, out, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace m5b
