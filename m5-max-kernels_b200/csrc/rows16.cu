// Register-streamed row-preparation kernel instantiations (see rows16_impl.cuh).
#include "rows16_impl.cuh"

namespace m5b {

bool rows16_applicable(const RowPrepArgs& a, int x_dtype, int block, int out) {
  if (x_dtype != DT_BF16 && x_dtype != DT_F16) return false;
  return rows16::applicable(a, block, out, 2, x_dtype);
}

cudaError_t launch_rows16(const RowPrepArgs& a, int x_dtype, int block, int out,
                          cudaStream_t stream) {
  if (x_dtype == DT_BF16) return rows16::launch<__nv_bfloat16>(a, block, out, stream);
  if (x_dtype == DT_F16) return rows16::launch<__half>(a, block, out, stream);
  return cudaErrorInvalidValue;
}

}  // namespace m5b
