// Row-preparation kernel instantiations for __nv_bfloat16 inputs (see prep_impl.cuh).
#include "prep_impl.cuh"
#include "rotq_impl.cuh"

namespace m5b {
cudaError_t launch_row_prep_bf16(const RowPrepArgs& a, const RowMaps& m, int block, int out,
                                 cudaStream_t stream) {
  if (rotq::applicable(a, m, block, out, sizeof(__nv_bfloat16), DT_BF16)) return rotq::launch<__nv_bfloat16>(a, m, block, out, stream);
  return launch_o<__nv_bfloat16>(a, m, block, out, stream);
}
}  // namespace m5b
