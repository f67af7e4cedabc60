// Row-preparation kernel instantiations for float inputs (see prep_impl.cuh).
#include "prep_impl.cuh"
#include "rotq_impl.cuh"

namespace m5b {
cudaError_t launch_row_prep_f32(const RowPrepArgs& a, const RowMaps& m, int block, int out,
                                 cudaStream_t stream) {
  if (rotq::applicable(a, m, block, out, sizeof(float), DT_F32)) return rotq::launch<float>(a, m, block, out, stream);
  return launch_o<float>(a, m, block, out, stream);
}
}  // namespace m5b
