// Row-preparation kernel instantiations for __half inputs (see prep_impl.cuh).
#include "prep_impl.cuh"
#include "rotq_impl.cuh"

namespace m5b {
cudaError_t launch_row_prep_f16(const RowPrepArgs& a, const RowMaps& m, int block, int out,
                                 cudaStream_t stream) {
  if (rotq::applicable(a, m, block, out, sizeof(__half), DT_F16)) return rotq::launch<__half>(a, m, block, out, stream);
  return launch_o<__half>(a, m, block, out, stream);
}
}  // namespace m5b
