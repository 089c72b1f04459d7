// Prefill-regime int4 linear on the 5th-generation tensor cores (placeholder
// until the tcgen05 kernel lands: reports the regime as unavailable).
#include "qlinear.cuh"

namespace tf {

bool gemm_supported(const QLinearProblem&) { return false; }
size_t gemm_workspace_bytes(int64_t, int64_t, int64_t) { return kWsHeader; }
int gemm_launch(const QLinearProblem&, cudaStream_t) {
  return fail(TF_ERR_UNSUPPORTED, "qlinear: tcgen05 GEMM regime not built");
}

}  // namespace tf
