// gemm_tc.cu -- tensor-core (tcgen05) linear layer.  Not wired yet: every
// problem is reported unsupported so ct_linear_fwd uses the CUDA-core kernel.
#include "ct_internal.h"

namespace ct {

bool linear_tc_supported(const GemmProblem&) { return false; }

int launch_linear_tc(const GemmProblem&, const DeviceInfo&, cudaStream_t) {
  return CT_ERR_INVALID_ARGUMENT;
}

}  // namespace ct
