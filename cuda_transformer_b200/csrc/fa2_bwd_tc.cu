// fa2_bwd_tc.cu -- tensor-core FlashAttention-2 backward.  Not wired yet:
// every problem is reported unsupported so the C ABI uses the CUDA-core path.
#include "ct_internal.h"

namespace ct {

bool fa2_bwd_tc_supported(const Fa2Problem&) { return false; }

int launch_fa2_bwd_dq_tc(const Fa2Problem&, Strided4, Strided4, Strided4, Strided4, const float*,
                         const int64_t*, const float*, float*, const DeviceInfo&, cudaStream_t) {
  return CT_ERR_INVALID_ARGUMENT;
}

int launch_fa2_bwd_dkdv_tc(const Fa2Problem&, Strided4, Strided4, Strided4, Strided4,
                           const float*, const int64_t*, const float*, float*, float*,
                           const DeviceInfo&, cudaStream_t) {
  return CT_ERR_INVALID_ARGUMENT;
}

}  // namespace ct
