// gemm_tc.cu — K3: tcgen05 INT8 GEMM (placeholder until the tensor-core
// kernel lands; the dispatcher then uses the streaming GEMV per 8-row chunk).
#include "internal.h"

namespace mri {

bool gemm_i8_tc_supported(const DeviceInfo&, size_t, size_t, size_t) { return false; }

cudaError_t launch_gemm_i8_tc(const DeviceInfo&, cudaStream_t, const int8_t*, const float*, int,
                              const int8_t*, const float*, size_t, size_t, size_t, float*,
                              int32_t*, int*, LaunchStats*) {
  return cudaErrorNotSupported;
}

}  // namespace mri
