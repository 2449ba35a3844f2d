// tcgen05 dequant-GEMM (prefill, M >= 128). Placeholder until the kernel lands.
#include "gemm_tc.cuh"

namespace qi4 {

bool tc_supported(int64_t, int64_t, int64_t, int) { return false; }

cudaError_t launch_gemm_tc(const void*, int, int64_t, int64_t, const uint8_t*, const uint16_t*, const uint8_t*,
                           const void*, int, void*, int64_t, cudaStream_t, bool, int) {
  return cudaErrorNotSupported;
}

}  // namespace qi4
