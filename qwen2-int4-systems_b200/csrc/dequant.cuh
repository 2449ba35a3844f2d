// Host interface of the format primitives (dequant.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace qi4 {

cudaError_t launch_unpack(const uint8_t* packed, int8_t* out, int64_t elements, cudaStream_t stream,
                          int num_sms);

cudaError_t launch_dequant_f32(const uint8_t* qweight, const uint16_t* scales, const uint8_t* zeros, float* out,
                               int64_t N, int64_t K, cudaStream_t stream, int num_sms);

}  // namespace qi4
