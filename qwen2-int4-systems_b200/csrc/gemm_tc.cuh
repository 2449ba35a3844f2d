// Host interface of the tcgen05 dequant-GEMM (gemm_tc.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace qi4 {

// Whether the tensor-core kernel handles this problem.
bool tc_supported(int64_t M, int64_t N, int64_t K, int x_dtype);

cudaError_t launch_gemm_tc(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qweight,
                           const uint16_t* scales, const uint8_t* zeros, const void* bias, int bias_dtype, void* out,
                           int64_t N, cudaStream_t stream, bool pdl, int num_sms);

// Up to three weight matrices that share the activations (q/k/v, gate/up) in
// one launch: each CTA takes a 128-row tile of one matrix; every output has
// the activation dtype.
cudaError_t launch_gemm_tc_multi(const void* x, int x_dtype, int64_t M, int64_t K, int count,
                                 const uint8_t* const* qweights, const uint16_t* const* scales,
                                 const uint8_t* const* zeros, const void* const* biases, int bias_dtype,
                                 void* const* outs, const int64_t* Ns, cudaStream_t stream, bool pdl, int num_sms);

// FP32-activation tensor-core linear whose scratch is a fixed static device
// array (no allocation); x and out are FP32. M * K * 4 bytes must not exceed
// static_scratch_bytes(). Not reentrant across concurrent streams.
size_t static_scratch_bytes();
cudaError_t launch_gemm_tc_f32_static(const float* x, int64_t M, int64_t K, const uint8_t* qweight,
                                      const uint16_t* scales, const uint8_t* zeros, const void* bias, int bias_dtype,
                                      float* out, int64_t N, cudaStream_t stream, int num_sms);

// Forces the token-tile width (32, 64, 128, 192 or 256; FP32 activations at
// most 128) and the K split (1..8, tiles of at most 128 tokens) of later
// launches from the calling thread; bn = 0 restores the library's choice.
void set_gemm_tc_override(int bn, int ksplit);

// Reads and clears the kernel's device error flag (synchronises `stream`); -1 on failure.
int read_gemm_tc_error(cudaStream_t stream);

}  // namespace qi4
