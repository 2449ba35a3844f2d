// Residual add + RMSNorm of a decoder block boundary (sm_100a), one CTA per row.
//
// The reference decoder adds each block's output to the bf16 residual stream
// and normalises it for the next block (src/qwen_int4/model.py:151-159
// DecoderLayer.forward, 31-42 RMSNorm.forward):
//   h   = bf16(h + bf16(delta))                       (delta bf16 or FP32)
//   out = bf16(bf16(h * rsqrt(mean(h^2) + eps)) * w)   (FP32 statistics)
// Both in one pass over the row: h is updated in place (delta may be NULL:
// normalisation only). Launched as a programmatic dependent of the kernel
// before it (which produced delta).
#include "qi4_common.cuh"

namespace qi4 {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxPerThread = 16;  // D <= 4096

__global__ void __launch_bounds__(kThreads) add_rmsnorm_kernel(__nv_bfloat16* __restrict__ h,
                                                               const void* __restrict__ delta, int delta_dtype,
                                                               const __nv_bfloat16* __restrict__ w,
                                                               __nv_bfloat16* __restrict__ out, int D, float eps) {
  const int row = blockIdx.x, tid = threadIdx.x;
  pdl_launch_dependents();
  pdl_wait();  // delta is the previous kernel's output
  __nv_bfloat16* hr = h + (int64_t)row * D;
  float v[kMaxPerThread];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxPerThread; ++j) {
    const int i = tid + j * kThreads;
    v[j] = 0.f;
    if (i < D) {
      float x = __bfloat162float(hr[i]);
      if (delta) {
        const float d = delta_dtype == QI4_DTYPE_F32
                            ? __bfloat162float(__float2bfloat16_rn(static_cast<const float*>(delta)[(int64_t)row * D + i]))
                            : __bfloat162float(static_cast<const __nv_bfloat16*>(delta)[(int64_t)row * D + i]);
        x = __bfloat162float(__float2bfloat16_rn(x + d));
        hr[i] = __float2bfloat16_rn(x);
      }
      v[j] = x;
      ss = fmaf(x, x, ss);
    }
  }
  __shared__ float part[kThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) part[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < kThreads / 32; ++k) tot += part[k];
  const float r = rsqrtf(tot / (float)D + eps);
#pragma unroll
  for (int j = 0; j < kMaxPerThread; ++j) {
    const int i = tid + j * kThreads;
    if (i < D) {
      const float nrm = __bfloat162float(__float2bfloat16_rn(v[j] * r));
      out[(int64_t)row * D + i] = __float2bfloat16_rn(nrm * __bfloat162float(w[i]));
    }
  }
}

}  // namespace

}  // namespace qi4

extern "C" QI4_API int qi4_add_rmsnorm(void* h, const void* delta, int delta_dtype, const void* weight, void* out,
                                       int64_t B, int64_t D, float eps, void* stream) {
  using namespace qi4;
  clear_error();
  if (!h || !weight || !out || B <= 0 || D <= 0) {
    set_error("h, weight and out must be non-null and B, D positive");
    return QI4_ERR_ARGUMENT;
  }
  if (D > kThreads * kMaxPerThread || B > (1 << 30)) {
    set_error("add_rmsnorm supports D <= %d (got %lld)", kThreads * kMaxPerThread, (long long)D);
    return QI4_ERR_SHAPE;
  }
  if (delta && delta_dtype != QI4_DTYPE_BF16 && delta_dtype != QI4_DTYPE_F32) {
    set_error("delta dtype %d is not BF16 or F32", delta_dtype);
    return QI4_ERR_DTYPE;
  }
  // A programmatic dependent launch: the kernel's prologue overlaps the tail
  // of the kernel before it, and it waits for that kernel before reading.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)B, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, add_rmsnorm_kernel, static_cast<__nv_bfloat16*>(h), delta, delta_dtype,
                     static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(out), (int)D, eps);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("add_rmsnorm launch failed: %s", cudaGetErrorString(e));
    return QI4_ERR_LAUNCH;
  }
  return launch_status("add_rmsnorm");
}
