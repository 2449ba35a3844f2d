// Host interface of the decode GEMV (gemv.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace qi4 {

struct GemvPlan {
  int mt;                // padded token count (template width): 1, 2, 4, 8 or 16
  int lpr;               // lanes that share one weight row: 8, 16 or 32
  int warps;             // warps per CTA
  int ksplit;            // CTAs (one cluster) per row tile along K
  int depth;             // chunk loads each lane keeps in flight: 4 or 8
  int chunks_per_split;  // 32-code chunks of K per CTA
  int rows_per_cta;
  size_t smem;           // dynamic shared memory bytes
};

constexpr int kGemvMaxM = 16;

// Picks the launch shape for an [M<=16, K] x [N, K]^T product.
GemvPlan plan_gemv(int64_t M, int64_t N, int64_t K, int num_sms);

// Forces the launch shape of subsequent GEMV plans on this thread (lpr = 0
// restores the model-based choice). Used by tuning sweeps.
void set_gemv_override(int lpr, int warps, int ksplit, int depth);

cudaError_t launch_gemv(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qweight,
                        const uint16_t* scales, const uint8_t* zeros, const void* bias, int bias_dtype,
                        void* out, int64_t N, cudaStream_t stream, bool pdl, const GemvPlan& plan);

}  // namespace qi4
