// Host interface of the TMA + tensor-core decode GEMV (gemv_mma.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace qi4 {

// Residual add + RMSNorm formed while a launch stages its activations (bf16
// only): hn = bf16(h_in + bf16(delta)), x = bf16(bf16(hn * rsqrt(mean(hn^2) +
// eps)) * weight); hn is written to h_out (which must not alias h_in).
struct NormPrologue {
  const void* h_in;    // bf16 [M, K]
  const void* delta;   // bf16 or FP32 [M, K]; null: hn = h_in
  int delta_dtype;
  float eps;
  const void* weight;  // bf16 [K]
  void* h_out;         // bf16 [M, K]
};

struct MmaGemvPlan {
  int rows;             // output rows per CTA: 16, 32, 64 or 128
  int ksplit;           // CTAs per cluster along K (1..8)
  int warps;            // warps per CTA: 2, 4, 8 or 16 (rows / 16 <= warps)
  int boxes_per_split;  // 128-byte (4-group) boxes of K per CTA
  int nt;               // n8 token tiles: 1 (M <= 8) or 2 (M <= 16)
  int pre;              // 1: weight fragments expanded before the dependency wait
  int copy_log2;        // log2 of the 128-byte boxes per TMA copy
  int three_d;          // 1: 3-D box-major copies (K a multiple of 256)
  size_t smem;
};

bool gemv_mma_supported(int64_t M, int64_t K);
MmaGemvPlan plan_gemv_mma(int64_t M, int64_t N, int64_t K, int x_dtype, int num_sms);
void set_gemv_mma_override(int rows, int ksplit, int warps);  // rows = 0 restores the model
cudaError_t launch_gemv_mma(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qweight,
                            const uint16_t* scales, const uint8_t* zeros, const void* bias, int bias_dtype,
                            void* out, int64_t N, cudaStream_t stream, bool pdl, const MmaGemvPlan& plan);
// One launch over `count` (1..3) weight matrices that share the activations x
// (q/k/v, gate/up): matrix i writes outs[i] (M x Ns[i]); biases may be null.
// The plan is that of an N of sum(round_up(Ns[i], 16)).
cudaError_t launch_gemv_mma_multi(const void* x, int x_dtype, int64_t M, int64_t K, int count,
                                  const uint8_t* const* qweights, const uint16_t* const* scales,
                                  const uint8_t* const* zeros, const void* const* biases, int bias_dtype,
                                  void* const* outs, const int64_t* Ns, cudaStream_t stream, bool pdl,
                                  const MmaGemvPlan& plan, const NormPrologue* norm = nullptr);
// Fused gate/up + SwiGLU for M <= 16: out[M, N] (FP32) = silu(g) * u with g, u
// the two projections of x rounded to the activation dtype (the reference
// MLP's composition). qweights/scales/zeros hold {gate, up}.
MmaGemvPlan plan_gemv_swiglu(int64_t M, int64_t K, int x_dtype);
cudaError_t launch_gemv_swiglu(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* const* qweights,
                               const uint16_t* const* scales, const uint8_t* const* zeros, float* out, int64_t N,
                               cudaStream_t stream, bool pdl, const MmaGemvPlan& plan,
                               const NormPrologue* norm = nullptr);
// out[i] = silu(g[i]) * u[i] in FP32 from two activation-dtype arrays.
cudaError_t launch_swiglu_elementwise(const void* g, const void* u, int dtype, float* out, int64_t n,
                                      cudaStream_t stream, int num_sms);
// Reads and clears the kernel's device error flag (synchronises `stream`); -1 on failure.
int read_gemv_mma_error(cudaStream_t stream);

// One CTA whose bounded mbarrier wait runs out after limit_ns (failure-detection self-test).
cudaError_t launch_bounded_wait_selftest(uint64_t limit_ns, cudaStream_t stream);

}  // namespace qi4
