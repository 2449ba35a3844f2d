// Tied bf16 lm_head: logits = x @ W^T as a streaming GEMV, with the greedy
// token (argmax) fused in. sm_100a.
//
// Replaces, for decode sizes (M <= 8 tokens), the reference's lm_head
// (src/qwen_int4/model.py:217-218,243: nn.Linear over the tied embedding,
// bf16 weight [V, D]) and the greedy pick on its output
// (src/qwen_int4/generation.py:51: logits[:, -1].argmax(dim=-1)).
// The weight (467 MB for Qwen2-1.5B) is read once per call with 16-byte
// streaming loads; each warp walks its rows two at a time (all twelve loads of
// a lane in flight), dots them with the tokens' activations (bf16 in shared
// memory, FP32 products and sums), sums the lanes with shuffles and rounds the
// logit to bf16 - the value the reference's bf16 linear returns. The argmax
// is over those rounded values, first index on ties (torch.argmax's rule):
// each CTA keeps its best (value, row) per token and merges it into a 64-bit
// key (order-preserving bits of the value, inverted row) with one atomicMax;
// a final kernel turns the keys into indices. Writing the full logits is
// optional (a caller that only needs the greedy token skips the 0.3 MB/token
// store).
#include "qi4_common.cuh"

namespace qi4 {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxTok = 8;
constexpr int kRows = 2;  // rows per warp iteration

__device__ __forceinline__ uint4 ld_stream(const void* p) { return ldg_stream16(p); }

// Order-preserving unsigned image of a float (-0 taken as +0).
__device__ __forceinline__ uint32_t ordered(float v) {
  uint32_t u = __float_as_uint(v == 0.f ? 0.f : v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <int M>
__global__ void __launch_bounds__(kThreads) gemv_argmax_kernel(const __nv_bfloat16* __restrict__ W,
                                                               const __nv_bfloat16* __restrict__ x, int64_t N,
                                                               int K, __nv_bfloat16* __restrict__ logits,
                                                               unsigned long long* __restrict__ keys,
                                                               int64_t rows_per_cta) {
  extern __shared__ uint4 xs_raw[];  // [M][K] bf16
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  pdl_launch_dependents();
  pdl_wait();  // x is the previous kernel's output
  for (int i = tid; i < M * K / 8; i += kThreads) xs_raw[i] = reinterpret_cast<const uint4*>(x)[i];
  __syncthreads();
  const uint32_t xs = (uint32_t)__cvta_generic_to_shared(xs_raw);
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_cta, r1 = min(N, r0 + rows_per_cta);
  const int chunks = K / 8;  // 16-byte chunks per row
  float best[M];
  int64_t best_row[M];
#pragma unroll
  for (int t = 0; t < M; ++t) {
    best[t] = -INFINITY;
    best_row[t] = -1;
  }
  for (int64_t r = r0 + warp * kRows; r < r1; r += (kThreads / 32) * kRows) {
    float acc[kRows][M];
#pragma unroll
    for (int j = 0; j < kRows; ++j)
#pragma unroll
      for (int t = 0; t < M; ++t) acc[j][t] = 0.f;
    for (int c0 = lane; c0 < chunks; c0 += 32 * 6) {
      uint4 w[kRows][6];
#pragma unroll
      for (int j = 0; j < kRows; ++j)
#pragma unroll
        for (int u = 0; u < 6; ++u) {
          const int c = c0 + u * 32;
          w[j][u] = (r + j < r1 && c < chunks) ? ld_stream(W + (r + j) * K + (int64_t)c * 8) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
      for (int u = 0; u < 6; ++u) {
        const int c = c0 + u * 32;
        if (c >= chunks) break;
#pragma unroll
        for (int t = 0; t < M; ++t) {
          uint4 xv;
          asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];"
                       : "=r"(xv.x), "=r"(xv.y), "=r"(xv.z), "=r"(xv.w)
                       : "r"(xs + (uint32_t)((t * K + c * 8) * 2)));
          const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
          for (int j = 0; j < kRows; ++j) {
            const uint32_t ww[4] = {w[j][u].x, w[j][u].y, w[j][u].z, w[j][u].w};
            float a = acc[j][t];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              a = fmaf(__uint_as_float(ww[e] << 16), __uint_as_float(xw[e] << 16), a);
              a = fmaf(__uint_as_float(ww[e] & 0xFFFF0000u), __uint_as_float(xw[e] & 0xFFFF0000u), a);
            }
            acc[j][t] = a;
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
      if (r + j >= r1) break;
#pragma unroll
      for (int t = 0; t < M; ++t) {
        float v = acc[j][t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        const __nv_bfloat16 rb = __float2bfloat16_rn(v);
        const float vr = __bfloat162float(rb);
        if (lane == 0 && logits) logits[(int64_t)t * N + r + j] = rb;
        if (vr > best[t]) {  // rows ascend, so a later row never wins a tie
          best[t] = vr;
          best_row[t] = r + j;
        }
      }
    }
  }
  // CTA merge (warps in order, ties to the smaller row), then one atomic per token.
  __shared__ float wb[kThreads / 32][kMaxTok];
  __shared__ long long wr[kThreads / 32][kMaxTok];
  if (lane == 0) {
#pragma unroll
    for (int t = 0; t < M; ++t) {
      wb[warp][t] = best[t];
      wr[warp][t] = best_row[t];
    }
  }
  __syncthreads();
  if (tid < M) {
    float bv = -INFINITY;
    long long br = -1;
    for (int w = 0; w < kThreads / 32; ++w) {
      if (wr[w][tid] < 0) continue;
      if (br < 0 || wb[w][tid] > bv || (wb[w][tid] == bv && wr[w][tid] < br)) {
        bv = wb[w][tid];
        br = wr[w][tid];
      }
    }
    if (br >= 0) {
      const unsigned long long key = ((unsigned long long)ordered(bv) << 32) | (0xFFFFFFFFull - (unsigned long long)br);
      atomicMax(keys + tid, key);
    }
  }
}

// Keys -> indices; the keys are left zero again, ready for the next call.
__global__ void argmax_finalize_kernel(unsigned long long* keys, int64_t* out, int M) {
  pdl_launch_dependents();
  pdl_wait();
  const int t = threadIdx.x;
  if (t < M) {
    out[t] = keys[t] ? (int64_t)(0xFFFFFFFFull - (keys[t] & 0xFFFFFFFFull)) : 0;
    keys[t] = 0;
  }
}

// Row-wise argmax of bf16 logits (torch.argmax(dim=-1): the first index of
// the largest value, a NaN counting as larger than every number). One CTA
// per row; a thread keeps the best 64-bit key of its elements (order-
// preserving value bits over the inverted index: the largest key is the
// largest value at the smallest index), then warp shuffles and a pass over
// the warps' keys. 16-byte loads when the rows allow them.
constexpr int kArgmaxThreads = 1024, kArgmaxLoads = 8;

__device__ __forceinline__ unsigned long long argmax_key(uint32_t bits16, int64_t i) {
  const float v = __uint_as_float(bits16 << 16);
  const uint32_t o = v != v ? 0xFFFFFFFFu : ordered(v);
  return ((unsigned long long)o << 32) | (0xFFFFFFFFull - (unsigned long long)i);
}

__global__ void __launch_bounds__(kArgmaxThreads) argmax_rows_kernel(const uint16_t* __restrict__ logits, int64_t V,
                                                                     int64_t ld, int64_t* __restrict__ out,
                                                                     int vec) {
  pdl_launch_dependents();
  pdl_wait();
  const uint16_t* row = logits + (int64_t)blockIdx.x * ld;
  unsigned long long best = 0;
  if (vec) {
    // kArgmaxLoads 16-byte loads of a thread in flight at once (a row is one
    // CTA's: its bytes in flight set the row's speed).
    const uint4* r4 = reinterpret_cast<const uint4*>(row);
    const int64_t n16 = V / 8;
    for (int64_t c0 = threadIdx.x; c0 < n16; c0 += (int64_t)kArgmaxThreads * kArgmaxLoads) {
      uint4 w[kArgmaxLoads];
#pragma unroll
      for (int u = 0; u < kArgmaxLoads; ++u) {
        const int64_t c = c0 + (int64_t)u * kArgmaxThreads;
        w[u] = c < n16 ? __ldg(r4 + c) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < kArgmaxLoads; ++u) {
        const int64_t c = c0 + (int64_t)u * kArgmaxThreads;
        if (c >= n16) break;
        const uint32_t ws[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const unsigned long long k0 = argmax_key(ws[e] & 0xFFFFu, c * 8 + 2 * e);
          const unsigned long long k1 = argmax_key(ws[e] >> 16, c * 8 + 2 * e + 1);
          best = k0 > best ? k0 : best;
          best = k1 > best ? k1 : best;
        }
      }
    }
    for (int64_t i = V / 8 * 8 + threadIdx.x; i < V; i += kArgmaxThreads) {
      const unsigned long long k = argmax_key(row[i], i);
      best = k > best ? k : best;
    }
  } else {
    for (int64_t i = threadIdx.x; i < V; i += kArgmaxThreads) {
      const unsigned long long k = argmax_key(row[i], i);
      best = k > best ? k : best;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
    best = k > best ? k : best;
  }
  __shared__ unsigned long long wk[kArgmaxThreads / 32];
  if ((threadIdx.x & 31) == 0) wk[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = wk[0];
    for (int w = 1; w < kArgmaxThreads / 32; ++w) b = wk[w] > b ? wk[w] : b;
    out[blockIdx.x] = (int64_t)(0xFFFFFFFFull - (b & 0xFFFFFFFFull));
  }
}

cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t stream, cudaLaunchAttribute* attr) {
  attr->id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr->val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

template <int M>
cudaError_t launch_m(const void* w, const void* x, int64_t N, int K, void* logits, unsigned long long* keys, int sms,
                     cudaStream_t stream) {
  const size_t smem = (size_t)M * K * 2;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(gemv_argmax_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)smem);
    if (e != cudaSuccess) return e;
  }
  // One wave: as many CTAs as fit on the SMs at once (registers bound it: at
  // M = 1, 76 registers allow three 256-thread CTAs per SM), each an equal
  // share of the rows - a fixed four per SM left a thin second wave.
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_argmax_kernel<M>, kThreads, smem) != cudaSuccess ||
      occ < 1) {
    cudaGetLastError();
    occ = 1;
  }
  const int grid = sms * occ;
  const int64_t rows_per_cta = ((N + grid - 1) / grid + kRows - 1) / kRows * kRows;
  cudaLaunchAttribute attr;
  const cudaLaunchConfig_t cfg = pdl_config(dim3(grid), dim3(kThreads), smem, stream, &attr);
  return cudaLaunchKernelEx(&cfg, gemv_argmax_kernel<M>, static_cast<const __nv_bfloat16*>(w),
                            static_cast<const __nv_bfloat16*>(x), N, K, static_cast<__nv_bfloat16*>(logits), keys,
                            rows_per_cta);
}

}  // namespace

}  // namespace qi4

namespace qi4 {
namespace {

int lm_head_impl(const void* weight, const void* x, int64_t M, int64_t K, int64_t N, void* logits, int64_t* argmax,
                 unsigned long long* keys_ws, void* stream_ptr) {
  clear_error();
  if (!weight || !x || (!logits && !argmax)) {
    set_error("weight and x must be non-null, and at least one of logits / argmax");
    return QI4_ERR_ARGUMENT;
  }
  if (M < 1 || M > kMaxTok || K <= 0 || K % 8 || K > 16384 || N <= 0 || N >= (int64_t)1 << 32) {
    set_error("lm_head GEMV takes 1 <= M <= %d, K a multiple of 8 up to 16384 and N < 2^32 (got M=%lld K=%lld "
              "N=%lld)", kMaxTok, (long long)M, (long long)K, (long long)N);
    return QI4_ERR_SHAPE;
  }
  if ((reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(x)) & 15) {
    set_error("weight and x must be 16-byte aligned");
    return QI4_ERR_ALIGNMENT;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  void* keys = keys_ws;
  if (argmax && !keys) {
    if (scratch_alloc(&keys, kMaxTok * sizeof(unsigned long long), stream) != cudaSuccess) {
      cudaGetLastError();
      set_error("cannot allocate the argmax scratch");
      return QI4_ERR_LAUNCH;
    }
    cudaMemsetAsync(keys, 0, kMaxTok * sizeof(unsigned long long), stream);
  }
  auto k = argmax ? static_cast<unsigned long long*>(keys) : nullptr;
  cudaError_t e;
  switch (M) {
    case 1: e = launch_m<1>(weight, x, N, (int)K, logits, k, sms, stream); break;
    case 2: e = launch_m<2>(weight, x, N, (int)K, logits, k, sms, stream); break;
    case 3: e = launch_m<3>(weight, x, N, (int)K, logits, k, sms, stream); break;
    case 4: e = launch_m<4>(weight, x, N, (int)K, logits, k, sms, stream); break;
    case 5: e = launch_m<5>(weight, x, N, (int)K, logits, k, sms, stream); break;
    case 6: e = launch_m<6>(weight, x, N, (int)K, logits, k, sms, stream); break;
    case 7: e = launch_m<7>(weight, x, N, (int)K, logits, k, sms, stream); break;
    default: e = launch_m<8>(weight, x, N, (int)K, logits, k, sms, stream); break;  // M == 8
  }
  if (e == cudaSuccess && argmax) {
    cudaLaunchAttribute attr;
    const cudaLaunchConfig_t cfg = pdl_config(dim3(1), dim3(32), 0, stream, &attr);
    e = cudaLaunchKernelEx(&cfg, argmax_finalize_kernel, k, argmax, (int)M);
  }
  if (keys && !keys_ws) scratch_free(keys, stream);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("lm_head GEMV launch failed: %s", cudaGetErrorString(e));
    return QI4_ERR_LAUNCH;
  }
  return QI4_OK;
}

}  // namespace
}  // namespace qi4

extern "C" QI4_API int qi4_bf16_gemv_argmax(const void* weight, const void* x, int64_t M, int64_t K, int64_t N,
                                            void* logits, int64_t* argmax, void* stream_ptr) {
  return qi4::lm_head_impl(weight, x, M, K, N, logits, argmax, nullptr, stream_ptr);
}

extern "C" QI4_API int qi4_bf16_gemv_argmax_ws(const void* weight, const void* x, int64_t M, int64_t K, int64_t N,
                                               void* logits, int64_t* argmax, uint64_t* keys, void* stream_ptr) {
  using namespace qi4;
  if (argmax && (!keys || (reinterpret_cast<uintptr_t>(keys) & 7))) {
    clear_error();
    set_error("the argmax workspace must be 8 zeroed, 8-byte aligned 64-bit words");
    return QI4_ERR_ARGUMENT;
  }
  return lm_head_impl(weight, x, M, K, N, logits, argmax, reinterpret_cast<unsigned long long*>(keys), stream_ptr);
}

extern "C" QI4_API int qi4_bf16_argmax_rows(const void* logits, int64_t B, int64_t V, int64_t ld, int64_t* out,
                                            void* stream_ptr) {
  using namespace qi4;
  clear_error();
  if (!logits || !out) {
    set_error("logits and out must be non-null");
    return QI4_ERR_ARGUMENT;
  }
  if (B < 1 || B > INT32_MAX || V < 1 || V >= (int64_t)1 << 32 || ld < V) {
    set_error("argmax_rows takes 1 <= B < 2^31, 1 <= V < 2^32 and a row pitch ld >= V (got B=%lld V=%lld ld=%lld)",
              (long long)B, (long long)V, (long long)ld);
    return QI4_ERR_SHAPE;
  }
  const int vec = (reinterpret_cast<uintptr_t>(logits) & 15) == 0 && ld % 8 == 0;
  cudaLaunchAttribute attr;
  const cudaLaunchConfig_t cfg =
      pdl_config(dim3((unsigned)B), dim3(kArgmaxThreads), 0, static_cast<cudaStream_t>(stream_ptr), &attr);
  const cudaError_t e =
      cudaLaunchKernelEx(&cfg, argmax_rows_kernel, static_cast<const uint16_t*>(logits), V, ld, out, vec);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("argmax_rows launch failed: %s", cudaGetErrorString(e));
    return QI4_ERR_LAUNCH;
  }
  return QI4_OK;
}
