// Column-split gather fused into the SwiGLU pass, over peer memory (sm_100a).
//
// The out-feature split of the Qwen2 MLP (src/qwen_int4/model.py:125-136 run
// over several GPUs) gives each rank a column range of the FP32 intermediate
// silu(gate) * up; down_proj split by output features needs all of it on
// every rank. Instead of an NCCL all-gather after the pass, the pass itself
// stores each value into every rank's gathered buffer: its own (local
// stores) and its peers' (stores through CUDA IPC mappings over NVLink), so
// the exchange overlaps the arithmetic element by element. Completion is a
// per-call epoch: every CTA orders its stores before a device-scope counter
// increment with a system-scope fence; the CTA that counts last fences again
// and writes the epoch into slot `rank` of every rank's flag array with a
// system-scope release store. A rank's consumer then runs a one-CTA wait
// (acquire loads of its flag array, bounded by the global timer; on time-out
// it records QI4_DEVICE_WAIT_TIMEOUT and returns) before reading the
// gathered buffer.
//
// Only plain loads and stores touch peer memory: no TMA, no multicast object.
#include "peer_exchange.cuh"
#include "qi4_common.cuh"
#include "tma_util.cuh"

namespace qi4 {

__device__ int g_peer_error;

namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float silu_mul(float g, float u) { return g / (1.0f + expf(-g)) * u; }

template <typename T>
__device__ __forceinline__ float to_f32(T v) {
  return static_cast<float>(v);
}

// g, u: [M, n] (the shard's projections, activation dtype, contiguous).
// Element (m, c) goes to outs[p][m * ld + col0 + c] for every rank p.
// VEC: four consecutive columns per thread with 16-byte stores (n, ld and
// col0 multiples of 4, 16-byte-aligned buffers).
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) swiglu_scatter_kernel(const T* __restrict__ g, const T* __restrict__ u,
                                                             const PeerTargets t, int64_t M, int64_t n) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if constexpr (VEC) {
    const int64_t n4 = n / 4, total = M * n4;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
      const int64_t m = i / n4, c = (i - m * n4) * 4;
      const int64_t src = m * n + c;
      const float4 v = make_float4(silu_mul(to_f32(g[src]), to_f32(u[src])),
                                   silu_mul(to_f32(g[src + 1]), to_f32(u[src + 1])),
                                   silu_mul(to_f32(g[src + 2]), to_f32(u[src + 2])),
                                   silu_mul(to_f32(g[src + 3]), to_f32(u[src + 3])));
      const int64_t dst = m * t.ld + t.col0 + c;
#pragma unroll 1
      for (int p = 0; p < t.world; ++p) *reinterpret_cast<float4*>(t.out[p] + dst) = v;
    }
  } else {
    const int64_t total = M * n;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
      const int64_t m = i / n, c = i - m * n;
      const float v = silu_mul(to_f32(g[i]), to_f32(u[i]));
      const int64_t dst = m * t.ld + t.col0 + c;
#pragma unroll 1
      for (int p = 0; p < t.world; ++p) t.out[p][dst] = v;
    }
  }
  // Publish: this thread's stores, then the CTA count; the last CTA writes
  // the epoch into every rank's flag array and re-arms the counter.
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(t.counter, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int p = 0; p < t.world; ++p) st_release_sys(t.flags[p] + t.rank, t.epoch);
      *t.counter = 0u;
    }
  }
}

// Thread r < world waits until flags[r] has reached epoch (wrapping
// comparison), polling with acquire loads; past limit_ns it records a
// time-out and stops.
__global__ void __launch_bounds__(32) flag_wait_kernel(const uint32_t* flags, int world, uint32_t epoch,
                                                       uint64_t limit_ns) {
  const int r = threadIdx.x;
  if (r < world) {
    const uint64_t t0 = global_timer_ns();
    while ((int32_t)(ld_acquire_sys(flags + r) - epoch) < 0) {
      if (global_timer_ns() - t0 > limit_ns) {
        atomicOr(&g_peer_error, kErrWaitTimeout);
        break;
      }
      __nanosleep(200);
    }
  }
  __syncwarp();
}

}  // namespace

namespace {

template <typename T>
void launch_scatter_t(const void* g, const void* u, const PeerTargets& t, int64_t M, int64_t n, bool vec, int blocks,
                      cudaStream_t stream) {
  if (vec)
    swiglu_scatter_kernel<T, true><<<blocks, 256, 0, stream>>>(static_cast<const T*>(g), static_cast<const T*>(u), t,
                                                               M, n);
  else
    swiglu_scatter_kernel<T, false><<<blocks, 256, 0, stream>>>(static_cast<const T*>(g), static_cast<const T*>(u), t,
                                                                M, n);
}

}  // namespace

cudaError_t launch_swiglu_scatter(const void* g, const void* u, int dtype, const PeerTargets& t, int64_t M, int64_t n,
                                  cudaStream_t stream, int num_sms) {
  bool vec = n % 4 == 0 && t.ld % 4 == 0 && t.col0 % 4 == 0;
  for (int p = 0; p < t.world; ++p) vec = vec && (reinterpret_cast<uintptr_t>(t.out[p]) & 15) == 0;
  const int64_t items = vec ? M * (n / 4) : M * n;
  // At least one CTA, so that the epoch is published even for an empty shard.
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256, (int64_t)num_sms * 8));
  switch (dtype) {
    case QI4_DTYPE_F16: launch_scatter_t<__half>(g, u, t, M, n, vec, blocks, stream); break;
    case QI4_DTYPE_BF16: launch_scatter_t<__nv_bfloat16>(g, u, t, M, n, vec, blocks, stream); break;
    default: launch_scatter_t<float>(g, u, t, M, n, vec, blocks, stream); break;
  }
  return cudaGetLastError();
}

cudaError_t launch_flag_wait(const uint32_t* flags, int world, uint32_t epoch, uint64_t limit_ns,
                             cudaStream_t stream) {
  flag_wait_kernel<<<1, 32, 0, stream>>>(flags, world, epoch, limit_ns);
  return cudaGetLastError();
}

int read_peer_error(cudaStream_t stream) {
  int v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, g_peer_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return -1;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return -1;
  if (v) {
    const int zero = 0;
    cudaMemcpyToSymbolAsync(g_peer_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    cudaStreamSynchronize(stream);
  }
  return v;
}

}  // namespace qi4
