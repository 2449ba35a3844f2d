// extern "C" boundary of libqi4_b200.so (declared in include/qi4_b200.h).
//
// Validates arguments, checks the device, picks a kernel and launches it on
// the caller's stream. Device scratch comes from the library's stream-ordered
// pool; the qi4_ipc_* helpers (shared buffers of the multi-GPU exchange) are
// the only entry points that allocate, map or free device memory directly,
// and they synchronise.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "dequant.cuh"
#include "gemm_tc.cuh"
#include "gemv.cuh"
#include "gemv_mma.cuh"
#include "peer_exchange.cuh"
#include "qi4_common.cuh"

namespace qi4 {
int read_chain_error(cudaStream_t stream);      // decode_chain.cu
int read_attention_error(cudaStream_t stream);  // attention.cu
}

namespace qi4 {

namespace {
thread_local std::string g_last_error;

struct DeviceInfo {
  int sms = 0;
  int major = 0;
  bool ok = false;
};

// Per-device properties, filled on first use.
DeviceInfo device_info(int dev) {
  static std::mutex mu;
  static DeviceInfo cache[64];
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 0 || dev >= 64) return DeviceInfo{};
  if (!cache[dev].ok) {
    int sms = 0, major = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return DeviceInfo{};
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return DeviceInfo{};
    cache[dev] = DeviceInfo{sms, major, true};
  }
  return cache[dev];
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

bool valid_act_dtype(int d) { return d == QI4_DTYPE_F16 || d == QI4_DTYPE_BF16 || d == QI4_DTYPE_F32; }

int current_device(DeviceInfo& info) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    set_error("no CUDA device is available");
    return QI4_ERR_DEVICE;
  }
  info = device_info(dev);
  if (!info.ok) {
    set_error("cannot query CUDA device %d", dev);
    return QI4_ERR_DEVICE;
  }
  if (info.major != 10) {
    set_error("device %d has compute capability %d.x; this library is built for sm_100a (B200)", dev,
              info.major);
    return QI4_ERR_DEVICE;
  }
  return QI4_OK;
}

}  // namespace

// One pool per device, created on first use and kept for the life of the
// process (the pool handle belongs to the device context current then: a
// process that calls cudaDeviceReset must not use the FP32-activation paths
// on that device afterwards).
cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t stream) {
  // Under stream capture, allocate from the device's default stream-ordered
  // allocator: the graph turns it into its own allocation node.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) == cudaSuccess && cap == cudaStreamCaptureStatusActive)
    return cudaMallocAsync(p, bytes, stream);
  cudaGetLastError();
  static std::mutex mu;
  static cudaMemPool_t pools[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  cudaMemPool_t pool;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!pools[dev]) {
      cudaMemPoolProps props = {};
      props.allocType = cudaMemAllocationTypePinned;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev;
      e = cudaMemPoolCreate(&pools[dev], &props);
      if (e != cudaSuccess) {
        pools[dev] = nullptr;
        return e;
      }
      uint64_t keep = UINT64_MAX;
      cudaMemPoolSetAttribute(pools[dev], cudaMemPoolAttrReleaseThreshold, &keep);
    }
    pool = pools[dev];
  }
  return cudaMallocFromPoolAsync(p, bytes, pool, stream);
}

void scratch_free(void* p, cudaStream_t stream) {
  if (p) cudaFreeAsync(p, stream);
}

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

void clear_error() { g_last_error.clear(); }

int launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s launch failed: %s", what, cudaGetErrorString(e));
    return QI4_ERR_LAUNCH;
  }
  return QI4_OK;
}

static int check_launch(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("%s launch failed: %s", what, cudaGetErrorString(e));
    return QI4_ERR_LAUNCH;
  }
  return QI4_OK;
}

static int validate_linear(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qweight,
                           const uint16_t* scales, const void* bias, int bias_dtype, void* out, int64_t N) {
  if (!x || !qweight || !scales || !out) {
    set_error("x, qweight, scales and out must be non-null device pointers");
    return QI4_ERR_ARGUMENT;
  }
  if (M <= 0 || N <= 0 || K <= 0) {
    set_error("M, N and K must be positive (got M=%lld N=%lld K=%lld)", (long long)M, (long long)N,
              (long long)K);
    return QI4_ERR_ARGUMENT;
  }
  if (K % kGroup) {
    set_error("canonical W4G64 requires K divisible by 64 (got K=%lld)", (long long)K);
    return QI4_ERR_SHAPE;
  }
  if (K > (int64_t)1 << 24 || N > (int64_t)1 << 30 || M > (int64_t)1 << 30) {
    set_error("problem size out of range (M=%lld N=%lld K=%lld)", (long long)M, (long long)N, (long long)K);
    return QI4_ERR_SHAPE;
  }
  if (!valid_act_dtype(x_dtype)) {
    set_error("activation dtype code %d is not F16, BF16 or F32", x_dtype);
    return QI4_ERR_DTYPE;
  }
  if (bias != nullptr && !valid_act_dtype(bias_dtype)) {
    set_error("bias dtype code %d is not F16, BF16 or F32", bias_dtype);
    return QI4_ERR_DTYPE;
  }
  if (!aligned(qweight, 16)) {
    set_error("qweight must be 16-byte aligned");
    return QI4_ERR_ALIGNMENT;
  }
  if (!aligned(x, 16)) {
    set_error("x must be 16-byte aligned");
    return QI4_ERR_ALIGNMENT;
  }
  if (!aligned(scales, 2) || !aligned(out, x_dtype == QI4_DTYPE_F32 ? 4 : 2)) {
    set_error("scales / out are not naturally aligned");
    return QI4_ERR_ALIGNMENT;
  }
  return QI4_OK;
}

static int linear_impl(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qweight,
                       const uint16_t* scales, const uint8_t* zeros, const void* bias, int bias_dtype, void* out,
                       int64_t N, void* stream_ptr, int algo, int pdl) {
  clear_error();
  int rc = validate_linear(x, x_dtype, M, K, qweight, scales, bias, bias_dtype, out, N);
  if (rc) return rc;
  DeviceInfo info;
  rc = current_device(info);
  if (rc) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (!bias) bias_dtype = QI4_DTYPE_NONE;

  if (algo == QI4_ALGO_AUTO) {
    algo = (M > kGemvMaxM && tc_supported(M, N, K, x_dtype)) ? QI4_ALGO_TC : QI4_ALGO_GEMV;
  } else if (algo == QI4_ALGO_TC && !tc_supported(M, N, K, x_dtype)) {
    set_error("the tensor-core kernel does not support M=%lld N=%lld K=%lld dtype=%d", (long long)M,
              (long long)N, (long long)K, x_dtype);
    return QI4_ERR_SHAPE;
  }

  if (algo == QI4_ALGO_TC) {
    return check_launch(launch_gemm_tc(x, x_dtype, M, K, qweight, scales, zeros, bias, bias_dtype, out, N, stream,
                                       pdl != 0, info.sms),
                        "w4g64 tcgen05 GEMM");
  }
  if (algo != QI4_ALGO_GEMV && algo != QI4_ALGO_GEMV_FMA) {
    set_error("unknown algorithm code %d", algo);
    return QI4_ERR_ARGUMENT;
  }
  // A GEMV launch covers up to 16 token rows; larger M is processed in row
  // blocks (each block re-streams the weights).
  const size_t xsize = x_dtype == QI4_DTYPE_F32 ? 4 : 2;
  for (int64_t m0 = 0; m0 < M; m0 += kGemvMaxM) {
    const int64_t mb = (M - m0) < kGemvMaxM ? (M - m0) : kGemvMaxM;
    const void* xb = static_cast<const char*>(x) + m0 * K * xsize;
    void* ob = static_cast<char*>(out) + m0 * N * xsize;
    if (algo == QI4_ALGO_GEMV) {
      const MmaGemvPlan plan = plan_gemv_mma(mb, N, K, x_dtype, info.sms);
      if (plan.rows == 0) {
        set_error("no GEMV launch shape fits N=%lld K=%lld", (long long)N, (long long)K);
        return QI4_ERR_SHAPE;
      }
      rc = check_launch(
          launch_gemv_mma(xb, x_dtype, mb, K, qweight, scales, zeros, bias, bias_dtype, ob, N, stream, pdl != 0, plan),
          "w4g64 GEMV");
    } else {
      const GemvPlan plan = plan_gemv(mb, N, K, info.sms);
      if (plan.mt == 0) {
        set_error("no GEMV launch shape fits N=%lld K=%lld", (long long)N, (long long)K);
        return QI4_ERR_SHAPE;
      }
      rc = check_launch(
          launch_gemv(xb, x_dtype, mb, K, qweight, scales, zeros, bias, bias_dtype, ob, N, stream, pdl != 0, plan),
          "w4g64 FMA GEMV");
    }
    if (rc) return rc;
  }
  return QI4_OK;
}

// Checks a fused norm prologue and converts it; x of the launch is then h_in.
static int validate_norm(const qi4_rmsnorm_prologue* n, int64_t M, int64_t K, NormPrologue* out) {
  if (!n || !n->h_in || !n->weight || !n->h_out) {
    set_error("the norm prologue and its h_in, weight and h_out must be non-null");
    return QI4_ERR_ARGUMENT;
  }
  if (M < 1 || M > kGemvMaxM) {
    set_error("the fused norm prologue covers 1..%d tokens (got M=%lld)", kGemvMaxM, (long long)M);
    return QI4_ERR_SHAPE;
  }
  if (n->delta && n->delta_dtype != QI4_DTYPE_BF16 && n->delta_dtype != QI4_DTYPE_F32) {
    set_error("norm delta dtype %d is not BF16 or F32", n->delta_dtype);
    return QI4_ERR_DTYPE;
  }
  if (!aligned(n->h_in, 16) || !aligned(n->h_out, 16) || !aligned(n->weight, 16) ||
      (n->delta && !aligned(n->delta, 16))) {
    set_error("norm h_in, delta, weight and h_out must be 16-byte aligned");
    return QI4_ERR_ALIGNMENT;
  }
  const uintptr_t a = reinterpret_cast<uintptr_t>(n->h_in), b = reinterpret_cast<uintptr_t>(n->h_out);
  const uintptr_t bytes = (uintptr_t)(M * K * 2);
  if (a < b + bytes && b < a + bytes) {
    set_error("norm h_out must not overlap h_in (alternate two residual buffers)");
    return QI4_ERR_ARGUMENT;
  }
  if (!(n->eps >= 0.f) || n->eps > 1.f) {
    set_error("norm eps must be in [0, 1]");
    return QI4_ERR_ARGUMENT;
  }
  *out = NormPrologue{n->h_in, n->delta, n->delta_dtype, n->eps, n->weight, n->h_out};
  return QI4_OK;
}

static int linear_multi_impl(const void* x, int x_dtype, int64_t M, int64_t K, int count,
                             const uint8_t* const* qweights, const uint16_t* const* scales,
                             const uint8_t* const* zeros, const void* const* biases, int bias_dtype,
                             void* const* outs, const int64_t* Ns, void* stream_ptr,
                             const qi4_rmsnorm_prologue* norm = nullptr) {
  clear_error();
  NormPrologue np{};
  if (norm) {
    const int rc = validate_norm(norm, M, K, &np);
    if (rc) return rc;
    x = norm->h_in;
    x_dtype = QI4_DTYPE_BF16;
  }
  if (count < 1 || count > 3 || !qweights || !scales || !outs || !Ns) {
    set_error("count must be 1..3 and qweights, scales, outs, Ns non-null host arrays");
    return QI4_ERR_ARGUMENT;
  }
  bool any_bias = false;
  for (int i = 0; i < count; ++i) {
    const void* b = biases ? biases[i] : nullptr;
    any_bias |= b != nullptr;
    const int rc = validate_linear(x, x_dtype, M, K, qweights[i], scales[i], b, bias_dtype, outs[i], Ns[i]);
    if (rc) return rc;
  }
  if (!any_bias) bias_dtype = QI4_DTYPE_NONE;
  DeviceInfo info;
  int rc = current_device(info);
  if (rc) return rc;
  if (M > kGemvMaxM) {
    // Prefill sizes: one tensor-core launch over the tiles of every matrix.
    return check_launch(launch_gemm_tc_multi(x, x_dtype, M, K, count, qweights, scales, zeros, biases, bias_dtype,
                                             outs, Ns, static_cast<cudaStream_t>(stream_ptr), true, info.sms),
                        "w4g64 grouped tensor-core GEMM");
  }
  const uint8_t* zs[3] = {nullptr, nullptr, nullptr};
  const void* bs[3] = {nullptr, nullptr, nullptr};
  int64_t n_eff = 0;
  for (int i = 0; i < count; ++i) {
    zs[i] = zeros ? zeros[i] : nullptr;
    bs[i] = biases ? biases[i] : nullptr;
    n_eff += (Ns[i] + 15) / 16 * 16;
  }
  const MmaGemvPlan plan = plan_gemv_mma(M, n_eff, K, x_dtype, info.sms);
  if (plan.rows == 0) {
    set_error("no GEMV launch shape fits N=%lld K=%lld", (long long)n_eff, (long long)K);
    return QI4_ERR_SHAPE;
  }
  return check_launch(launch_gemv_mma_multi(x, x_dtype, M, K, count, qweights, scales, zs, bs, bias_dtype, outs, Ns,
                                            static_cast<cudaStream_t>(stream_ptr), true, plan, norm ? &np : nullptr),
                      "w4g64 grouped GEMV");
}

static int gate_up_silu_impl(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qw_gate,
                             const uint16_t* sc_gate, const uint8_t* z_gate, const uint8_t* qw_up,
                             const uint16_t* sc_up, const uint8_t* z_up, float* out, int64_t N, void* stream_ptr,
                             const qi4_rmsnorm_prologue* norm = nullptr) {
  clear_error();
  NormPrologue np{};
  if (norm) {
    const int rc = validate_norm(norm, M, K, &np);
    if (rc) return rc;
    x = norm->h_in;
    x_dtype = QI4_DTYPE_BF16;
  }
  int rc = validate_linear(x, x_dtype, M, K, qw_gate, sc_gate, nullptr, QI4_DTYPE_NONE, out, N);
  if (!rc) rc = validate_linear(x, x_dtype, M, K, qw_up, sc_up, nullptr, QI4_DTYPE_NONE, out, N);
  if (rc) return rc;
  if (!aligned(out, 4)) {
    set_error("out (FP32) must be 4-byte aligned");
    return QI4_ERR_ALIGNMENT;
  }
  DeviceInfo info;
  rc = current_device(info);
  if (rc) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const uint8_t* qws[2] = {qw_gate, qw_up};
  const uint16_t* scs[2] = {sc_gate, sc_up};
  const uint8_t* zs[2] = {z_gate, z_up};
  if (M <= kGemvMaxM) {
    const MmaGemvPlan plan = plan_gemv_swiglu(M, K, x_dtype);
    if (plan.rows == 0) {
      set_error("no fused gate/up launch shape fits K=%lld", (long long)K);
      return QI4_ERR_SHAPE;
    }
    return check_launch(launch_gemv_swiglu(x, x_dtype, M, K, qws, scs, zs, out, N, stream, true, plan,
                                           norm ? &np : nullptr),
                        "w4g64 fused gate/up SwiGLU GEMV");
  }
  // Prefill sizes: both projections in one tensor-core launch into scratch
  // (their outputs in the activation dtype, as QuantLinear returns them),
  // then the elementwise SwiGLU.
  const size_t xsize = x_dtype == QI4_DTYPE_F32 ? 4 : 2;
  const size_t bytes = (size_t)M * (size_t)N * xsize;
  const size_t half = (bytes + 255) / 256 * 256;
  void* scratch = nullptr;
  if (scratch_alloc(&scratch, 2 * half, stream) != cudaSuccess) {
    set_error("scratch allocation of %zu bytes failed", 2 * half);
    return QI4_ERR_DEVICE;
  }
  void* g = scratch;
  void* u = static_cast<char*>(scratch) + half;
  void* outs[2] = {g, u};
  const int64_t Ns[2] = {N, N};
  rc = check_launch(launch_gemm_tc_multi(x, x_dtype, M, K, 2, qws, scs, zs, nullptr, QI4_DTYPE_NONE, outs, Ns, stream,
                                         true, info.sms),
                    "w4g64 gate/up tensor-core GEMM");
  if (!rc) rc = check_launch(launch_swiglu_elementwise(g, u, x_dtype, out, M * N, stream, info.sms), "SwiGLU");
  scratch_free(scratch, stream);
  return rc;
}

// The shard's gate/up SwiGLU stored into every rank's gathered buffer
// (peer_exchange.cu), then the epoch published on every rank's flags.
static int gate_up_silu_scatter_impl(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qw_gate,
                                     const uint16_t* sc_gate, const uint8_t* z_gate, const uint8_t* qw_up,
                                     const uint16_t* sc_up, const uint8_t* z_up, int64_t N, float* const* outs,
                                     int64_t ld, int64_t col0, uint32_t* const* flags, int world, int rank,
                                     uint32_t epoch, void* stream_ptr) {
  clear_error();
  if (!outs || !flags || world < 1 || world > kMaxPeers || rank < 0 || rank >= world) {
    set_error("outs and flags must be host arrays of `world` device pointers, 1 <= world <= %d, 0 <= rank < world "
              "(got world=%d rank=%d)", kMaxPeers, world, rank);
    return QI4_ERR_ARGUMENT;
  }
  if (ld <= 0 || col0 < 0 || N < 0 || col0 + N > ld) {
    set_error("the shard's columns [col0, col0 + N) = [%lld, %lld) must lie within the row pitch ld=%lld",
              (long long)col0, (long long)(col0 + N), (long long)ld);
    return QI4_ERR_SHAPE;
  }
  PeerTargets t{};
  for (int p = 0; p < world; ++p) {
    if (!outs[p] || !flags[p] || !aligned(outs[p], 4) || !aligned(flags[p], 4)) {
      set_error("outs[%d] and flags[%d] must be non-null and 4-byte aligned", p, p);
      return QI4_ERR_ARGUMENT;
    }
    t.out[p] = outs[p];
    t.flags[p] = flags[p];
  }
  t.counter = flags[rank] + world;
  t.ld = ld;
  t.col0 = col0;
  t.world = world;
  t.rank = rank;
  t.epoch = epoch;
  DeviceInfo info;
  int rc = current_device(info);
  if (rc) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (N == 0) {  // an empty shard still publishes its epoch
    if (!x || M <= 0) {
      set_error("x must be non-null and M positive");
      return QI4_ERR_ARGUMENT;
    }
    return check_launch(launch_swiglu_scatter(x, x, x_dtype, t, M, 0, stream, info.sms), "SwiGLU scatter");
  }
  rc = validate_linear(x, x_dtype, M, K, qw_gate, sc_gate, nullptr, QI4_DTYPE_NONE, outs[rank], N);
  if (!rc) rc = validate_linear(x, x_dtype, M, K, qw_up, sc_up, nullptr, QI4_DTYPE_NONE, outs[rank], N);
  if (rc) return rc;
  const uint8_t* qws[2] = {qw_gate, qw_up};
  const uint16_t* scs[2] = {sc_gate, sc_up};
  const uint8_t* zs[2] = {z_gate, z_up};
  // gate and up of the shard into scratch, in the activation dtype (what the
  // reference's QuantLinear returns), then the scatter pass.
  const size_t xsize = x_dtype == QI4_DTYPE_F32 ? 4 : 2;
  const size_t half = ((size_t)M * (size_t)N * xsize + 255) / 256 * 256;
  void* scratch = nullptr;
  if (scratch_alloc(&scratch, 2 * half, stream) != cudaSuccess) {
    set_error("scratch allocation of %zu bytes failed", 2 * half);
    return QI4_ERR_DEVICE;
  }
  void* g = scratch;
  void* u = static_cast<char*>(scratch) + half;
  void* gu[2] = {g, u};
  const int64_t Ns[2] = {N, N};
  if (M > kGemvMaxM) {
    rc = check_launch(launch_gemm_tc_multi(x, x_dtype, M, K, 2, qws, scs, zs, nullptr, QI4_DTYPE_NONE, gu, Ns, stream,
                                           true, info.sms),
                      "w4g64 gate/up tensor-core GEMM");
  } else {
    const void* bs[3] = {nullptr, nullptr, nullptr};
    const MmaGemvPlan plan = plan_gemv_mma(M, 2 * ((N + 15) / 16 * 16), K, x_dtype, info.sms);
    if (plan.rows == 0) {
      set_error("no GEMV launch shape fits N=%lld K=%lld", (long long)N, (long long)K);
      rc = QI4_ERR_SHAPE;
    } else {
      rc = check_launch(launch_gemv_mma_multi(x, x_dtype, M, K, 2, qws, scs, zs, bs, QI4_DTYPE_NONE, gu, Ns, stream,
                                              true, plan, nullptr),
                        "w4g64 gate/up GEMV");
    }
  }
  if (!rc) rc = check_launch(launch_swiglu_scatter(g, u, x_dtype, t, M, N, stream, info.sms), "SwiGLU scatter");
  scratch_free(scratch, stream);
  return rc;
}

}  // namespace qi4

using namespace qi4;

extern "C" {

int qi4_w4g64_gate_up_silu_scatter(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qweight_gate,
                                   const uint16_t* scales_gate_f16, const uint8_t* zeros_gate,
                                   const uint8_t* qweight_up, const uint16_t* scales_up_f16, const uint8_t* zeros_up,
                                   int64_t N, float* const* outs, int64_t ld, int64_t col0, uint32_t* const* flags,
                                   int world, int rank, uint32_t epoch, void* stream) {
  return gate_up_silu_scatter_impl(x, x_dtype, M, K, qweight_gate, scales_gate_f16, zeros_gate, qweight_up,
                                   scales_up_f16, zeros_up, N, outs, ld, col0, flags, world, rank, epoch, stream);
}

int qi4_peer_flag_wait(const uint32_t* flags, int world, uint32_t epoch, uint64_t limit_ns, void* stream) {
  clear_error();
  if (!flags || world < 1 || world > kMaxPeers || limit_ns < 1000 || limit_ns > 10000000000ull) {
    set_error("flags must be non-null, 1 <= world <= %d and limit_ns in [1 us, 10 s]", kMaxPeers);
    return QI4_ERR_ARGUMENT;
  }
  DeviceInfo info;
  const int rc = current_device(info);
  if (rc) return rc;
  return check_launch(launch_flag_wait(flags, world, epoch, limit_ns, static_cast<cudaStream_t>(stream)),
                      "peer flag wait");
}

int qi4_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  clear_error();
  if (!ptr || !handle || bytes == 0) {
    set_error("ptr and handle must be non-null and bytes positive");
    return QI4_ERR_ARGUMENT;
  }
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    cudaGetLastError();
    set_error("IPC buffer of %zu bytes: %s", bytes, cudaGetErrorString(e));
    return QI4_ERR_DEVICE;
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return QI4_OK;
}

int qi4_ipc_open(const void* handle, void** ptr) {
  clear_error();
  if (!ptr || !handle) {
    set_error("handle and ptr must be non-null");
    return QI4_ERR_ARGUMENT;
  }
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    return QI4_ERR_DEVICE;
  }
  return QI4_OK;
}

int qi4_ipc_close(void* ptr) {
  clear_error();
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
    return QI4_ERR_DEVICE;
  }
  return QI4_OK;
}

int qi4_ipc_free(void* ptr) {
  clear_error();
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("cudaFree: %s", cudaGetErrorString(e));
    return QI4_ERR_DEVICE;
  }
  return QI4_OK;
}

int qi4_w4g64_gate_up_silu(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qweight_gate,
                           const uint16_t* scales_gate_f16, const uint8_t* zeros_gate, const uint8_t* qweight_up,
                           const uint16_t* scales_up_f16, const uint8_t* zeros_up, float* out, int64_t N,
                           void* stream) {
  return gate_up_silu_impl(x, x_dtype, M, K, qweight_gate, scales_gate_f16, zeros_gate, qweight_up, scales_up_f16,
                           zeros_up, out, N, stream);
}

int qi4_w4g64_linear_multi(const void* x, int x_dtype, int64_t M, int64_t K, int count,
                           const uint8_t* const* qweights, const uint16_t* const* scales_f16,
                           const uint8_t* const* zeros, const void* const* biases, int bias_dtype,
                           void* const* outs, const int64_t* Ns, void* stream) {
  return linear_multi_impl(x, x_dtype, M, K, count, qweights, scales_f16, zeros, biases, bias_dtype, outs, Ns,
                           stream);
}

int qi4_w4g64_linear_multi_norm(const qi4_rmsnorm_prologue* norm, int64_t M, int64_t K, int count,
                                const uint8_t* const* qweights, const uint16_t* const* scales_f16,
                                const uint8_t* const* zeros, const void* const* biases, int bias_dtype,
                                void* const* outs, const int64_t* Ns, void* stream) {
  if (!norm) {
    clear_error();
    set_error("the norm prologue must be non-null");
    return QI4_ERR_ARGUMENT;
  }
  return linear_multi_impl(norm->h_in, QI4_DTYPE_BF16, M, K, count, qweights, scales_f16, zeros, biases, bias_dtype,
                           outs, Ns, stream, norm);
}

int qi4_w4g64_gate_up_silu_norm(const qi4_rmsnorm_prologue* norm, int64_t M, int64_t K,
                                const uint8_t* qweight_gate, const uint16_t* scales_gate_f16,
                                const uint8_t* zeros_gate, const uint8_t* qweight_up,
                                const uint16_t* scales_up_f16, const uint8_t* zeros_up, float* out, int64_t N,
                                void* stream) {
  if (!norm) {
    clear_error();
    set_error("the norm prologue must be non-null");
    return QI4_ERR_ARGUMENT;
  }
  return gate_up_silu_impl(norm->h_in, QI4_DTYPE_BF16, M, K, qweight_gate, scales_gate_f16, zeros_gate, qweight_up,
                           scales_up_f16, zeros_up, out, N, stream, norm);
}

int qi4_w4g64_linear(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qweight,
                     const uint16_t* scales_f16, const uint8_t* zeros, const void* bias, int bias_dtype, void* out,
                     int64_t N, void* stream) {
  return linear_impl(x, x_dtype, M, K, qweight, scales_f16, zeros, bias, bias_dtype, out, N, stream,
                     QI4_ALGO_AUTO, 1);
}

int qi4_w4g64_linear_ex(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qweight,
                        const uint16_t* scales_f16, const uint8_t* zeros, const void* bias, int bias_dtype,
                        void* out, int64_t N, void* stream, int algo, int pdl) {
  return linear_impl(x, x_dtype, M, K, qweight, scales_f16, zeros, bias, bias_dtype, out, N, stream, algo, pdl);
}

int qi4_w4g64_dequant_f32(const uint8_t* qweight, const uint16_t* scales_f16, const uint8_t* zeros, float* out,
                          int64_t N, int64_t K, void* stream) {
  clear_error();
  if (!qweight || !scales_f16 || !out) {
    set_error("qweight, scales and out must be non-null device pointers");
    return QI4_ERR_ARGUMENT;
  }
  if (N <= 0 || K <= 0) {
    set_error("N and K must be positive");
    return QI4_ERR_ARGUMENT;
  }
  if (K % kGroup) {
    set_error("canonical W4G64 dequantization requires K divisible by 64 (got K=%lld)", (long long)K);
    return QI4_ERR_SHAPE;
  }
  if (!aligned(qweight, 16) || !aligned(out, 16) || !aligned(scales_f16, 2)) {
    set_error("qweight and out must be 16-byte aligned");
    return QI4_ERR_ALIGNMENT;
  }
  DeviceInfo info;
  int rc = current_device(info);
  if (rc) return rc;
  return check_launch(launch_dequant_f32(qweight, scales_f16, zeros, out, N, K, static_cast<cudaStream_t>(stream),
                                         info.sms),
                      "w4g64 dequant");
}

int qi4_w4_unpack(const uint8_t* packed, int8_t* out, int64_t elements, void* stream) {
  clear_error();
  if (elements < 0) {
    set_error("elements must be non-negative");
    return QI4_ERR_ARGUMENT;
  }
  if (elements == 0) return QI4_OK;
  if (!packed || !out) {
    set_error("packed and out must be non-null device pointers");
    return QI4_ERR_ARGUMENT;
  }
  if (!aligned(packed, 16) || !aligned(out, 16)) {
    set_error("packed and out must be 16-byte aligned");
    return QI4_ERR_ALIGNMENT;
  }
  DeviceInfo info;
  int rc = current_device(info);
  if (rc) return rc;
  return check_launch(launch_unpack(packed, out, elements, static_cast<cudaStream_t>(stream), info.sms),
                      "int4 unpack");
}

int qi4_gemv_plan_override(int lanes_per_row, int warps, int ksplit, int depth) {
  clear_error();
  if (lanes_per_row == 0) {
    set_gemv_override(0, 0, 0, 0);
    return QI4_OK;
  }
  const bool ok = (lanes_per_row == 8 || lanes_per_row == 16 || lanes_per_row == 32) &&
                  (warps == 4 || warps == 8) && ksplit >= 1 && ksplit <= 8 && (depth == 4 || depth == 8);
  if (!ok) {
    set_error("invalid GEMV plan override (lanes_per_row %d, warps %d, ksplit %d, depth %d)", lanes_per_row,
              warps, ksplit, depth);
    return QI4_ERR_ARGUMENT;
  }
  set_gemv_override(lanes_per_row, warps, ksplit, depth);
  return QI4_OK;
}

int qi4_gemv_mma_plan(int64_t M, int64_t N, int64_t K, int x_dtype, int num_sms, int64_t* plan) {
  clear_error();
  if (plan == nullptr || num_sms <= 0 || N <= 0) {
    set_error("qi4_gemv_mma_plan: plan must be non-null, N and num_sms positive");
    return QI4_ERR_ARGUMENT;
  }
  if (!gemv_mma_supported(M, K)) {
    set_error("qi4_gemv_mma_plan: no GEMV plan for M=%lld K=%lld", (long long)M, (long long)K);
    return QI4_ERR_SHAPE;
  }
  const MmaGemvPlan p = plan_gemv_mma(M, N, K, x_dtype, num_sms);
  if (p.rows == 0) {
    set_error("qi4_gemv_mma_plan: no plan fits shared memory");
    return QI4_ERR_SHAPE;
  }
  plan[0] = p.rows;
  plan[1] = p.ksplit;
  plan[2] = p.warps;
  plan[3] = p.boxes_per_split;
  plan[4] = (int64_t)p.smem;
  plan[5] = p.pre;
  return QI4_OK;
}

int qi4_gemm_tc_plan_override(int bn, int ksplit) {
  clear_error();
  if (bn == 0) {
    set_gemm_tc_override(0, 0);
    return QI4_OK;
  }
  if ((bn != 32 && bn != 64 && bn != 128 && bn != 192 && bn != 256) || ksplit < 1 || ksplit > 8 ||
      (ksplit > 1 && bn > 128)) {
    set_error("invalid tensor-core GEMM plan override (bn %d, ksplit %d)", bn, ksplit);
    return QI4_ERR_ARGUMENT;
  }
  set_gemm_tc_override(bn, ksplit);
  return QI4_OK;
}

int qi4_gemv_mma_plan_override(int rows, int ksplit, int warps) {
  clear_error();
  if (rows == 0) {
    set_gemv_mma_override(0, 0, 0);
    return QI4_OK;
  }
  if ((rows != 16 && rows != 32 && rows != 64 && rows != 128) || ksplit < 1 || ksplit > 8 ||
      (warps != 2 && warps != 4 && warps != 8 && warps != 16 && warps != 32) || rows / 16 > warps) {
    set_error("invalid GEMV plan override (rows %d, ksplit %d, warps %d)", rows, ksplit, warps);
    return QI4_ERR_ARGUMENT;
  }
  set_gemv_mma_override(rows, ksplit, warps);
  return QI4_OK;
}

int qi4_device_status(void* stream) {
  clear_error();
  const int v1 = read_gemv_mma_error(static_cast<cudaStream_t>(stream));
  const int v2 = read_gemm_tc_error(static_cast<cudaStream_t>(stream));
  const int v3 = read_chain_error(static_cast<cudaStream_t>(stream));
  const int v4 = read_attention_error(static_cast<cudaStream_t>(stream));
  const int v5 = read_peer_error(static_cast<cudaStream_t>(stream));
  const int v = (v1 < 0 || v2 < 0 || v3 < 0 || v4 < 0 || v5 < 0) ? -1 : (v1 | v2 | v3 | v4 | v5);
  if (v < 0) {
    set_error("cannot read the device error flags: %s", cudaGetErrorString(cudaGetLastError()));
    return QI4_ERR_LAUNCH;
  }
  return v;
}

int qi4_selftest_bounded_wait(uint64_t limit_ns, void* stream) {
  clear_error();
  if (limit_ns < 1000 || limit_ns > 1000000000ull) {
    set_error("limit_ns must lie in [1 us, 1 s] (got %llu ns)", (unsigned long long)limit_ns);
    return QI4_ERR_ARGUMENT;
  }
  DeviceInfo info;
  const int rc = current_device(info);
  if (rc) return rc;
  return check_launch(launch_bounded_wait_selftest(limit_ns, static_cast<cudaStream_t>(stream)),
                      "bounded-wait self-test");
}

int qi4_w4g64_linear_f32_noalloc(const float* x, int64_t M, int64_t K, const uint8_t* qweight,
                                 const uint16_t* scales_f16, const uint8_t* zeros, const void* bias, int bias_dtype,
                                 float* out, int64_t N, void* stream) {
  clear_error();
  int rc = validate_linear(x, QI4_DTYPE_F32, M, K, qweight, scales_f16, bias, bias_dtype, out, N);
  if (rc) return rc;
  const size_t need = 2 * (size_t)M * (size_t)K * 2;
  if (need > static_scratch_bytes()) {
    set_error("M*K = %lld exceeds the fixed scratch of this entry point: it holds %zu bytes (M*K <= %zu); "
              "use qi4_w4g64_linear for larger inputs",
              (long long)(M * K), static_scratch_bytes(), static_scratch_bytes() / 4);
    return QI4_ERR_SHAPE;
  }
  DeviceInfo info;
  rc = current_device(info);
  if (rc) return rc;
  if (!bias) bias_dtype = QI4_DTYPE_NONE;
  return check_launch(launch_gemm_tc_f32_static(x, M, K, qweight, scales_f16, zeros, bias, bias_dtype, out, N,
                                                static_cast<cudaStream_t>(stream), info.sms),
                      "w4g64 allocation-free FP32 GEMM");
}

int qi4_last_error(char* buf, size_t len) {
  const std::string& s = g_last_error;
  if (buf && len) {
    const size_t n = s.size() < len - 1 ? s.size() : len - 1;
    memcpy(buf, s.data(), n);
    buf[n] = '\0';
  }
  return (int)s.size();
}

int qi4_version(void) { return 100; }

}  // extern "C"
