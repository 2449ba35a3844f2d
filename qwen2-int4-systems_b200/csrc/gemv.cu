// Fused unpack + group-dequant W4G64 GEMV for decode (M <= 16), sm_100a.
//
// Replaces, for small M, the fused gather-decode-dequant loop of
// _linear_canonical_w4g64_kernel (reference src/qwen_int4/triton_kernels.py:66-116)
// with the numerics of torch_reference_linear (src/qwen_int4/backends.py:73-98):
// FP32 dequantised weights, FP32 accumulation, FP32 bias, final cast.
//
// Work split
//   * A CTA owns `rows_per_cta` consecutive output features (rows of W) and one
//     K slice. A row is read by LPR lanes of one warp, lane j of the row taking
//     16-byte chunks j, j+LPR, ... (32 codes = half of a 64-group per chunk), so
//     each warp-wide load covers LPR*16 contiguous bytes of each of 32/LPR rows.
//   * The kernel is bound by memory latency as much as by bandwidth (a 7 MB
//     weight is about one DRAM round trip per SM), so every lane keeps a ring of
//     D chunk loads in flight, issued before anything else - before
//     griddepcontrol.wait under programmatic dependent launch, so a chain of
//     linears streams the next layer's weights during the previous one's tail.
//   * The CTA's K slice of x is staged once in shared memory as FP32 (chunk
//     rows padded to 36 floats, which keeps the 16-byte LDS of lanes that read
//     different chunks free of bank conflicts).
//   * Code expansion: one LOP3 per 4 codes and one PRMT per code turn a packed
//     nibble into f = 1 + (c + 8)/16; then w = fma(f, 16 s, -(24 + z) s) is the
//     reference's FP32 weight (c - z) * s exactly (every product and the sum
//     are representable), and the dot product accumulates in FP32.
//   * Row partials are combined with warp shuffles; K slices of one row tile
//     form a thread-block cluster and are summed over distributed shared
//     memory by the cluster's rank-0 CTA, which adds the bias and stores.
#include <cooperative_groups.h>

#include <algorithm>
#include <cmath>

#include "gemv.cuh"
#include "qi4_common.cuh"

namespace cg = cooperative_groups;

namespace qi4 {

namespace {

constexpr int kPad = 36;  // floats per staged 32-element chunk

struct GemvArgs {
  const void* x;
  int x_dtype;
  int M;
  int64_t K;
  const uint8_t* qweight;
  const __half* scales;
  const uint8_t* zeros;
  const void* bias;
  int bias_dtype;
  void* out;
  int64_t N;
  int chunks_per_split;  // 32-code chunks of K handled by one CTA
  int rows_per_cta;
};

// Scale/zero terms of a chunk: w = fma(f, s16, nz) with s16 = 16 s and
// nz = -(24 + z) s, both exact in FP32.
__device__ __forceinline__ void load_chunk(const GemvArgs& a, const uint8_t* qrow, const __half* srow,
                                           int64_t zrow, int c, uint4& q, float& s16, float& nz) {
  q = ldg_stream16(qrow + (int64_t)c * kChunkBytes);
  const float sc = __half2float(__ldg(srow + (c >> 1)));
  const int z = load_zero(a.zeros, zrow + (c >> 1));
  s16 = 16.0f * sc;
  nz = -static_cast<float>(24 + z) * sc;
}

// Accumulate one 32-code chunk into acc[0..MT).
template <int MT>
__device__ __forceinline__ void consume_chunk(const uint4& q, float s16, float nz, const float* xs_chunk,
                                              int m_stride, float (&acc)[MT]) {
  const uint32_t words[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    uint32_t lo, hi;
    expand_nibbles(words[w], lo, hi);
    const float w0 = fmaf(nibble_float<0>(lo), s16, nz), w1 = fmaf(nibble_float<0>(hi), s16, nz);
    const float w2 = fmaf(nibble_float<1>(lo), s16, nz), w3 = fmaf(nibble_float<1>(hi), s16, nz);
    const float w4 = fmaf(nibble_float<2>(lo), s16, nz), w5 = fmaf(nibble_float<2>(hi), s16, nz);
    const float w6 = fmaf(nibble_float<3>(lo), s16, nz), w7 = fmaf(nibble_float<3>(hi), s16, nz);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float4* xv = reinterpret_cast<const float4*>(xs_chunk + m * m_stride) + 2 * w;
      const float4 u = xv[0], v = xv[1];
      float t = acc[m];
      t = fmaf(w0, u.x, t);
      t = fmaf(w1, u.y, t);
      t = fmaf(w2, u.z, t);
      t = fmaf(w3, u.w, t);
      t = fmaf(w4, v.x, t);
      t = fmaf(w5, v.y, t);
      t = fmaf(w6, v.z, t);
      t = fmaf(w7, v.w, t);
      acc[m] = t;
    }
  }
}

template <int MT, int LPR, int D>
__global__ void __launch_bounds__(256) w4g64_gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) float smem[];
  const int nch = a.chunks_per_split;
  const int C = (int)(a.K / kChunkCodes);
  const int c_begin = blockIdx.y * nch;
  const int c_end = C < c_begin + nch ? C : c_begin + nch;
  const int nloc = c_end - c_begin;
  float* xs = smem;                    // [MT][nch][kPad]
  float* part = xs + MT * nch * kPad;  // [MT][rows_per_cta] (split-K only)

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  constexpr int RPW = 32 / LPR;
  const int row_in_cta = (tid >> 5) * RPW + lane / LPR;
  const int sub = lane % LPR;
  const int64_t row = (int64_t)blockIdx.x * a.rows_per_cta + row_in_cta;
  const bool row_ok = row < a.N;
  const int64_t G = a.K / kGroup;
  const int c0 = c_begin + sub;
  const int iters = (row_ok && c0 < c_end) ? (c_end - c0 + LPR - 1) / LPR : 0;
  const uint8_t* qrow = a.qweight + (row_ok ? row : 0) * (a.K >> 1);
  const __half* srow = a.scales + (row_ok ? row : 0) * G;
  const int64_t zrow = (row_ok ? row : 0) * G;

  // Weights do not depend on the previous kernel: put D chunks in flight first.
  uint4 q[D];
  float s16[D], nz[D];
#pragma unroll
  for (int i = 0; i < D; ++i)
    if (i < iters) load_chunk(a, qrow, srow, zrow, c0 + i * LPR, q[i], s16[i], nz[i]);
  pdl_wait();

  // Stage x[:, slice] as FP32 (rows m >= M are zero).
  const int64_t k0 = (int64_t)c_begin * kChunkCodes;
  const int quads = nloc * (kChunkCodes / 4);
  for (int i = tid; i < MT * quads; i += blockDim.x) {
    const int m = i / quads, j = i - m * quads;
    const int ch = j >> 3, e = (j & 7) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (m < a.M) v = load4_as_f32(a.x, a.x_dtype, (int64_t)m * a.K + k0 + ch * kChunkCodes + e);
    *reinterpret_cast<float4*>(xs + (m * nch + ch) * kPad + e) = v;
  }
  __syncthreads();
  pdl_launch_dependents();

  float acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = 0.f;
  for (int base = 0; base < iters; base += D) {
#pragma unroll
    for (int i = 0; i < D; ++i) {
      const int it = base + i;
      if (it < iters) {
        consume_chunk<MT>(q[i], s16[i], nz[i], xs + (c0 + it * LPR - c_begin) * kPad, nch * kPad, acc);
        if (it + D < iters) load_chunk(a, qrow, srow, zrow, c0 + (it + D) * LPR, q[i], s16[i], nz[i]);
      }
    }
  }

#pragma unroll
  for (int m = 0; m < MT; ++m) {
#pragma unroll
    for (int off = LPR / 2; off > 0; off >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], off);
  }

  if (gridDim.y == 1) {
    if (row_ok && sub == 0) {
      const float b = a.bias ? load_as_f32(a.bias, a.bias_dtype, row) : 0.f;
#pragma unroll
      for (int m = 0; m < MT; ++m)
        if (m < a.M) store_from_f32(a.out, a.x_dtype, (int64_t)m * a.N + row, acc[m] + b);
    }
    return;
  }

  // Split-K: the CTAs of one row tile form a cluster along y.
  if (sub == 0) {
#pragma unroll
    for (int m = 0; m < MT; ++m) part[m * a.rows_per_cta + row_in_cta] = acc[m];
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  if (cluster.block_rank() == 0) {
    const int nranks = (int)cluster.num_blocks();
    for (int i = tid; i < a.M * a.rows_per_cta; i += blockDim.x) {
      const int m = i / a.rows_per_cta, r = i - m * a.rows_per_cta;
      const int64_t orow = (int64_t)blockIdx.x * a.rows_per_cta + r;
      if (orow >= a.N) continue;
      float sum = 0.f;
      for (int rk = 0; rk < nranks; ++rk) sum += cluster.map_shared_rank(part, rk)[m * a.rows_per_cta + r];
      const float b = a.bias ? load_as_f32(a.bias, a.bias_dtype, orow) : 0.f;
      store_from_f32(a.out, a.x_dtype, (int64_t)m * a.N + orow, sum + b);
    }
  }
  cluster.sync();  // keep every CTA's shared memory alive until rank 0 is done
}

template <int MT, int LPR, int D>
cudaError_t launch_one(const GemvArgs& a, int warps, int ksplit, size_t smem, cudaStream_t stream, bool pdl) {
  auto kernel = w4g64_gemv_kernel<MT, LPR, D>;
  // Function attributes are per device: remember which devices are set up.
  static unsigned long long configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured |= bit;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((a.N + a.rows_per_cta - 1) / a.rows_per_cta), (unsigned)ksplit, 1);
  cfg.blockDim = dim3(32 * warps, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int n = 0;
  attrs[n].id = cudaLaunchAttributeClusterDimension;
  attrs[n].val.clusterDim.x = 1;
  attrs[n].val.clusterDim.y = (unsigned)ksplit;
  attrs[n].val.clusterDim.z = 1;
  ++n;
  if (pdl) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, a);
}

template <int MT, int LPR>
cudaError_t launch_d(const GemvArgs& a, int depth, int warps, int ksplit, size_t smem, cudaStream_t s, bool pdl) {
  return depth >= 8 ? launch_one<MT, LPR, 8>(a, warps, ksplit, smem, s, pdl)
                    : launch_one<MT, LPR, 4>(a, warps, ksplit, smem, s, pdl);
}

template <int MT>
cudaError_t launch_mt(const GemvArgs& a, const GemvPlan& p, cudaStream_t s, bool pdl) {
  switch (p.lpr) {
    case 8: return launch_d<MT, 8>(a, p.depth, p.warps, p.ksplit, p.smem, s, pdl);
    case 16: return launch_d<MT, 16>(a, p.depth, p.warps, p.ksplit, p.smem, s, pdl);
    default: return launch_d<MT, 32>(a, p.depth, p.warps, p.ksplit, p.smem, s, pdl);
  }
}

}  // namespace

namespace {
thread_local GemvPlan g_override{};  // tuning hook (qi4_gemv_plan_override)
}

void set_gemv_override(int lpr, int warps, int ksplit, int depth) {
  g_override = GemvPlan{};
  g_override.lpr = lpr;
  g_override.warps = warps;
  g_override.ksplit = ksplit;
  g_override.depth = depth;
}

static GemvPlan make_plan(int mt, int64_t N, int64_t K, int lpr, int warps, int ks, int depth) {
  const int64_t C = K / kChunkCodes;
  GemvPlan p{};
  p.mt = mt;
  p.lpr = lpr;
  p.warps = warps;
  p.ksplit = ks;
  p.depth = depth;
  p.chunks_per_split = (int)((C + ks - 1) / ks);
  p.rows_per_cta = warps * (32 / lpr);
  p.smem = (size_t)mt * p.chunks_per_split * kPad * sizeof(float) +
           (ks > 1 ? (size_t)mt * p.rows_per_cta * sizeof(float) : 0);
  return p;
}

GemvPlan plan_gemv(int64_t M, int64_t N, int64_t K, int num_sms) {
  const int mt = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : M <= 8 ? 8 : 16;
  const int64_t C = K / kChunkCodes;
  if (g_override.lpr) {
    GemvPlan p = make_plan(mt, N, K, g_override.lpr, g_override.warps, g_override.ksplit, g_override.depth);
    return p.smem <= 200 * 1024 ? p : GemvPlan{};
  }
  // Latency/bandwidth model: the kernel time is the largest of the HBM time,
  // the number of DRAM round trips the resident loads need, and the issue
  // time of the expansion + FMA work; a K split adds a cluster reduction.
  const double bytes = (double)N * (double)K / 2.0;
  const double hbm = 6.5e12, latency = 0.8e-6, issue = (double)num_sms * 4 * 1.8e9;
  GemvPlan best{};
  double best_t = 1e30;
  for (int lpr : {8, 16, 32}) {
    for (int ks = 1; ks <= 8; ++ks) {
      if (ks > 1 && C % ks) continue;
      for (int depth : {4, 8}) {
        const int warps = 4;
        const GemvPlan p = make_plan(mt, N, K, lpr, warps, ks, depth);
        if (p.smem > 200 * 1024) continue;
        const int64_t iters = (p.chunks_per_split + lpr - 1) / lpr;
        const double lane_eff = (double)p.chunks_per_split / (double)(iters * lpr);
        // Registers per thread from ptxas (-Xptxas -v) for MT = 1, 2, 4, 8, 16.
        static const int kRegs4[5] = {60, 64, 71, 98, 128}, kRegs8[5] = {78, 80, 102, 128, 164};
        const int mi = mt == 1 ? 0 : mt == 2 ? 1 : mt == 4 ? 2 : mt == 8 ? 3 : 4;
        const int regs = depth >= 8 ? kRegs8[mi] : kRegs4[mi];
        int per_sm = 2048 / (32 * warps);
        per_sm = std::min(per_sm, (int)(65536 / (32 * warps * regs)));
        per_sm = std::min(per_sm, (int)((227 * 1024) / (p.smem + 1024)));
        per_sm = std::max(1, std::min(per_sm, 32));
        const int64_t ctas = ((N + p.rows_per_cta - 1) / p.rows_per_cta) * ks;
        const double resident = std::min<double>((double)ctas, (double)num_sms * per_sm);
        const double in_flight = resident * 32 * warps * std::min<int64_t>(iters, depth) * kChunkBytes;
        const double waves = std::ceil((double)ctas / ((double)num_sms * per_sm));
        const double t_lat = std::max(1.0, bytes / in_flight) * latency * std::max(1.0, waves * 0.5);
        const double t_bw = bytes / hbm;
        const double t_issue = (double)N * (double)K * (2.0 + mt) / 32.0 / lane_eff / issue;
        const double t = std::max(std::max(t_lat, t_bw), t_issue) + (ks > 1 ? 0.4e-6 : 0.0) + 1e-9 * depth;
        if (t < best_t) {
          best_t = t;
          best = p;
        }
      }
    }
  }
  return best;
}

cudaError_t launch_gemv(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qweight,
                        const uint16_t* scales, const uint8_t* zeros, const void* bias, int bias_dtype,
                        void* out, int64_t N, cudaStream_t stream, bool pdl, const GemvPlan& p) {
  GemvArgs a;
  a.x = x;
  a.x_dtype = x_dtype;
  a.M = (int)M;
  a.K = K;
  a.qweight = qweight;
  a.scales = reinterpret_cast<const __half*>(scales);
  a.zeros = zeros;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.out = out;
  a.N = N;
  a.chunks_per_split = p.chunks_per_split;
  a.rows_per_cta = p.rows_per_cta;
  switch (p.mt) {
    case 1: return launch_mt<1>(a, p, stream, pdl);
    case 2: return launch_mt<2>(a, p, stream, pdl);
    case 4: return launch_mt<4>(a, p, stream, pdl);
    case 8: return launch_mt<8>(a, p, stream, pdl);
    default: return launch_mt<16>(a, p, stream, pdl);
  }
}

}  // namespace qi4
