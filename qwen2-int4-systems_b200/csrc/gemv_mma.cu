// Decode GEMV (M <= 16): TMA-staged packed weights, register nibble expansion,
// warp-level tensor-core dot products, FP32 group scaling. sm_100a.
//
// Replaces, for small M, _linear_canonical_w4g64_kernel (reference
// src/qwen_int4/triton_kernels.py:66-116) with the numerics of
// torch_reference_linear (src/qwen_int4/backends.py:73-98).
//
// Data path per CTA (R = 16/32/64 output rows, one K slice of whole 128-byte
// boxes = 4 groups each):
//   1. One thread issues the CTA's whole weight slab as 2-D TMA boxes of
//      [R rows x 128 B] with 128-byte swizzle into shared memory, before
//      anything else and before griddepcontrol.wait; the kernel then triggers
//      its dependents at once, so in a chain of linears the next layers' weight
//      slabs stream while this one computes (cascaded programmatic launch).
//   2. Group scales and zero points of the slab go to a shared table.
//   3. Each warp owns a 16-row block and a range of groups. Per group a lane
//      reads 8 packed bytes of rows g and g+8 (16 codes each) from shared
//      memory and expands each byte into a bf16x2 / f16x2 pair of exact
//      integers (c - z): XOR 0x8, PRMT + LOP3 into the 0x43xx (bf16) or
//      0x64xx (f16) magic exponent, one packed subtract of (magic + z).
//   4. Four m16n8k16 MMAs per group multiply the exact (c - z) fragment by the
//      activations (bf16/f16 as given; FP32 activations as a bf16 hi + lo
//      pair, two MMAs), accumulating in FP32; the per-row group scale is then
//      applied in FP32: acc += scale * D. Products are exact and sums are
//      FP32, as in the reference's dequantise-then-matmul.
//   5. Warps that split K reduce through shared memory; CTAs that split K form
//      a cluster and reduce over distributed shared memory. Bias is added in
//      FP32 and the result is cast to the activation dtype.
// The reduction over K happens inside the MMAs (the tensor pipe replaces the
// CUDA-core FMAs and shuffles of a scalar GEMV); the kernel is bound by HBM.
#include <cooperative_groups.h>

#include <algorithm>
#include <cmath>

#include "gemv_mma.cuh"
#include "qi4_common.cuh"
#include "tma_util.cuh"

namespace cg = cooperative_groups;

namespace qi4 {

__device__ int g_gemv_mma_error;

namespace {

constexpr int kThreads = 256;   // 8 warps
constexpr int kBoxBytes = 128;  // inner TMA box: 128 bytes = 256 codes = 4 groups
constexpr int kGroupsPerBox = 4;
constexpr int kPreGroups = 4;  // groups per warp expanded before the dependency wait

constexpr int kMaxMats = 3;  // weight matrices sharing one activation block per launch

// One weight matrix of a launch (several share the activations: q/k/v, gate/up).
struct Mat {
  const __half* scales;
  const uint8_t* zeros;
  const void* bias;
  void* out;
  int64_t N;
};

struct Args {
  const void* x;
  int M;
  int64_t K;
  Mat mat[kMaxMats];
  int tiles_end[kMaxMats];  // cumulative row tiles: matrix m owns tiles [tiles_end[m-1], tiles_end[m])
  int nmats;
  int bias_dtype;
  int rows;             // R
  int rows_log2;
  int boxes_per_split;  // boxes along K per CTA
  int copy_log2;        // log2 of the 128-byte boxes fetched per TMA copy
  int three_d;          // 1: 3-D box-major copies (rows of K/2 bytes a multiple of 128); 0: 2-D, one box each
  int G;                // groups per row (K / 64)
  int has_norm;         // 1: x is formed from `norm` while staging (bf16 activations)
  NormPrologue norm;
};

struct TableEntry {
  float scale;
  uint32_t zc2;  // packed (magic + z, magic + z) in the MMA operand type
};

template <int XT>
struct Fmt;
template <>
struct Fmt<QI4_DTYPE_BF16> {  // bf16 operands: 0x4300 | v == 128 + v
  static constexpr uint32_t kMagic = 0x43004300u;
  static constexpr int kBase = 136;  // 128 + 8 (codes are stored + 8 after the XOR)
};
template <>
struct Fmt<QI4_DTYPE_F16> {  // f16 operands: 0x6400 | v == 1024 + v
  static constexpr uint32_t kMagic = 0x64006400u;
  static constexpr int kBase = 1032;
};
template <>
struct Fmt<QI4_DTYPE_F32> : Fmt<QI4_DTYPE_BF16> {};

template <int XT>
__device__ __forceinline__ uint32_t sub2(uint32_t a, uint32_t b) {
  uint32_t d;
  if constexpr (XT == QI4_DTYPE_F16)
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Nibbles i and i+4 of word w -> packed pair (magic + c_i + 8, magic + c_{i+4} + 8):
// one LOP3 does the mask, the XOR 8 that turns the two's-complement nibble
// into c + 8, and the OR of the magic exponent ((n & 0xF) ^ 0x8 | magic ==
// (n & 0xF) ^ (0x8 | magic) because the magic bits are clear in the nibble).
template <int XT>
__device__ __forceinline__ uint32_t nibble_pair(uint32_t w_shifted) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;"  // (a & b) ^ c
      : "=r"(d)
      : "r"(w_shifted), "r"(0x000F000Fu), "r"(Fmt<XT>::kMagic | 0x00080008u));
  return d;
}

// Word w (8 codes) -> four operand registers holding code pairs
// (i, i+4), i = 0..3, each minus (magic + 8 + z) = exact (c - z).
template <int XT>
__device__ __forceinline__ void expand_word(uint32_t w, uint32_t zc2, uint32_t* r) {
  r[0] = sub2<XT>(nibble_pair<XT>(w), zc2);
  r[1] = sub2<XT>(nibble_pair<XT>(w >> 4), zc2);
  r[2] = sub2<XT>(nibble_pair<XT>(w >> 8), zc2);
  r[3] = sub2<XT>(nibble_pair<XT>(w >> 12), zc2);
}

// Packed (magic + 8 + z, magic + 8 + z) in the operand type (exact integers).
template <int XT>
__device__ __forceinline__ uint32_t zero_code(int z) {
  const int v = Fmt<XT>::kBase + z;
  const uint32_t bits = XT == QI4_DTYPE_F16 ? (uint32_t)__half_as_ushort(__int2half_rn(v))
                                            : (uint32_t)__bfloat16_as_ushort(__int2bfloat16_rn(v));
  return bits | (bits << 16);
}

template <int XT>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (XT == QI4_DTYPE_F16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

__device__ __forceinline__ uint32_t prmt_lo(uint32_t a, uint32_t b) {  // (a.lo16, b.lo16)
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t prmt_hi(uint32_t a, uint32_t b) {  // (a.hi16, b.hi16)
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Activations are staged once per CTA in shared memory, right after the
// dependency wait (one round trip to L2 for the whole K slice), already in
// the k order of the weight fragments. Those pair codes (i, i+4) of each
// 8-code word, so within every 8 consecutive elements the staged order is
// x0 x4 x1 x5 x2 x6 x3 x7 and each B register of a k-step is one aligned
// 32-bit word: lane tq of token t reads its 16 elements of group g as two
// 16-byte words at t * xstride + 128 g + 32 tq. FP32 activations are staged
// as a bf16 hi plane followed by a lo plane (x - hi, rounded), 128 gs bytes
// each. The token stride is padded by 16 bytes so that the 8 tokens of a
// quarter-warp hit distinct banks.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// MULTI: also stage 2..8 chunks per thread through registers (unrolled; kept
// out of kernels whose post-wait code should stay short).
template <int XT, bool MULTI>
__device__ __forceinline__ void stage_x(const Args& a, uint8_t* xs, int xstride, int g0, int gs, int tid,
                                        int nthreads) {
  const int per_tok = gs * 8;  // 8-element chunks per token
  const int total = a.M * per_tok;
  const uint32_t base = smem_addr(xs);
  constexpr int kRegChunks = 8;  // chunks per thread staged through registers
  if (XT != QI4_DTYPE_F32 && total <= nthreads) {
    // One chunk per thread at most: load, permute, store.
    if (tid < total) {
      const int tok = a.M == 1 ? 0 : tid / per_tok, c = tid - tok * per_tok;
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(static_cast<const unsigned short*>(a.x) +
                                                           (int64_t)tok * a.K + (int64_t)g0 * kGroup + c * 8));
      sts128(base + tok * xstride + c * 16,
             make_uint4(prmt_lo(v.x, v.z), prmt_hi(v.x, v.z), prmt_lo(v.y, v.w), prmt_hi(v.y, v.w)));
    }
  } else if (MULTI && XT != QI4_DTYPE_F32 && total <= kRegChunks * nthreads) {
    // Up to kRegChunks chunks per thread: all loads first (one round trip),
    // then permute and store.
    uint4 v[kRegChunks];
#pragma unroll
    for (int u = 0; u < kRegChunks; ++u) {
      const int i = tid + u * nthreads;
      if (i < total) {
        const int tok = a.M == 1 ? 0 : i / per_tok, c = i - tok * per_tok;
        v[u] = __ldg(reinterpret_cast<const uint4*>(static_cast<const unsigned short*>(a.x) + (int64_t)tok * a.K +
                                                    (int64_t)g0 * kGroup + c * 8));
      }
    }
#pragma unroll
    for (int u = 0; u < kRegChunks; ++u) {
      const int i = tid + u * nthreads;
      if (i < total) {
        const int tok = a.M == 1 ? 0 : i / per_tok, c = i - tok * per_tok;
        sts128(base + tok * xstride + c * 16, make_uint4(prmt_lo(v[u].x, v[u].z), prmt_hi(v[u].x, v[u].z),
                                                         prmt_lo(v[u].y, v[u].w), prmt_hi(v[u].y, v[u].w)));
      }
    }
  } else if constexpr (XT != QI4_DTYPE_F32) {
    // Asynchronous 16-byte copies straight into place (all in flight at
    // once), then each thread permutes the chunks it copied.
    for (int i = tid; i < total; i += nthreads) {
      const int tok = a.M == 1 ? 0 : i / per_tok, c = i - tok * per_tok;
      cp_async16(base + tok * xstride + c * 16,
                 static_cast<const unsigned short*>(a.x) + (int64_t)tok * a.K + (int64_t)g0 * kGroup + c * 8);
    }
    cp_async_wait_all();
    for (int i = tid; i < total; i += nthreads) {
      const int tok = a.M == 1 ? 0 : i / per_tok, c = i - tok * per_tok;
      const uint32_t at = base + tok * xstride + c * 16;
      const uint4 v = lds128(at);
      sts128(at, make_uint4(prmt_lo(v.x, v.z), prmt_hi(v.x, v.z), prmt_lo(v.y, v.w), prmt_hi(v.y, v.w)));
    }
  } else {
    // FP32: through registers (bf16 hi and lo planes), several loads in flight.
#pragma unroll 4
    for (int i = tid; i < total; i += nthreads) {
      const int tok = a.M == 1 ? 0 : i / per_tok, c = i - tok * per_tok;
      const int64_t e = (int64_t)tok * a.K + (int64_t)g0 * kGroup + (int64_t)c * 8;
      const float4 v0 = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + e));
      const float4 v1 = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + e) + 1);
      const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      uint32_t w[4], l[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        w[q] = pack_bf16x2(v[2 * q], v[2 * q + 1]);
        l[q] = pack_bf16x2(v[2 * q] - __uint_as_float(w[q] << 16), v[2 * q + 1] - __uint_as_float(w[q] & 0xFFFF0000u));
      }
      sts128(base + tok * xstride + c * 16,
             make_uint4(prmt_lo(w[0], w[2]), prmt_hi(w[0], w[2]), prmt_lo(w[1], w[3]), prmt_hi(w[1], w[3])));
      sts128(base + tok * xstride + gs * 128 + c * 16,
             make_uint4(prmt_lo(l[0], l[2]), prmt_hi(l[0], l[2]), prmt_lo(l[1], l[3]), prmt_hi(l[1], l[3])));
    }
  }
}

// The decoder-block boundary folded into the staging (bf16 activations):
// hn = bf16(h_in + bf16(delta)) (delta absent: hn = h_in), then
// x = bf16(bf16(hn * rsqrt(mean(hn^2) + eps)) * w), the reference's residual
// add and RMSNorm (src/qwen_int4/model.py:31-42,151-159) with FP32
// statistics. Every CTA sums its tokens' whole rows (from L2), then forms
// and stages its own K slice; the CTAs of the first row tile (blockIdx.x ==
// 0: one per K slice) also write hn to h_out, which must not alias h_in
// (other CTAs still read h_in).
__device__ __forceinline__ void residual8(const NormPrologue& nm, int64_t e, float (&v)[8]) {
  const uint4 hw = __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(nm.h_in) + e));
  const uint32_t hs[4] = {hw.x, hw.y, hw.z, hw.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    v[2 * q] = __uint_as_float(hs[q] << 16);
    v[2 * q + 1] = __uint_as_float(hs[q] & 0xFFFF0000u);
  }
  if (nm.delta == nullptr) return;
  float d[8];
  if (nm.delta_dtype == QI4_DTYPE_F32) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(nm.delta) + e));
    const float4 b = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(nm.delta) + e) + 1);
    const float t[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) d[j] = __bfloat162float(__float2bfloat16_rn(t[j]));
  } else {
    const uint4 dw = __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(nm.delta) + e));
    const uint32_t ds[4] = {dw.x, dw.y, dw.z, dw.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      d[2 * q] = __uint_as_float(ds[q] << 16);
      d[2 * q + 1] = __uint_as_float(ds[q] & 0xFFFF0000u);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = __bfloat162float(__float2bfloat16_rn(v[j] + d[j]));
}

__device__ __forceinline__ void stage_x_norm(const Args& a, uint8_t* xs, int xstride, int g0, int gs, int tid,
                                             int nthreads, float* rs) {
  const NormPrologue& nm = a.norm;
  const int K = (int)a.K, chunks = K / 8;
  const int warp = tid >> 5, lane = tid & 31, nw = nthreads >> 5;
  // Sum of squares per token. Up to 4 tokens: the whole CTA works on every
  // token (each thread a share of the row's 8-element chunks, the loads of
  // all tokens in flight at once), then per warp by shuffles and over the
  // warps in order - one warp per token would walk the row alone, a chain of
  // dependent L2 round trips. More tokens: one warp per token, the warps
  // working on different tokens at once.
  constexpr int kTokAll = 4;
  if (a.M <= kTokAll) {
    __shared__ float red[kTokAll][32];  // [token][warp]
    float ss[kTokAll] = {0.f, 0.f, 0.f, 0.f};
    for (int c = tid; c < chunks; c += nthreads) {
#pragma unroll
      for (int t = 0; t < kTokAll; ++t) {
        if (t < a.M) {
          float v[8];
          residual8(nm, (int64_t)t * K + c * 8, v);
#pragma unroll
          for (int j = 0; j < 8; ++j) ss[t] = fmaf(v[j], v[j], ss[t]);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < kTokAll; ++t) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss[t] += __shfl_xor_sync(0xffffffffu, ss[t], o);
      if (lane == 0) red[t][warp] = ss[t];
    }
    __syncthreads();
    if (tid < a.M) {
      float tot = 0.f;
      for (int w = 0; w < nw; ++w) tot += red[tid][w];
      rs[tid] = rsqrtf(tot / (float)K + nm.eps);
    }
  } else {
    for (int tok = warp; tok < a.M; tok += nw) {
      float ss = 0.f;
      for (int c = lane; c < chunks; c += 32) {
        float v[8];
        residual8(nm, (int64_t)tok * K + c * 8, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) rs[tok] = rsqrtf(ss / (float)K + nm.eps);
    }
  }
  __syncthreads();
  const int per_tok = gs * 8;  // 8-element chunks of the slice per token
  const uint32_t base = smem_addr(xs);
  const bool write_h = blockIdx.x == 0;
  const __nv_bfloat16* w = static_cast<const __nv_bfloat16*>(nm.weight);
  for (int i = tid; i < a.M * per_tok; i += nthreads) {
    const int tok = i / per_tok, c = i - tok * per_tok;
    const int64_t k0 = (int64_t)g0 * kGroup + c * 8;
    float v[8];
    residual8(nm, (int64_t)tok * K + k0, v);
    const uint4 ww = __ldg(reinterpret_cast<const uint4*>(w + k0));
    const uint32_t wv[4] = {ww.x, ww.y, ww.z, ww.w};
    const float r = rs[tok];
    uint32_t xo[4], ho[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float n0 = __bfloat162float(__float2bfloat16_rn(v[2 * q] * r));
      const float n1 = __bfloat162float(__float2bfloat16_rn(v[2 * q + 1] * r));
      xo[q] = pack_bf16x2(n0 * __uint_as_float(wv[q] << 16), n1 * __uint_as_float(wv[q] & 0xFFFF0000u));
      ho[q] = pack_bf16x2(v[2 * q], v[2 * q + 1]);  // exact: v holds bf16 values
    }
    if (write_h)
      *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(nm.h_out) + (int64_t)tok * K + k0) =
          make_uint4(ho[0], ho[1], ho[2], ho[3]);
    sts128(base + tok * xstride + c * 16, make_uint4(prmt_lo(xo[0], xo[2]), prmt_hi(xo[0], xo[2]),
                                                     prmt_lo(xo[1], xo[3]), prmt_hi(xo[1], xo[3])));
  }
}

__host__ __device__ constexpr int alloc_boxes(int bps, int copy_log2) {
  return ((bps + (1 << copy_log2) - 1) >> copy_log2) << copy_log2;
}

#ifndef QI4_GEMV_COPY_MAX
#define QI4_GEMV_COPY_MAX 8
#endif
inline int copy_log2_for(int bps) {
  if (bps > QI4_GEMV_COPY_MAX) return 2;
  int l = 0;
  while ((1 << l) < bps) ++l;
  return l;
}

__host__ __device__ constexpr int x_stride_bytes(int bps, bool f32) { return bps * kGroupsPerBox * 128 * (f32 ? 2 : 1) + 16; }

// Scale / zero-point table of the CTA's slab, built before the dependency
// wait: entry (r, g) = {scale as float, packed (magic + 8 + z) pair}. Scales
// and zero points of four consecutive groups of a row are one 8-byte and one
// 2-byte load when the row length in groups is a multiple of four.
template <int XT>
__device__ __forceinline__ void build_table(const Args& a, const Mat& mt0, const Mat* mt1, TableEntry* table,
                                            int tstride, int64_t row0, int g0, int gs, int tid, int nthreads) {
  const int R = a.rows;
  const int nch = (gs + 3) >> 2;
  const bool vec = (a.G & 3) == 0;
  for (int e = tid; e < R * nch; e += nthreads) {
    const int r = e & (R - 1), g = (e >> a.rows_log2) << 2;
    // mt1 (gate/up SwiGLU): rows 16..31 of the tile are the second matrix's rows row0..row0+15.
    const Mat& mt = (mt1 && r >= 16) ? *mt1 : mt0;
    const int64_t row = row0 + (mt1 ? (r & 15) : r);
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t znib = 0;  // the four groups' stored zero nibbles (two's complement; 0 when absent)
    if (row < mt.N) {
      const int64_t gi = row * a.G + g0 + g;
      if (vec && g + 4 <= gs) {
        const uint2 sv = __ldg(reinterpret_cast<const uint2*>(mt.scales + gi));
        const float2 s01 = __half22float2(*reinterpret_cast<const __half2*>(&sv.x));
        const float2 s23 = __half22float2(*reinterpret_cast<const __half2*>(&sv.y));
        s[0] = s01.x; s[1] = s01.y; s[2] = s23.x; s[3] = s23.y;
        if (mt.zeros) znib = __ldg(reinterpret_cast<const unsigned short*>(mt.zeros + (gi >> 1)));
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (g + j < gs) {
            s[j] = __half2float(__ldg(mt.scales + gi + j));
            if (mt.zeros) znib |= (uint32_t)((__ldg(mt.zeros + ((gi + j) >> 1)) >> (((gi + j) & 1) * 4)) & 0xF) << (4 * j);
          }
        }
      }
    }
    TableEntry* t = table + r * tstride + g;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (g + j < gs)
        t[j] = TableEntry{s[j], Fmt<XT>::kMagic + (((znib >> (4 * j)) & 0xF) ^ 0x8u) * 0x00010001u};
  }
}

// v rounded to the activation dtype (identity for FP32).
template <int XT>
__device__ __forceinline__ float round_act(float v) {
  if constexpr (XT == QI4_DTYPE_BF16)
    return __bfloat162float(__float2bfloat16_rn(v));
  else if constexpr (XT == QI4_DTYPE_F16)
    return __half2float(__float2half_rn(v));
  else
    return v;
}

// The output has the activations' dtype (FP32 for FP32 activations).
template <int XT>
__device__ __forceinline__ void store_out(void* out, int64_t i, float v) {
  if constexpr (XT == QI4_DTYPE_F32)
    static_cast<float*>(out)[i] = v;
  else if constexpr (XT == QI4_DTYPE_BF16)
    static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
  else
    static_cast<__half*>(out)[i] = __float2half_rn(v);
}

// One warp waits for the prerequisite grid (griddepcontrol.wait makes its
// memory visible to the whole grid); the other warps sleep on the CTA barrier
// instead of waiting themselves, so that a CTA resident ahead of its turn
// issues nothing while the previous kernel still computes on the same SM.
__device__ __forceinline__ void wait_prerequisites(int tid) {
  if (tid < 32) pdl_wait();
  __syncthreads();
}

// D = (c - z) . x for one group of 64 k and the lane's token tile(s), then
// acc += scale * D (rows r and r + 8 of the lane; FP32 activations as two
// MMAs of the bf16 hi and lo planes). x_row[n] is the staged row of the
// lane's token in tile n; lanes past the last token read the last token's
// row (no fill, no predicate), and their output columns are never stored.
template <int XT, int NT>
__device__ __forceinline__ void mma_group(float (&acc)[NT][4], const uint32_t* al, const uint32_t* ah, float s_lo,
                                          float s_hi, int g, const uint32_t (&x_row)[NT], int gs) {
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    uint4 xb[4];
    {
      const uint32_t xp = x_row[n] + (uint32_t)(g * 128);
      xb[0] = lds128(xp);
      xb[1] = lds128(xp + 16);
      if constexpr (XT == QI4_DTYPE_F32) {
        xb[2] = lds128(xp + gs * 128);
        xb[3] = lds128(xp + gs * 128 + 16);
      } else {
        xb[2] = xb[3] = make_uint4(0, 0, 0, 0);
      }
    }
    const uint32_t bh[8] = {xb[0].x, xb[0].y, xb[0].z, xb[0].w, xb[1].x, xb[1].y, xb[1].z, xb[1].w};
    const uint32_t bl[8] = {xb[2].x, xb[2].y, xb[2].z, xb[2].w, xb[3].x, xb[3].y, xb[3].z, xb[3].w};
    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int st = 0; st < 4; ++st) {
      const uint32_t af[4] = {al[2 * st], ah[2 * st], al[2 * st + 1], ah[2 * st + 1]};
      mma16816<XT>(d, af, bh[2 * st], bh[2 * st + 1]);
      if constexpr (XT == QI4_DTYPE_F32) mma16816<XT>(d, af, bl[2 * st], bl[2 * st + 1]);
    }
    acc[n][0] = fmaf(s_lo, d[0], acc[n][0]);
    acc[n][1] = fmaf(s_lo, d[1], acc[n][1]);
    acc[n][2] = fmaf(s_hi, d[2], acc[n][2]);
    acc[n][3] = fmaf(s_hi, d[3], acc[n][3]);
  }
}

// CTAs that must fit on one SM: 16-warp CTAs two (64 registers); the 8-warp,
// one-token-tile kernel of 16- and 32-bit activations four, so that a 560-CTA
// grid (gate/up at M = 1) is resident in one wave.
template <int XT, int NT, int WARPS, int PRE>
constexpr int kMinBlocks = WARPS == 16 ? 2 : (WARPS == 8 && NT == 1 && PRE == 0 && XT != QI4_DTYPE_F32) ? 4 : 1;

template <int XT, int NT, int WARPS, int PRE, bool SW = false, bool NORM = false>
__global__ void __launch_bounds__(WARPS * 32, kMinBlocks<XT, NT, WARPS, PRE>) gemv_mma_kernel(const __grid_constant__ CUtensorMap wmap0, const __grid_constant__ CUtensorMap wmap1,
                const __grid_constant__ CUtensorMap wmap2, const Args a) {
  // PRE > 0: every warp has at most PRE groups, expanded into registers
  // before the dependency wait (single-wave grids, whose CTAs start early).
  // SW: fused gate/up + SwiGLU. A CTA owns the same 16 output rows of both
  // matrices (its 32-row tile: 16 gate rows, then 16 up rows) and writes
  // silu(g) * u in FP32.
  constexpr int kThr = WARPS * 32;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms.
  // Offset from the shared array itself (not an integer round trip), so that
  // every pointer derived from it stays in the shared address space.
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  // NORM: x is formed from the residual stream while staging (a compile-time
  // variant, so that the plain kernels keep their register budget).
  __shared__ float norm_rs[NORM ? 16 : 1];  // per-token RMSNorm factors (M <= 16)
  constexpr int kWarpsLog2 = WARPS == 32 ? 5 : WARPS == 16 ? 4 : WARPS == 8 ? 3 : WARPS == 4 ? 2 : WARPS == 2 ? 1 : 0;
  static_assert((1 << kWarpsLog2) == WARPS, "warps per CTA must be a power of two");
  const int R = a.rows;
  const int rb_log2 = a.rows_log2 - 4;   // R is a power of two, 16 <= R <= 16 WARPS
  const int RB = R >> 4;                 // 16-row blocks
  const int kp_log2 = kWarpsLog2 - rb_log2;
  const int KP = 1 << kp_log2;           // warps that share one 16-row block
  const int nbox_total = (a.G + kGroupsPerBox - 1) / kGroupsPerBox;
  const int box0 = blockIdx.y * a.boxes_per_split;
  const int nbox = max(0, min(a.boxes_per_split, nbox_total - box0));  // 0 only for a CTA past the end
  const int g0 = box0 * kGroupsPerBox;
  const int gs = max(0, min(a.G - g0, nbox * kGroupsPerBox));  // groups of this CTA
  // The CTA's matrix and its row tile within that matrix.
  const int tile = blockIdx.x;
  const int m = (a.nmats > 1 && tile >= a.tiles_end[0]) + (a.nmats > 2 && tile >= a.tiles_end[1]);
  const Mat& mt = m == 0 ? a.mat[0] : (m == 1 ? a.mat[1] : a.mat[2]);
  const CUtensorMap* wmap = m == 0 ? &wmap0 : (m == 1 ? &wmap1 : &wmap2);
  const int64_t row0 = SW ? (int64_t)tile * 16 : (int64_t)(tile - (m == 0 ? 0 : a.tiles_end[m - 1])) * R;

  const int tstride = a.boxes_per_split * kGroupsPerBox + 1;  // odd stride: conflict-free table reads
  const int copies = (nbox + (1 << a.copy_log2) - 1) >> a.copy_log2;
  uint8_t* wsm = smem;  // boxes x R x 128, box-major (rounded up to whole copies)
  TableEntry* table = reinterpret_cast<TableEntry*>(wsm + (size_t)alloc_boxes(a.boxes_per_split, a.copy_log2) * R * kBoxBytes);
  float* red = reinterpret_cast<float*>(table + (size_t)R * tstride);
  uint8_t* xs = reinterpret_cast<uint8_t*>(red + (size_t)(KP - 1) * RB * 32 * NT * 4 + (size_t)R * NT * 8);
  const int xstride = x_stride_bytes(a.boxes_per_split, XT == QI4_DTYPE_F32);
  uint64_t* bars = reinterpret_cast<uint64_t*>(xs + (size_t)a.M * xstride);

  // Everything that depends only on the weights happens before
  // griddepcontrol.wait, overlapping the previous kernels of a chain.
  pdl_launch_dependents();
  const int tid = threadIdx.x;
  if (SW && tid == 0 && nbox > 0) {
    // One barrier per box, completed by a 16-row copy from each matrix.
    for (int b = 0; b < nbox; ++b) mbar_init(bars + b, 1);
    fence_barrier_init();
    for (int b = 0; b < nbox; ++b) {
      mbar_arrive_expect_tx(bars + b, (uint32_t)(R * kBoxBytes));
      tma_load_2d(wsm + (size_t)b * R * kBoxBytes, &wmap0, (box0 + b) * kBoxBytes, (int)row0, bars + b);
      tma_load_2d(wsm + (size_t)b * R * kBoxBytes + 16 * kBoxBytes, &wmap1, (box0 + b) * kBoxBytes, (int)row0,
                  bars + b);
    }
  } else if (tid == 0 && nbox > 0) {
    // One 3-D copy brings (1 << copy_log2) boxes of the R rows, box-major;
    // boxes past the end of a row arrive zero-filled (and are never read).
    for (int c = 0; c < copies; ++c) mbar_init(bars + c, 1);
    fence_barrier_init();
    const int cb = 1 << a.copy_log2;
    for (int c = 0; c < copies; ++c) {
      mbar_arrive_expect_tx(bars + c, (uint32_t)(cb * R * kBoxBytes));
      if (a.three_d)
        tma_load_3d(wsm + (size_t)c * cb * R * kBoxBytes, wmap, 0, (int)row0, box0 + c * cb, bars + c);
      else  // cb == 1
        tma_load_2d(wsm + (size_t)c * R * kBoxBytes, wmap, (box0 + c) * kBoxBytes, (int)row0, bars + c);
    }
  }
  build_table<XT>(a, mt, SW ? &a.mat[1] : nullptr, table, tstride, row0, g0, gs, tid, kThr);
  // The bias of the row this thread stores (row tid % R: the thread count is
  // a multiple of R), read before the dependency wait.
  float bias_r = 0.f;
  if (!SW && mt.bias != nullptr && gridDim.y == 1) {
    const int64_t brow = row0 + (tid & (R - 1));
    if (brow < mt.N) bias_r = load_as_f32(mt.bias, a.bias_dtype, brow);
  }
  __syncthreads();  // barriers initialised, table complete

  const int warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;  // MMA groupID / thread-in-group
  const int rb = warp & (RB - 1), kp = warp >> rb_log2;
  const int gb = (gs * kp) >> kp_log2, ge = (gs * (kp + 1)) >> kp_log2;  // this warp's groups

  const int r_lo = rb * 16 + gq;
  // Rows r and r + 8 share r % 8 (the swizzle phase): the lane's 8 bytes of
  // group g sit in 16-byte chunk (2 (g % 4) + tq / 2) XOR (r % 8), half tq % 2.
  const uint32_t a_row = smem_addr(wsm) + r_lo * kBoxBytes + ((tq & 1) << 3);
  uint32_t x_row[NT];
#pragma unroll
  for (int n = 0; n < NT; ++n) x_row[n] = smem_addr(xs) + min(n * 8 + gq, a.M - 1) * xstride + tq * 32;
  const TableEntry* t_lo = table + r_lo * tstride;
  const TableEntry* t_hi = t_lo + 8 * tstride;

  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[n][q] = 0.f;

  if constexpr (PRE > 0) {
    uint32_t fa[PRE][16];
    float fs[PRE][2];
#pragma unroll
    for (int j = 0; j < PRE; ++j) {
      const int g = gb + j;
      if (g < ge) {
        mbar_wait(bars + ((g >> 2) >> a.copy_log2), 0, &g_gemv_mma_error);
        const uint32_t ap = a_row + (uint32_t)((g >> 2) * R * kBoxBytes) +
                            (uint32_t)(((((g & 3) << 1) | (tq >> 1)) ^ (gq & 7)) << 4);
        const uint2 wl = lds64(ap);
        const uint2 wh = lds64(ap + 8 * kBoxBytes);
        const TableEntry el = t_lo[g], eh = t_hi[g];
        expand_word<XT>(wl.x, el.zc2, fa[j]);
        expand_word<XT>(wl.y, el.zc2, fa[j] + 4);
        expand_word<XT>(wh.x, eh.zc2, fa[j] + 8);
        expand_word<XT>(wh.y, eh.zc2, fa[j] + 12);
        fs[j][0] = el.scale;
        fs[j][1] = eh.scale;
      }
    }
    wait_prerequisites(tid);  // activations come from the previous kernel
    if constexpr (NORM)
      stage_x_norm(a, xs, xstride, g0, gs, tid, kThr, norm_rs);
    else
      stage_x<XT, PRE == 0>(a, xs, xstride, g0, gs, tid, kThr);
    __syncthreads();
#pragma unroll
    for (int j = 0; j < PRE; ++j)
      if (gb + j < ge) mma_group<XT, NT>(acc, fa[j], fa[j] + 8, fs[j][0], fs[j][1], gb + j, x_row, gs);
  } else {
    wait_prerequisites(tid);  // activations come from the previous kernel
    if constexpr (NORM)
      stage_x_norm(a, xs, xstride, g0, gs, tid, kThr, norm_rs);
    else
      stage_x<XT, PRE == 0>(a, xs, xstride, g0, gs, tid, kThr);
    __syncthreads();

    if (KP % 4 == 0 && gs <= 4 * KP) {
      // At most four groups per warp, interleaved over the KP warps of a row
      // block (warp kp takes g = kp, kp + KP, ...): when the last box lands, each warp has at most
      // one of its groups left, instead of one warp owning the whole box. All
      // of a warp's groups sit at position kp % 4 of their box, so its
      // swizzled chunk offset is fixed.
      const uint32_t coff = (uint32_t)(((((kp & 3) << 1) | (tq >> 1)) ^ (gq & 7)) << 4);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int g = kp + (j << kp_log2);
        if (g >= gs) break;
        mbar_wait(bars + ((g >> 2) >> a.copy_log2), 0, &g_gemv_mma_error);
        const uint32_t ap = a_row + (uint32_t)((g >> 2) * R * kBoxBytes) + coff;
        const uint2 wl = lds64(ap);
        const uint2 wh = lds64(ap + 8 * kBoxBytes);
        const TableEntry el = t_lo[g], eh = t_hi[g];
        uint32_t al[8], ah[8];
        expand_word<XT>(wl.x, el.zc2, al);
        expand_word<XT>(wl.y, el.zc2, al + 4);
        expand_word<XT>(wh.x, eh.zc2, ah);
        expand_word<XT>(wh.y, eh.zc2, ah + 4);
        mma_group<XT, NT>(acc, al, ah, el.scale, eh.scale, g, x_row, gs);
      }
    } else {
      uint32_t coff[4];  // 16-byte chunk of group j of a box for this lane (swizzled)
#pragma unroll
      for (int j = 0; j < 4; ++j) coff[j] = (uint32_t)((((j << 1) | (tq >> 1)) ^ (gq & 7)) << 4);
      for (int b = gb >> 2; b < (ge + 3) >> 2; ++b) {
        // Each box has its own barrier: the first groups are used while later
        // boxes are still in flight.
        mbar_wait(bars + (b >> a.copy_log2), 0, &g_gemv_mma_error);
        const uint32_t box = a_row + (uint32_t)(b * R * kBoxBytes);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int g = 4 * b + j;
          if (g < gb || g >= ge) continue;
          const uint2 wl = lds64(box + coff[j]);
          const uint2 wh = lds64(box + coff[j] + 8 * kBoxBytes);
          const TableEntry el = t_lo[g], eh = t_hi[g];
          uint32_t al[8], ah[8];
          expand_word<XT>(wl.x, el.zc2, al);
          expand_word<XT>(wl.y, el.zc2, al + 4);
          expand_word<XT>(wh.x, eh.zc2, ah);
          expand_word<XT>(wh.y, eh.zc2, ah + 4);
          mma_group<XT, NT>(acc, al, ah, el.scale, eh.scale, g, x_row, gs);
        }
      }
    }
    }

  // Every warp leaves its partial sums in shared memory ([kp][row][token]);
  // then one thread per (row, token) adds the KP partials (independent loads,
  // one round of latency) and stores the output, or, when K is split across a
  // cluster, keeps the CTA's sum for the cluster reduction below.
  float* part = red;  // [KP][R][NT * 8]
  const int ld = NT * 8;
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int q = 0; q < 4; ++q)
      part[((size_t)kp * R + r_lo + (q < 2 ? 0 : 8)) * ld + n * 8 + 2 * tq + (q & 1)] = acc[n][q];
  __syncthreads();
  if constexpr (SW) {
    // g and u are rounded to the activation dtype (the projections' output
    // dtype), then silu(g) * u in FP32, as the reference MLP computes it.
    float* out = static_cast<float*>(mt.out);
    for (int i = tid; i < 16 * a.M; i += kThr) {
      const int tok = i >> 4, r = i & 15;
      const int64_t row = row0 + r;
      float g = 0.f, u = 0.f;
#pragma unroll
      for (int q = 0; q < WARPS; ++q)
        if (q < KP) {
          g += part[((size_t)q * R + r) * ld + tok];
          u += part[((size_t)q * R + 16 + r) * ld + tok];
        }
      if (row < mt.N) {
        g = round_act<XT>(g);
        u = round_act<XT>(u);
        out[(int64_t)tok * mt.N + row] = g / (1.0f + expf(-g)) * u;
      }
    }
    return;
  }
  const bool split = gridDim.y > 1;
  for (int i = tid; i < R * a.M; i += kThr) {
    const int tok = i >> a.rows_log2, r = i - (tok << a.rows_log2);
    float sum = 0.f;
#pragma unroll
    for (int q = 0; q < WARPS; ++q)  // KP <= WARPS
      if (q < KP) sum += part[((size_t)q * R + r) * ld + tok];
    if (split) {
      part[(size_t)r * ld + tok] = sum;
    } else {
      const int64_t row = row0 + r;
      if (row < mt.N) store_out<XT>(mt.out, (int64_t)tok * mt.N + row, sum + bias_r);
    }
  }
  if (!split) return;

  // Split K: the cluster's CTAs reduce over distributed shared memory, each
  // CTA finishing an equal share of the slab's outputs.
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  {
    const int nranks = (int)cluster.num_blocks();
    const int me = (int)cluster.block_rank();
    const int total = R * NT * 8;
    const int per = (total + nranks - 1) / nranks;
    const int lo = me * per, hi = min(total, lo + per);
    for (int i = lo + tid; i < hi; i += kThr) {
      const int r = i / (NT * 8), tok = i - r * (NT * 8);
      const int64_t row = row0 + r;
      if (tok >= a.M || row >= mt.N) continue;
      float sum = 0.f;
      for (int q = 0; q < nranks; ++q) sum += cluster.map_shared_rank(part, q)[i];
      const float b = mt.bias ? load_as_f32(mt.bias, a.bias_dtype, row) : 0.f;
      store_out<XT>(mt.out, (int64_t)tok * mt.N + row, sum + b);
    }
  }
  cluster.sync();
}

size_t smem_bytes(int R, int warps, int bps, int NT, int M, bool f32, int copy_log2) {
  const int RB = R / 16;
  const int KP = warps / RB > 0 ? warps / RB : 1;
  const size_t table = (size_t)R * (bps * kGroupsPerBox + 1) * sizeof(TableEntry);
  const size_t red = ((size_t)(KP - 1) * RB * 32 * NT * 4 + (size_t)R * NT * 8) * sizeof(float);
  const size_t xs = (size_t)M * x_stride_bytes(bps, f32);
  return 1024 + (size_t)alloc_boxes(bps, copy_log2) * R * kBoxBytes + table + red + xs + (size_t)bps * 8;
}

template <int XT, int NT, int WARPS, int PRE, bool SW = false, bool NORM = false>
cudaError_t launch_t(const CUtensorMap* maps, const Args& a, int ksplit, cudaStream_t stream, bool pdl) {
  auto kernel = gemv_mma_kernel<XT, NT, WARPS, PRE, SW, NORM>;
  static unsigned long long configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    configured |= bit;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.tiles_end[a.nmats - 1], (unsigned)ksplit, 1);
  cfg.blockDim = dim3(WARPS * 32, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes(a.rows, WARPS, a.boxes_per_split, NT, a.M, XT == QI4_DTYPE_F32, a.copy_log2);
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int n = 0;
  if (ksplit > 1) {  // a K split reduces over its cluster; whole-K grids launch without one
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = 1;
    attrs[n].val.clusterDim.y = (unsigned)ksplit;
    attrs[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, maps[0], maps[1], maps[2], a);
}

template <int XT, int NT>
cudaError_t launch_w(const CUtensorMap* map, const Args& a, int warps, int ksplit, int pre, cudaStream_t s,
                     bool pdl) {
  switch (warps) {
    case 2: return launch_t<XT, NT, 2, 0>(map, a, ksplit, s, pdl);
    case 4: return launch_t<XT, NT, 4, 0>(map, a, ksplit, s, pdl);
    case 8: return pre ? launch_t<XT, NT, 8, kPreGroups>(map, a, ksplit, s, pdl) : launch_t<XT, NT, 8, 0>(map, a, ksplit, s, pdl);
    case 32: return launch_t<XT, NT, 32, 0>(map, a, ksplit, s, pdl);
    default: return launch_t<XT, NT, 16, 0>(map, a, ksplit, s, pdl);
  }
}

template <int XT>
cudaError_t launch_x(const CUtensorMap* map, const Args& a, int nt, int warps, int ksplit, int pre,
                     cudaStream_t s, bool pdl) {
  if (a.has_norm) {  // the fused block boundary: bf16, decode plans of 8 or 16 warps
    // (with pre-wait expansion where the plan has it: 137 registers, one CTA
    // per SM, still measured faster in the decode step than without it)
    if constexpr (XT == QI4_DTYPE_BF16) {
      if (warps == 8)
        return nt <= 1 ? (pre ? launch_t<XT, 1, 8, kPreGroups, false, true>(map, a, ksplit, s, pdl)
                              : launch_t<XT, 1, 8, 0, false, true>(map, a, ksplit, s, pdl))
                       : (pre ? launch_t<XT, 2, 8, kPreGroups, false, true>(map, a, ksplit, s, pdl)
                              : launch_t<XT, 2, 8, 0, false, true>(map, a, ksplit, s, pdl));
      if (warps == 16)
        return nt <= 1 ? launch_t<XT, 1, 16, 0, false, true>(map, a, ksplit, s, pdl)
                       : launch_t<XT, 2, 16, 0, false, true>(map, a, ksplit, s, pdl);
    }
    return cudaErrorInvalidValue;
  }
  return nt <= 1 ? launch_w<XT, 1>(map, a, warps, ksplit, pre, s, pdl)
                 : launch_w<XT, 2>(map, a, warps, ksplit, pre, s, pdl);
}

thread_local MmaGemvPlan g_override{};

}  // namespace

void set_gemv_mma_override(int rows, int ksplit, int warps) {
  g_override = MmaGemvPlan{};
  g_override.rows = rows;
  g_override.ksplit = ksplit;
  g_override.warps = warps;
}

MmaGemvPlan plan_gemv_mma(int64_t M, int64_t N, int64_t K, int x_dtype, int num_sms) {
  const int G = (int)(K / kGroup);
  const int nboxes = (G + kGroupsPerBox - 1) / kGroupsPerBox;
  const int nt = M <= 8 ? 1 : 2;
  auto make = [&](int R, int ks, int warps) {
    MmaGemvPlan p{};
    p.rows = R;
    p.warps = warps;
    p.boxes_per_split = (nboxes + ks - 1) / ks;
    p.ksplit = (nboxes + p.boxes_per_split - 1) / p.boxes_per_split;  // every CTA gets at least one box
    p.nt = nt;
    // Boxes per TMA copy: the whole slab in one copy up to 8 boxes (fewer,
    // larger copies stream faster), else copies of 4 boxes so that the
    // first groups are used while later copies are in flight.
    // (3-D copies need rows of whole 128-byte boxes: K a multiple of 256.)
    p.three_d = K % 256 == 0;
    p.copy_log2 = p.three_d ? copy_log2_for(p.boxes_per_split) : 0;
    p.smem = smem_bytes(R, warps, p.boxes_per_split, nt, (int)M, x_dtype == QI4_DTYPE_F32, p.copy_log2);
    // A single-wave grid (one CTA per SM at most) starts ahead of the
    // previous kernel's end; with at most kPreGroups groups per warp its
    // weight fragments are expanded before the dependency wait.
    const int kp = warps / (R / 16);
    p.pre = warps == 8 && (N + R - 1) / R * p.ksplit <= num_sms &&
            (p.boxes_per_split * kGroupsPerBox + kp - 1) / kp <= kPreGroups;
    return p;
  };
  if (g_override.rows) {
    const int w = g_override.warps ? g_override.warps : 4;
    if (g_override.rows / 16 > w) return MmaGemvPlan{};
    MmaGemvPlan p = make(g_override.rows, std::min(g_override.ksplit, nboxes), w);
    return p.smem <= 200 * 1024 ? p : MmaGemvPlan{};
  }
  // Measured on B200 over Qwen2-1.5B shapes (chains of 28 PDL launches and
  // the mixed 196-launch step, M = 1..16): 8 warps per CTA (16 for long rows,
  // below); 16-row tiles, except from M = 8 on for grids of more than two
  // 16-row tiles per SM or rows of 16+ boxes, which take 32-row tiles (the
  // activation fragments then serve more rows).
  // K stays whole for M < 4 unless shared memory runs out. From M = 4 on, rows
  // of at least 16 boxes are split over a cluster until the grid has 1.5 CTAs
  // per SM, keeping each CTA within 110 KB so that two fit on an SM.
  const int R = (M >= 8 && ((N + 15) / 16 > 2 * (int64_t)num_sms || nboxes >= 16)) ? 32 : 16;
  const int64_t tiles = (N + R - 1) / R;
  // `req` is the requested split; make() may round it down to the number of
  // CTAs that get boxes, so the loops step `req`, which always terminates.
  int req = 1;
  MmaGemvPlan best = make(R, req, 8);
  // FP32 activations stage twice the bytes per token: from 13 tokens on a
  // split of at most 8 still needs more than 110 KB per CTA (one CTA per SM,
  // 2.3 waves for down_proj at M = 16: 31.6 us against 17.4 us at M = 12), so
  // their split may grow to 16 CTAs (a non-portable cluster size).
  const int max_req = x_dtype == QI4_DTYPE_F32 ? 16 : 8;
  if (M >= 4 && nboxes >= 16) {
    while (req < nboxes && ((req < 8 && (tiles * best.ksplit < (int64_t)(1.5 * num_sms) ||
                                         best.smem > 110 * 1024)) ||
                            (req < max_req && best.smem > 110 * 1024)))
      best = make(R, ++req, 8);
  }
  while (best.smem > 200 * 1024 && req < 8 && req < nboxes) best = make(R, ++req, 8);
  // A single-wave grid with K whole whose warps would each own more than 8
  // groups (long rows such as down_proj at M = 1) runs 16 warps per CTA
  // (64 registers, so two CTAs still fit an SM).
  const int kp8 = 8 / (R / 16);
  if (best.ksplit == 1 && tiles <= num_sms && (best.boxes_per_split * kGroupsPerBox + kp8 - 1) / kp8 > 8) {
    const MmaGemvPlan wide = make(R, 1, 16);
    if (wide.smem <= 200 * 1024) best = wide;
  }
  if (best.smem > 200 * 1024) best = MmaGemvPlan{};
  return best;
}

bool gemv_mma_supported(int64_t M, int64_t K) { return M >= 1 && M <= 16 && K % kGroup == 0; }

cudaError_t launch_gemv_mma_multi(const void* x, int x_dtype, int64_t M, int64_t K, int count,
                                  const uint8_t* const* qweights, const uint16_t* const* scales,
                                  const uint8_t* const* zeros, const void* const* biases, int bias_dtype,
                                  void* const* outs, const int64_t* Ns, cudaStream_t stream, bool pdl,
                                  const MmaGemvPlan& p, const NormPrologue* norm) {
  if (count < 1 || count > kMaxMats) return cudaErrorInvalidValue;
  if (norm && (x_dtype != QI4_DTYPE_BF16 || M > 16)) return cudaErrorInvalidValue;
  CUtensorMap maps[kMaxMats];
  Args a{};
  a.x = x;
  a.M = (int)M;
  a.K = K;
  a.nmats = count;
  a.bias_dtype = bias_dtype;
  a.rows = p.rows;
  a.rows_log2 = __builtin_ctz((unsigned)p.rows);
  a.boxes_per_split = p.boxes_per_split;
  a.copy_log2 = p.copy_log2;
  a.three_d = p.three_d;
  a.G = (int)(K / kGroup);
  a.has_norm = norm != nullptr;
  if (norm) a.norm = *norm;
  int64_t tiles = 0;
  for (int i = 0; i < kMaxMats; ++i) {
    const int j = i < count ? i : count - 1;  // unused slots repeat the last matrix
    if (i < count) {
      const bool ok = p.three_d ? tensor_map_row_boxes(&maps[i], qweights[i], (uint64_t)(K / 2), (uint64_t)Ns[i],
                                                       (uint32_t)p.rows, 1u << p.copy_log2)
                                : tensor_map_2d(&maps[i], qweights[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)(K / 2),
                                                (uint64_t)Ns[i], (uint64_t)(K / 2), kBoxBytes, (uint32_t)p.rows,
                                                CU_TENSOR_MAP_SWIZZLE_128B);
      if (!ok) return cudaErrorInvalidValue;
      tiles += (Ns[i] + p.rows - 1) / p.rows;
    } else {
      maps[i] = maps[j];
    }
    a.mat[i].scales = reinterpret_cast<const __half*>(scales[j]);
    a.mat[i].zeros = zeros[j];
    a.mat[i].bias = biases ? biases[j] : nullptr;
    a.mat[i].out = outs[j];
    a.mat[i].N = Ns[j];
    if (tiles > INT32_MAX / 2) return cudaErrorInvalidValue;
    a.tiles_end[i] = (int)tiles;
  }
  switch (x_dtype) {
    case QI4_DTYPE_F16: return launch_x<QI4_DTYPE_F16>(maps, a, p.nt, p.warps, p.ksplit, p.pre, stream, pdl);
    case QI4_DTYPE_BF16: return launch_x<QI4_DTYPE_BF16>(maps, a, p.nt, p.warps, p.ksplit, p.pre, stream, pdl);
    default: return launch_x<QI4_DTYPE_F32>(maps, a, p.nt, p.warps, p.ksplit, p.pre, stream, pdl);
  }
}

cudaError_t launch_gemv_mma(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qweight,
                            const uint16_t* scales, const uint8_t* zeros, const void* bias, int bias_dtype,
                            void* out, int64_t N, cudaStream_t stream, bool pdl, const MmaGemvPlan& p) {
  return launch_gemv_mma_multi(x, x_dtype, M, K, 1, &qweight, &scales, &zeros, &bias, bias_dtype, &out, &N, stream,
                               pdl, p);
}

namespace {

template <int XT>
cudaError_t launch_swiglu_x(const CUtensorMap* maps, const Args& a, int nt, cudaStream_t s, bool pdl) {
  if (a.has_norm) {
    if constexpr (XT == QI4_DTYPE_BF16)
      return nt <= 1 ? launch_t<XT, 1, 8, 0, true, true>(maps, a, 1, s, pdl)
                     : launch_t<XT, 2, 8, 0, true, true>(maps, a, 1, s, pdl);
    return cudaErrorInvalidValue;
  }
  return nt <= 1 ? launch_t<XT, 1, 8, 0, true>(maps, a, 1, s, pdl) : launch_t<XT, 2, 8, 0, true>(maps, a, 1, s, pdl);
}

// out = silu(g) * u in FP32 from the two projections' outputs (activation
// dtype), for the tensor-core route of the fused call.
template <typename T>
__global__ void __launch_bounds__(256) swiglu_kernel(const T* __restrict__ g, const T* __restrict__ u,
                                                     float* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float gv = static_cast<float>(g[i]), uv = static_cast<float>(u[i]);
    out[i] = gv / (1.0f + expf(-gv)) * uv;
  }
}

}  // namespace

MmaGemvPlan plan_gemv_swiglu(int64_t M, int64_t K, int x_dtype) {
  const int G = (int)(K / kGroup);
  MmaGemvPlan p{};
  p.rows = 32;  // 16 gate rows + 16 up rows
  p.warps = 8;
  p.ksplit = 1;
  p.boxes_per_split = (G + kGroupsPerBox - 1) / kGroupsPerBox;
  p.nt = M <= 8 ? 1 : 2;
  p.pre = 0;
  p.three_d = 0;
  p.copy_log2 = 0;
  p.smem = smem_bytes(p.rows, p.warps, p.boxes_per_split, p.nt, (int)M, x_dtype == QI4_DTYPE_F32, 0);
  if (p.smem > 200 * 1024) p.rows = 0;
  return p;
}

cudaError_t launch_gemv_swiglu(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* const* qweights,
                               const uint16_t* const* scales, const uint8_t* const* zeros, float* out, int64_t N,
                               cudaStream_t stream, bool pdl, const MmaGemvPlan& p, const NormPrologue* norm) {
  if (norm && (x_dtype != QI4_DTYPE_BF16 || M > 16)) return cudaErrorInvalidValue;
  CUtensorMap maps[kMaxMats];
  for (int i = 0; i < 2; ++i)
    if (!tensor_map_2d(&maps[i], qweights[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)(K / 2), (uint64_t)N,
                       (uint64_t)(K / 2), kBoxBytes, 16, CU_TENSOR_MAP_SWIZZLE_128B))
      return cudaErrorInvalidValue;
  maps[2] = maps[1];
  Args a{};
  a.x = x;
  a.M = (int)M;
  a.K = K;
  a.nmats = 2;
  a.bias_dtype = QI4_DTYPE_NONE;
  a.rows = p.rows;
  a.rows_log2 = __builtin_ctz((unsigned)p.rows);
  a.boxes_per_split = p.boxes_per_split;
  a.copy_log2 = 0;
  a.three_d = 0;
  a.G = (int)(K / kGroup);
  a.has_norm = norm != nullptr;
  if (norm) a.norm = *norm;
  const int tiles = (int)((N + 15) / 16);
  for (int i = 0; i < kMaxMats; ++i) {
    const int j = i < 2 ? i : 1;
    a.mat[i].scales = reinterpret_cast<const __half*>(scales[j]);
    a.mat[i].zeros = zeros[j];
    a.mat[i].bias = nullptr;
    a.mat[i].out = out;
    a.mat[i].N = N;
    a.tiles_end[i] = tiles;
  }
  switch (x_dtype) {
    case QI4_DTYPE_F16: return launch_swiglu_x<QI4_DTYPE_F16>(maps, a, p.nt, stream, pdl);
    case QI4_DTYPE_BF16: return launch_swiglu_x<QI4_DTYPE_BF16>(maps, a, p.nt, stream, pdl);
    default: return launch_swiglu_x<QI4_DTYPE_F32>(maps, a, p.nt, stream, pdl);
  }
}

cudaError_t launch_swiglu_elementwise(const void* g, const void* u, int dtype, float* out, int64_t n,
                                      cudaStream_t stream, int num_sms) {
  if (n <= 0) return cudaSuccess;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, (int64_t)num_sms * 8);
  switch (dtype) {
    case QI4_DTYPE_F16:
      swiglu_kernel<__half><<<blocks, 256, 0, stream>>>(static_cast<const __half*>(g), static_cast<const __half*>(u),
                                                         out, n);
      break;
    case QI4_DTYPE_BF16:
      swiglu_kernel<__nv_bfloat16><<<blocks, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(g),
                                                                static_cast<const __nv_bfloat16*>(u), out, n);
      break;
    default:
      swiglu_kernel<float><<<blocks, 256, 0, stream>>>(static_cast<const float*>(g), static_cast<const float*>(u),
                                                        out, n);
  }
  return cudaGetLastError();
}

namespace {

// One thread waits, with the kernels' bounded wait, on a shared-memory
// barrier that nothing ever arrives on: the wait gives up after limit_ns and
// records the time-out in the same device flag the GEMV kernels use.
__global__ void __launch_bounds__(32) bounded_wait_selftest_kernel(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    mbar_wait_for(&bar, 0, &g_gemv_mma_error, limit_ns);
  }
}

}  // namespace

cudaError_t launch_bounded_wait_selftest(uint64_t limit_ns, cudaStream_t stream) {
  bounded_wait_selftest_kernel<<<1, 32, 0, stream>>>(limit_ns);
  return cudaGetLastError();
}

int read_gemv_mma_error(cudaStream_t stream) {
  int v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, g_gemv_mma_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream) !=
      cudaSuccess)
    return -1;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return -1;
  if (v) {
    const int zero = 0;
    cudaMemcpyToSymbolAsync(g_gemv_mma_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    cudaStreamSynchronize(stream);
  }
  return v;
}

}  // namespace qi4
