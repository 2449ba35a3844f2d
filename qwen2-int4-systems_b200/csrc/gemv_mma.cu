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

struct Args {
  const void* x;
  int M;
  int64_t K;
  const __half* scales;
  const uint8_t* zeros;
  const void* bias;
  int bias_dtype;
  void* out;
  int out_dtype;
  int64_t N;
  int rows;             // R
  int boxes_per_split;  // boxes along K per CTA
  int G;                // groups per row (K / 64)
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

// Activations of one token for one group, as the lane's B fragments: the 16
// elements x[16 tq .. 16 tq + 15] of the group, read straight from global
// memory (L2) and permuted into the k order of the weight fragments, which
// pair codes (i, i+4): k-step s takes elements {0,4,1,5} + 2s (s < 2) and
// {8,12,9,13} + 2(s-2). FP32 activations become a bf16 hi and lo pair.
struct XRaw {
  uint4 q[4];  // 16 elements: 2 x uint4 for 16-bit types, 4 x float4 for FP32
};

template <int XT>
__device__ __forceinline__ void load_x(const void* x, int64_t idx, XRaw& r) {
  if constexpr (XT == QI4_DTYPE_F32) {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const float*>(x) + idx);
#pragma unroll
    for (int q = 0; q < 4; ++q) r.q[q] = __ldg(p + q);
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const unsigned short*>(x) + idx);
    r.q[0] = __ldg(p);
    r.q[1] = __ldg(p + 1);
  }
}

__device__ __forceinline__ void zero_x(XRaw& r) {
#pragma unroll
  for (int q = 0; q < 4; ++q) r.q[q] = make_uint4(0, 0, 0, 0);
}

// b[2s], b[2s+1]: the two B registers of k-step s (hi part); lo likewise.
template <int XT>
__device__ __forceinline__ void x_frags(const XRaw& r, uint32_t (&hi)[8], uint32_t (&lo)[8]) {
  uint32_t w[8], l[8];
  if constexpr (XT == QI4_DTYPE_F32) {
    const float* v = reinterpret_cast<const float*>(r.q);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      w[q] = pack_bf16x2(v[2 * q], v[2 * q + 1]);
      l[q] = pack_bf16x2(v[2 * q] - __uint_as_float(w[q] << 16), v[2 * q + 1] - __uint_as_float(w[q] & 0xFFFF0000u));
    }
  } else {
    w[0] = r.q[0].x; w[1] = r.q[0].y; w[2] = r.q[0].z; w[3] = r.q[0].w;
    w[4] = r.q[1].x; w[5] = r.q[1].y; w[6] = r.q[1].z; w[7] = r.q[1].w;
  }
  hi[0] = prmt_lo(w[0], w[2]); hi[1] = prmt_hi(w[0], w[2]);
  hi[2] = prmt_lo(w[1], w[3]); hi[3] = prmt_hi(w[1], w[3]);
  hi[4] = prmt_lo(w[4], w[6]); hi[5] = prmt_hi(w[4], w[6]);
  hi[6] = prmt_lo(w[5], w[7]); hi[7] = prmt_hi(w[5], w[7]);
  if constexpr (XT == QI4_DTYPE_F32) {
    lo[0] = prmt_lo(l[0], l[2]); lo[1] = prmt_hi(l[0], l[2]);
    lo[2] = prmt_lo(l[1], l[3]); lo[3] = prmt_hi(l[1], l[3]);
    lo[4] = prmt_lo(l[4], l[6]); lo[5] = prmt_hi(l[4], l[6]);
    lo[6] = prmt_lo(l[5], l[7]); lo[7] = prmt_hi(l[5], l[7]);
  }
}

template <int XT, int NT>
__global__ void __launch_bounds__(kThreads, 1) gemv_mma_kernel(const __grid_constant__ CUtensorMap wmap, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int R = a.rows;
  const int RB = R >> 4;  // 16-row blocks
  const int nbox_total = (a.G + kGroupsPerBox - 1) / kGroupsPerBox;
  const int box0 = blockIdx.y * a.boxes_per_split;
  const int nbox = min(a.boxes_per_split, nbox_total - box0);
  const int g0 = box0 * kGroupsPerBox;
  const int gs = min(a.G - g0, nbox * kGroupsPerBox);  // groups of this CTA
  const int64_t row0 = (int64_t)blockIdx.x * R;

  const int tstride = a.boxes_per_split * kGroupsPerBox + 1;  // odd stride: conflict-free table reads
  const int KP = (kThreads / 32) / RB;                         // warps that share one 16-row block
  uint8_t* wsm = smem;                                         // nbox x R x 128
  TableEntry* table = reinterpret_cast<TableEntry*>(wsm + (size_t)a.boxes_per_split * R * kBoxBytes);
  float* red = reinterpret_cast<float*>(table + (size_t)R * tstride);
  uint64_t* bar = reinterpret_cast<uint64_t*>(red + (size_t)(KP - 1) * RB * 32 * NT * 4 + (size_t)R * NT * 8);

  // Everything that depends only on the weights happens before
  // griddepcontrol.wait, overlapping the previous kernel of a chain.
  pdl_launch_dependents();
  const int tid = threadIdx.x;
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0 && nbox > 0) {
    prefetch_tensor_map(&wmap);
    mbar_arrive_expect_tx(bar, (uint32_t)(nbox * R * kBoxBytes));
    for (int b = 0; b < nbox; ++b)
      tma_load_2d(wsm + (size_t)b * R * kBoxBytes, &wmap, (box0 + b) * kBoxBytes, (int)row0, bar);
  }
  const int entries = R * gs;
  for (int e = tid; e < entries; e += kThreads) {
    const int r = e / gs, g = e - r * gs;
    const int64_t row = row0 + r;
    float sv = 0.f;
    int z = 0;
    if (row < a.N) {
      const int64_t gi = row * a.G + g0 + g;
      sv = __half2float(__ldg(a.scales + gi));
      z = load_zero(a.zeros, gi);
    }
    table[r * tstride + g] = TableEntry{sv, zero_code<XT>(z)};
  }
  __syncthreads();

  const int warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;  // MMA groupID / thread-in-group
  const int rb = warp % RB, kp = warp / RB;
  const int gb = (gs * kp) / KP, ge = (gs * (kp + 1)) / KP;  // this warp's groups
  if (nbox > 0 && ge > gb) mbar_wait(bar, 0, &g_gemv_mma_error);

  pdl_wait();  // activations come from the previous kernel

  const int r_lo = rb * 16 + gq;
  // Rows r and r + 8 share r % 8 (the swizzle phase): the lane's 8 bytes of
  // group g sit in 16-byte chunk (2 (g % 4) + tq / 2) XOR (r % 8), half tq % 2.
  const uint32_t a_row = smem_addr(wsm) + r_lo * kBoxBytes + ((tq & 1) << 3);
  const TableEntry* t_lo = table + r_lo * tstride;
  const TableEntry* t_hi = t_lo + 8 * tstride;

  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[n][q] = 0.f;

  constexpr int kBatch = 4;  // groups whose activations are in flight together
  for (int gbat = gb; gbat < ge; gbat += kBatch) {
    XRaw xr[kBatch][NT];
#pragma unroll
    for (int j = 0; j < kBatch; ++j)
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int tok = n * 8 + gq;
        if (gbat + j < ge && tok < a.M)
          load_x<XT>(a.x, (int64_t)tok * a.K + (int64_t)(g0 + gbat + j) * kGroup + 16 * tq, xr[j][n]);
        else
          zero_x(xr[j][n]);
      }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int g = gbat + j;
      if (g >= ge) break;
      const int chunk = ((((g & 3) << 1) | (tq >> 1)) ^ (gq & 7)) << 4;
      const uint32_t ap = a_row + (uint32_t)((g >> 2) * R * kBoxBytes + chunk);
      const uint2 wl = lds64(ap);
      const uint2 wh = lds64(ap + 8 * kBoxBytes);
      const TableEntry el = t_lo[g], eh = t_hi[g];
      uint32_t al[8], ah[8];
      expand_word<XT>(wl.x, el.zc2, al);
      expand_word<XT>(wl.y, el.zc2, al + 4);
      expand_word<XT>(wh.x, eh.zc2, ah);
      expand_word<XT>(wh.y, eh.zc2, ah + 4);
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        uint32_t bh[8], bl[8];
        x_frags<XT>(xr[j][n], bh, bl);
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int st = 0; st < 4; ++st) {
          const uint32_t af[4] = {al[2 * st], ah[2 * st], al[2 * st + 1], ah[2 * st + 1]};
          mma16816<XT>(d, af, bh[2 * st], bh[2 * st + 1]);
          if constexpr (XT == QI4_DTYPE_F32) mma16816<XT>(d, af, bl[2 * st], bl[2 * st + 1]);
        }
        acc[n][0] = fmaf(el.scale, d[0], acc[n][0]);
        acc[n][1] = fmaf(el.scale, d[1], acc[n][1]);
        acc[n][2] = fmaf(eh.scale, d[2], acc[n][2]);
        acc[n][3] = fmaf(eh.scale, d[3], acc[n][3]);
      }
    }
  }

  // Reduce the KP warps of each row block through shared memory.
  if (KP > 1) {
    if (kp > 0) {
      float* dst = red + (((size_t)(kp - 1) * RB + rb) * 32 + lane) * NT * 4;
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int q = 0; q < 4; ++q) dst[n * 4 + q] = acc[n][q];
    }
    __syncthreads();
    if (kp == 0) {
      for (int q2 = 1; q2 < KP; ++q2) {
        const float* src = red + (((size_t)(q2 - 1) * RB + rb) * 32 + lane) * NT * 4;
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[n][q] += src[n * 4 + q];
      }
    }
  }

  const bool split = gridDim.y > 1;
  float* part = red + (size_t)(KP - 1) * RB * 32 * NT * 4;  // [R][NT*8] CTA partials for the cluster
  if (kp == 0) {
#pragma unroll
    for (int n = 0; n < NT; ++n) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int r = r_lo + (q < 2 ? 0 : 8);
        const int tok = n * 8 + 2 * tq + (q & 1);
        if (split) {
          part[r * NT * 8 + tok] = acc[n][q];
        } else {
          const int64_t row = row0 + r;
          if (tok < a.M && row < a.N) {
            const float bv = a.bias ? load_as_f32(a.bias, a.bias_dtype, row) : 0.f;
            store_from_f32(a.out, a.out_dtype, (int64_t)tok * a.N + row, acc[n][q] + bv);
          }
        }
      }
    }
  }
  if (!split) return;

  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  if (cluster.block_rank() == 0) {
    const int nranks = (int)cluster.num_blocks();
    for (int i = tid; i < R * NT * 8; i += kThreads) {
      const int r = i / (NT * 8), tok = i - r * (NT * 8);
      const int64_t row = row0 + r;
      if (tok >= a.M || row >= a.N) continue;
      float sum = 0.f;
      for (int q = 0; q < nranks; ++q) sum += cluster.map_shared_rank(part, q)[i];
      const float b = a.bias ? load_as_f32(a.bias, a.bias_dtype, row) : 0.f;
      store_from_f32(a.out, a.out_dtype, (int64_t)tok * a.N + row, sum + b);
    }
  }
  cluster.sync();
}

size_t smem_bytes(int R, int bps, int NT, int M, int x_dtype) {
  const int RB = R / 16;
  const int KP = (kThreads / 32) / RB > 0 ? (kThreads / 32) / RB : 1;
  const size_t table = (size_t)R * (bps * kGroupsPerBox + 1) * sizeof(TableEntry);
  (void)M;
  (void)x_dtype;
  const size_t red = ((size_t)(KP - 1) * RB * 32 * NT * 4 + (size_t)R * NT * 8) * sizeof(float);
  return 1024 + (size_t)bps * R * kBoxBytes + table + red + 16;
}

template <int XT, int NT>
cudaError_t launch_t(const CUtensorMap& map, const Args& a, int ksplit, cudaStream_t stream, bool pdl) {
  auto kernel = gemv_mma_kernel<XT, NT>;
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
  cfg.gridDim = dim3((unsigned)((a.N + a.rows - 1) / a.rows), (unsigned)ksplit, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes(a.rows, a.boxes_per_split, NT, a.M, XT);
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
  return cudaLaunchKernelEx(&cfg, kernel, map, a);
}

template <int XT>
cudaError_t launch_x(const CUtensorMap& map, const Args& a, int nt, int ksplit, cudaStream_t s, bool pdl) {
  return nt <= 1 ? launch_t<XT, 1>(map, a, ksplit, s, pdl) : launch_t<XT, 2>(map, a, ksplit, s, pdl);
}

thread_local MmaGemvPlan g_override{};

}  // namespace

void set_gemv_mma_override(int rows, int ksplit) {
  g_override = MmaGemvPlan{};
  g_override.rows = rows;
  g_override.ksplit = ksplit;
}

MmaGemvPlan plan_gemv_mma(int64_t M, int64_t N, int64_t K, int x_dtype, int num_sms) {
  MmaGemvPlan best{};
  const int G = (int)(K / kGroup);
  const int nboxes = (G + kGroupsPerBox - 1) / kGroupsPerBox;
  const int nt = M <= 8 ? 1 : 2;
  auto make = [&](int R, int ks) {
    MmaGemvPlan p{};
    p.rows = R;
    p.ksplit = ks;
    p.boxes_per_split = (nboxes + ks - 1) / ks;
    p.nt = nt;
    p.smem = smem_bytes(R, p.boxes_per_split, nt, (int)M, x_dtype);
    return p;
  };
  if (g_override.rows) {
    MmaGemvPlan p = make(g_override.rows, g_override.ksplit);
    return p.smem <= 200 * 1024 ? p : MmaGemvPlan{};
  }
  // Measured on B200 over Qwen2-1.5B shapes (chains of PDL launches): keep at
  // least ~1.5 CTAs per SM (the largest row tile that does so wins, else 16
  // rows), keep K whole for M <= 4, and for wider token tiles on long rows
  // split K so that each CTA holds about seven 128-byte boxes.
  int R = 16;
  for (int cand : {64, 32})
    if ((N + cand - 1) / cand >= (int64_t)(1.5 * num_sms)) {
      R = cand;
      break;
    }
  int ks = 1;
  if (M > 4 && nboxes >= 16) ks = std::min(8, std::max(1, (nboxes + 6) / 7));
  while (ks > 1 && (nboxes + (nboxes + ks - 1) / ks - 1) / ((nboxes + ks - 1) / ks) != ks) --ks;
  best = make(R, ks);
  while (best.smem > 100 * 1024 && best.ksplit < 8 && best.ksplit < nboxes) best = make(R, best.ksplit + 1);
  if (best.rows == 0) {
    best = make(16, std::min(8, nboxes));
    if (best.smem > 200 * 1024) best = MmaGemvPlan{};
  }
  return best;
}

bool gemv_mma_supported(int64_t M, int64_t K) { return M >= 1 && M <= 16 && K % kGroup == 0; }

cudaError_t launch_gemv_mma(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qweight,
                            const uint16_t* scales, const uint8_t* zeros, const void* bias, int bias_dtype,
                            void* out, int64_t N, cudaStream_t stream, bool pdl, const MmaGemvPlan& p) {
  CUtensorMap map;
  if (!tensor_map_2d(&map, qweight, CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)(K / 2), (uint64_t)N,
                     (uint64_t)(K / 2), kBoxBytes, (uint32_t)p.rows, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  Args a;
  a.x = x;
  a.M = (int)M;
  a.K = K;
  a.scales = reinterpret_cast<const __half*>(scales);
  a.zeros = zeros;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.out = out;
  a.out_dtype = x_dtype;
  a.N = N;
  a.rows = p.rows;
  a.boxes_per_split = p.boxes_per_split;
  a.G = (int)(K / kGroup);
  switch (x_dtype) {
    case QI4_DTYPE_F16: return launch_x<QI4_DTYPE_F16>(map, a, p.nt, p.ksplit, stream, pdl);
    case QI4_DTYPE_BF16: return launch_x<QI4_DTYPE_BF16>(map, a, p.nt, p.ksplit, stream, pdl);
    default: return launch_x<QI4_DTYPE_F32>(map, a, p.nt, p.ksplit, stream, pdl);
  }
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
