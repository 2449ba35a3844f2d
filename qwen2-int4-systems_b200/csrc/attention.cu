// GQA decode attention with in-place KV-cache append (sm_100a).
//
// Replaces, for decode steps (one new token per sequence), the reference
// attention's cache growth and head expansion (src/qwen_int4/model.py:80-91:
// torch.cat of the past and new key/value, repeat_interleave of the KV heads)
// and its masked scaled_dot_product_attention (model.py:107-118), with the
// RoPE of the new query and key (model.py:74-77) in front:
//
//   q', k' = RoPE(q), RoPE(k)  (bf16: q*cos and rotate_half(q)*sin each
//                               rounded to bf16, then their sum - the
//                               reference's three bf16 tensor ops)
//   cache[b, kvh, L_b] = k', v       (in place; L_b = lengths[b])
//   out[b, h] = softmax(q'_h . K[b, h / G]^T * scale + mask) V[b, h / G]
//
// over keys 0..L_b (the past and the new token), a key j counting only where
// key_mask[b, j] is non-zero (left padding). FP32 scores (exact bf16
// products), softmax and accumulation, the P.V products from 16-bit
// softmax weights; output bf16.
//
// Work split ("flash decoding"): a CTA owns one (batch, KV head, 64-key
// split) and all G query heads of that KV head, so K and V are read once for
// the group (no expansion). The split's keys and values are copied into
// shared memory (asynchronous 16-byte copies, all in flight while the queries
// are rotated), rows padded so that the reads below are conflict-free.
// Four warps take 16 keys each on the tensor cores (mma.sync m16n8k16, bf16
// operands, FP32 accumulators): scores Q K^T with the G query heads as the
// rows of a zero-padded 16-row operand, an online softmax on the score
// registers, and P.V with the FP32 weights split into two bf16 parts (high
// and remainder: the products keep 16 bits of each weight). The CTA's
// partial (max, sum, 128 sums per head) goes to scratch and a second kernel
// combines the splits per head; for small grids (at most 16 splits) the
// splits of a (sequence, KV head) form one thread-block cluster and merge
// over distributed shared memory in the same order instead. Launches are
// programmatic dependents (the next kernel's prologue overlaps this one's
// tail).
#include <cooperative_groups.h>

#include <algorithm>
#include <cmath>

#include "qi4_common.cuh"

namespace qi4 {

__device__ int g_attention_error;

namespace {

constexpr int kD = 128;          // head dim
constexpr int kMaxGroup = 8;     // query heads per KV head
constexpr int kSplitKeys = 64;   // keys per CTA
constexpr int kWarps = 4;        // per CTA: 16 keys of the split each
constexpr int kMaxClusterSplits = 16;  // splits merged inside one cluster (non-portable size above 8)
constexpr int kQbStride = kD + 8;  // bf16 per staged query row (conflict-free fragment loads)

struct AttnArgs {
  const __nv_bfloat16* q;      // [B, Hq, D]
  const __nv_bfloat16* k_new;  // [B, Hkv, D]
  const __nv_bfloat16* v_new;  // [B, Hkv, D]
  const __nv_bfloat16* cos;    // rows of D (row positions[b], or b), or null: no RoPE
  const __nv_bfloat16* sin;
  const int32_t* positions;    // [B] row of cos/sin per sequence, or null: row b
  __nv_bfloat16* k_cache;      // [B][Hkv][cap][D] at the given strides (elements)
  __nv_bfloat16* v_cache;
  int64_t cb, ch;              // batch / head strides of the caches
  const int32_t* lengths;      // [B] past length L_b (the new token goes at L_b)
  const uint8_t* key_mask;     // [B, mask_stride], or null
  int64_t mask_stride;
  float* partial;              // [B][Hkv][splits][G][kD + 2] (two-kernel path)
  __nv_bfloat16* out;          // [B, Hq, D] (cluster path: written by the kernel itself)
  int B, Hq, Hkv, G, cap, splits;
  float scale;
  int early;                   // 1: lengths, positions and the past cache rows are read before the dependency wait
};

__device__ __forceinline__ float bf(const __nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ uint32_t smem_addr_u(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ float rbf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// RoPE of element d of a head vector x (bf16 roundings as the reference's
// tensor ops: x*cos, rotate_half(x)*sin, their sum).
__device__ __forceinline__ float rope(const __nv_bfloat16* x, const __nv_bfloat16* c, const __nv_bfloat16* s, int d) {
  const float xd = bf(x[d]);
  const float rh = d < kD / 2 ? -bf(x[d + kD / 2]) : bf(x[d - kD / 2]);
  return rbf(rbf(xd * bf(c[d])) + rbf(rh * bf(s[d])));
}

constexpr int kRowBytes = kD * 2 + 16;  // a staged key / value row, padded (conflict-free 16-byte reads)

// D += A B, m16n8k16, bf16 operands, FP32 accumulators (A rows = query
// heads padded to 16, B = keys or values).
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Four 8x8 bf16 matrices from shared memory, transposed (lane l gives the
// row address of matrix l / 8, row l % 8).
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// The 8x8 b16 matrix held in fragment layout (lane = row * 4 + column pair),
// transposed.
__device__ __forceinline__ uint32_t movm_trans(uint32_t x) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(x));
  return d;
}

__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// One CTA's share: keys [split * 64, ...) of sequence b (past length L) for
// the G query heads of KV head kvh, appended key / value included; its
// partial (per head: max, sum, 128 weighted sums) goes to `out`
// ([G][kD + 2] floats, global or shared memory). Called with keys present
// and room in the cache.
__device__ __forceinline__ void attend_split(const AttnArgs& a, const int split, const int kvh, const int b,
                                             const int L, float* __restrict__ out) {
  const int nkeys = L + 1;
  const int k0 = split * kSplitKeys;
  const int k1 = min(nkeys, k0 + kSplitKeys);
  const int G = a.G;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  __shared__ __align__(16) uint8_t kv_s[2][kSplitKeys][kRowBytes];  // past keys / values of the split
  __shared__ __align__(16) __nv_bfloat16 qb[kMaxGroup][kQbStride];  // RoPE'd queries (rows G.. zero)
  __shared__ float red_m[kWarps][kMaxGroup], red_l[kWarps][kMaxGroup], red_f[kWarps][kMaxGroup];
  // After the key loop the staged rows are dead: the warps' partial sums
  // reuse them (rows padded by 4 floats: a warp's stores to its heads' rows
  // fall in different banks).
  constexpr int kAccStride = kD + 4;
  static_assert(sizeof(float) * kWarps * kMaxGroup * kAccStride <= sizeof(uint8_t) * 2 * kSplitKeys * kRowBytes, "");
  auto red_acc = reinterpret_cast<float (*)[kMaxGroup][kAccStride]>(&kv_s[0][0][0]);

  // 1. The split's past keys and values: all copies in flight at once.
  const __nv_bfloat16* kbase = a.k_cache + b * a.cb + kvh * a.ch;
  const __nv_bfloat16* vbase = a.v_cache + b * a.cb + kvh * a.ch;
  const int npast = min(k1, L) - k0;  // keys k0 .. min(k1, L) - 1 come from the cache
  for (int i = tid; i < npast * 16; i += blockDim.x) {
    const int r = i >> 4, c = i & 15;
    cp_async16(smem_addr_u(&kv_s[0][r][c * 16]), kbase + (int64_t)(k0 + r) * kD + c * 8);
    cp_async16(smem_addr_u(&kv_s[1][r][c * 16]), vbase + (int64_t)(k0 + r) * kD + c * 8);
  }
  // The RoPE row (a constant table, at positions[b]) travels with them.
  const bool rope_on = a.cos != nullptr;
  __shared__ __align__(16) __nv_bfloat16 cs_s[kD], sn_s[kD];    // cos / sin row
  __shared__ __align__(16) __nv_bfloat16 qraw_s[kMaxGroup][kD];  // the G query heads, as given
  __shared__ __align__(16) __nv_bfloat16 kn_s[kD], vn_s[kD];     // the new key / value
  if (rope_on && tid < 32) {
    const int64_t row = a.positions ? a.positions[b] : b;
    cp_async16(smem_addr_u((tid < 16 ? cs_s : sn_s) + (tid & 15) * 8),
               (tid < 16 ? a.cos : a.sin) + row * kD + (tid & 15) * 8);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  if (a.early) pdl_wait();  // the past rows stream in while the projections finish

  // 2. The projections' outputs (one more round of copies): the G query heads
  // and, in the split that holds key L, the new key and value.
  const bool has_new = k0 <= L && L < k1;
  for (int i = tid; i < G * 16; i += blockDim.x) {
    const int h = i >> 4, c = i & 15;
    cp_async16(smem_addr_u(&qraw_s[h][c * 8]), a.q + ((int64_t)b * a.Hq + kvh * G + h) * kD + c * 8);
  }
  if (has_new && tid < 32)
    cp_async16(smem_addr_u((tid < 16 ? kn_s : vn_s) + (tid & 15) * 8),
               (tid < 16 ? a.k_new : a.v_new) + ((int64_t)b * a.Hkv + kvh) * kD + (tid & 15) * 8);
  asm volatile("cp.async.commit_group;" ::: "memory");
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  // RoPE of the queries, and of the new key (staged as row L - k0 and
  // appended to the cache), from shared memory.
  for (int i = tid; i < G * kD; i += blockDim.x) {
    const int h = i / kD, d = i - h * kD;
    const float v = rope_on ? rope(qraw_s[h], cs_s, sn_s, d) : bf(qraw_s[h][d]);  // a bf16 value either way
    qb[h][d] = __float2bfloat16_rn(v);
  }
  {
    // Rows G..7 of the query operand are zero; value rows past the split's
    // last key, up to the warp's 16-key boundary, are zero (their weights are
    // zero, and 0 x a stale NaN pattern would not be).
    for (int i = tid; i < (kMaxGroup - G) * kD; i += blockDim.x) qb[G + i / kD][i % kD] = __float2bfloat16_rn(0.f);
    const int nv = k1 - k0, nz = ((nv + 15) & ~15) - nv;
    for (int i = tid; i < nz * 16; i += blockDim.x)
      *reinterpret_cast<uint4*>(&kv_s[1][nv + (i >> 4)][(i & 15) * 16]) = make_uint4(0u, 0u, 0u, 0u);
  }
  if (has_new) {
    __nv_bfloat16* kc = a.k_cache + b * a.cb + kvh * a.ch + (int64_t)L * kD;
    __nv_bfloat16* vc = a.v_cache + b * a.cb + kvh * a.ch + (int64_t)L * kD;
    __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(&kv_s[0][L - k0][0]);
    __nv_bfloat16* vs = reinterpret_cast<__nv_bfloat16*>(&kv_s[1][L - k0][0]);
    for (int d = tid; d < kD; d += blockDim.x) {
      const __nv_bfloat16 kv = rope_on ? __float2bfloat16_rn(rope(kn_s, cs_s, sn_s, d)) : kn_s[d];
      ks[d] = kv;
      vs[d] = vn_s[d];
      kc[d] = kv;
      vc[d] = vn_s[d];
    }
  }
  __syncthreads();

  // 3. Tensor cores: a warp takes 16 keys at a time (m16n8k16, bf16
  // operands, FP32 accumulators), with the keys / dims as the 16 rows and the
  // query heads as the 8 columns (heads G..7 zero). Scores S^T = K Q^T: lane
  // (gq = lane / 4, tq = lane % 4) holds keys gq and gq + 8 for heads 2tq,
  // 2tq + 1. Online softmax per head over the 16 keys (shuffles across gq).
  // O^T = V^T P^T: V^T fragments are transposed loads of the staged rows; the
  // weights, split into bf16 high and remainder parts (16 bits of each
  // weight reach the products), move into operand layout with in-register
  // 8x8 transposes.
  const int gq = lane >> 2, tq = lane & 3;
  uint32_t qf[kD / 16][2];  // Q^T operand per 16-dim step
#pragma unroll
  for (int ks = 0; ks < kD / 16; ++ks) {
    qf[ks][0] = *reinterpret_cast<const uint32_t*>(&qb[gq][ks * 16 + 2 * tq]);
    qf[ks][1] = *reinterpret_cast<const uint32_t*>(&qb[gq][ks * 16 + 2 * tq + 8]);
  }
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f}, o[kD / 16][4];
#pragma unroll
  for (int mt = 0; mt < kD / 16; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  const uint8_t* mrow = a.key_mask ? a.key_mask + (int64_t)b * a.mask_stride : nullptr;
  // ldmatrix lane addresses: matrix j = lane / 8 covers rows + (j % 2) * 8, columns + (j / 2) * 8.
  const int lrow = (lane & 7) + (((lane >> 3) & 1) << 3), lcol = (lane >> 4) << 4;  // column in bytes
  const uint32_t ks_base = smem_addr_u(&kv_s[0][0][0]) + lrow * kRowBytes + lcol;
  const uint32_t vs_base = smem_addr_u(&kv_s[1][0][0]) + lrow * kRowBytes + lcol;
  for (int g0 = k0 + warp * 16; g0 < k1; g0 += kWarps * 16) {
    const int r0 = g0 - k0;
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < kD / 16; ++ks) {
      uint32_t a0, a1, a2, a3;  // K rows r0.. (keys), dims 16 ks..: matrices (keys +0, +8) x (dims +0, +8)
      ldsm_x4(ks_base + r0 * kRowBytes + ks * 32, a0, a1, a2, a3);
      mma_bf16(sc, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
    }
    float mx[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {  // key g0 + gq + 8 r
      const int key = g0 + gq + 8 * r;
      const bool valid = key < k1 && (!mrow || mrow[key] != 0);
#pragma unroll
      for (int e = 0; e < 2; ++e) sc[2 * r + e] = valid ? sc[2 * r + e] * a.scale : -INFINITY;
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {  // head 2tq + e
      float t = fmaxf(sc[e], sc[2 + e]);
      t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, 4));
      t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, 8));
      mx[e] = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, 16));
    }
    float alpha[2], p[4];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float mn = fmaxf(m[e], mx[e]);
      alpha[e] = mn == -INFINITY ? 1.f : __expf(m[e] - mn);
      m[e] = mn;
      p[e] = sc[e] == -INFINITY ? 0.f : __expf(sc[e] - mn);
      p[2 + e] = sc[2 + e] == -INFINITY ? 0.f : __expf(sc[2 + e] - mn);
      l[e] = l[e] * alpha[e] + (p[e] + p[2 + e]);  // this lane's two keys; summed over gq at the end
    }
#pragma unroll
    for (int mt = 0; mt < kD / 16; ++mt) {
      o[mt][0] *= alpha[0];
      o[mt][1] *= alpha[1];
      o[mt][2] *= alpha[0];
      o[mt][3] *= alpha[1];
    }
    // P^T operand: rows = keys 2tq.., column = head gq; high and remainder parts.
    const uint32_t h0 = bf16x2(p[0], p[1]), h1 = bf16x2(p[2], p[3]);
    const uint32_t r0w = bf16x2(p[0] - __uint_as_float(h0 << 16), p[1] - __uint_as_float(h0 & 0xFFFF0000u));
    const uint32_t r1w = bf16x2(p[2] - __uint_as_float(h1 << 16), p[3] - __uint_as_float(h1 & 0xFFFF0000u));
    const uint32_t bh0 = movm_trans(h0), bh1 = movm_trans(h1), bl0 = movm_trans(r0w), bl1 = movm_trans(r1w);
#pragma unroll
    for (int mt = 0; mt < kD / 16; ++mt) {
      uint32_t a0, a1, a2, a3;  // V^T: transposed loads of rows (keys +0, +8) x (dims +0, +8)
      ldsm_x4_trans(vs_base + r0 * kRowBytes + mt * 32, a0, a2, a1, a3);
      mma_bf16(o[mt], a0, a1, a2, a3, bh0, bh1);
      mma_bf16(o[mt], a0, a1, a2, a3, bl0, bl1);
    }
  }
  __syncthreads();  // every warp is done with the staged rows
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    l[e] += __shfl_xor_sync(0xffffffffu, l[e], 4);
    l[e] += __shfl_xor_sync(0xffffffffu, l[e], 8);
    l[e] += __shfl_xor_sync(0xffffffffu, l[e], 16);
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int h = 2 * tq + e;
    if (h < G) {
      if (gq == 0) {
        red_m[warp][h] = m[e];
        red_l[warp][h] = l[e];
      }
#pragma unroll
      for (int mt = 0; mt < kD / 16; ++mt) {
        red_acc[warp][h][mt * 16 + gq] = o[mt][e];
        red_acc[warp][h][mt * 16 + gq + 8] = o[mt][2 + e];
      }
    }
  }
  __syncthreads();
  // Combine the warps into the CTA's partial (warps without keys have m = -inf):
  // per head the running max, each warp's weight e^(m_w - max) and the sum.
  if (tid < G) {
    const int h = tid;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, red_m[w][h]);
    float ls = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = red_m[w][h] == -INFINITY ? 0.f : __expf(red_m[w][h] - mm);
      red_f[w][h] = f;
      ls += red_l[w][h] * f;
    }
    out[h * (kD + 2)] = mm;
    out[h * (kD + 2) + 1] = ls;
  }
  __syncthreads();
  for (int i = tid; i < G * kD; i += blockDim.x) {
    const int h = i / kD, d = i - h * kD;
    float as = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) as += red_acc[w][h][d] * red_f[w][h];
    out[h * (kD + 2) + 2 + d] = as;
  }
}

// kCluster = false: one CTA per (split, KV head, sequence) writes its partial
// to the workspace; gqa_combine_kernel merges the splits. kCluster = true
// (grids whose splits fit one thread-block cluster): the splits of a
// (sequence, KV head) are one cluster, the partials stay in shared memory,
// and after a cluster barrier CTA r merges heads r, r + C, ... over
// distributed shared memory - the combine kernel's arithmetic in the same
// order, so the output is bit-identical - and writes the bf16 output. CTAs
// without keys still take both cluster barriers.
template <bool kCluster>
__global__ void __launch_bounds__(kWarps * 32, 5) gqa_decode_kernel(const AttnArgs a) {
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  // Programmatic dependent launch: the next kernel may start its prologue;
  // this one waits for its predecessor (the q/k/v projections) before it
  // reads q / k_new / v_new - and, unless the caller vouched that lengths and
  // the past cache rows are not written by the launches just before this one
  // (`early`), before anything at all.
  pdl_launch_dependents();
  if (!a.early) pdl_wait();
  const int L = a.lengths[b];  // past keys; the new one is key L
  const bool active = split * kSplitKeys < L + 1 && L < a.cap;  // keys of this sequence here, and room
  if constexpr (!kCluster) {
    if (!active) return;
    attend_split(a, split, kvh, b, L,
                 a.partial + (((int64_t)b * a.Hkv + kvh) * a.splits + split) * a.G * (kD + 2));
  } else {
    __shared__ __align__(16) float part_s[kMaxGroup][kD + 2];
    if (active) attend_split(a, split, kvh, b, L, &part_s[0][0]);
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();  // every partial of this (sequence, KV head) is written
    // The output may be read by a launch before the predecessor until that
    // one is done: write it only after the dependency wait.
    pdl_wait();
    const int G = a.G, C = (int)cluster.num_blocks(), r = (int)cluster.block_rank();
    const int d = threadIdx.x;  // blockDim = kD: one output dimension per thread
    const int used = L < a.cap ? min(C, (L + 1 + kSplitKeys - 1) / kSplitKeys) : 0;
    for (int hg = r; hg < G; hg += C) {
      __nv_bfloat16* o = a.out + ((int64_t)b * a.Hq + kvh * G + hg) * kD;
      if (L >= a.cap) {
        o[d] = __float2bfloat16_rn(0.f);
        if (d == 0 && kvh == 0 && hg == 0) atomicOr(&g_attention_error, 2);
        continue;
      }
      float M = -INFINITY;
      for (int sp = 0; sp < used; ++sp) M = fmaxf(M, cluster.map_shared_rank(&part_s[hg][0], sp)[0]);
      float num = 0.f, den = 0.f;
      for (int sp = 0; sp < used; ++sp) {
        const float* p = cluster.map_shared_rank(&part_s[hg][0], sp);
        const float m = p[0];
        const float f = m == -INFINITY ? 0.f : __expf(m - M);
        num += p[2 + d] * f;
        den += p[1] * f;
      }
      o[d] = __float2bfloat16_rn(den > 0.f ? num / den : 0.f);
    }
    cluster.sync();  // no CTA leaves while a peer still reads its partial
  }
}

// A sequence whose cache is full (L_b >= cap) was not processed: its output
// is zero (and qi4_device_status reports QI4_DEVICE_CACHE_FULL).
__global__ void __launch_bounds__(kD) gqa_combine_kernel(const float* __restrict__ partial,
                                                          const int32_t* __restrict__ lengths,
                                                          __nv_bfloat16* __restrict__ out, int Hkv, int G, int splits,
                                                          int cap) {
  const int h = blockIdx.x, b = blockIdx.y;  // query head
  pdl_launch_dependents();
  pdl_wait();
  const int kvh = h / G, hg = h - kvh * G;
  const int L = lengths[b];
  const int tid = threadIdx.x;  // output dim (blockDim = kD)
  if (L >= cap) {
    out[((int64_t)b * Hkv * G + h) * kD + tid] = __float2bfloat16_rn(0.f);
    if (tid == 0 && h == 0) atomicOr(&g_attention_error, 2);
    return;
  }
  const int used = min(splits, (L + 1 + kSplitKeys - 1) / kSplitKeys);
  const int64_t stride = (int64_t)G * (kD + 2);  // between splits
  const float* base = partial + ((int64_t)b * Hkv + kvh) * splits * stride + hg * (kD + 2);
  // The largest running max over the splits (threads stride over splits; max is order-free).
  __shared__ float red[kD / 32];
  float mx = -INFINITY;
  for (int sp = tid; sp < used; sp += kD) mx = fmaxf(mx, base[sp * stride]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  float M = red[0];
#pragma unroll
  for (int w = 1; w < kD / 32; ++w) M = fmaxf(M, red[w]);
  // Per split (one thread each, a chunk of kD splits at a time): its weight
  // e^(m - M) and sum l, in shared memory; then each thread sums its dim over
  // the splits in split order (the loads of a chunk are independent).
  __shared__ float f_s[kD], l_s[kD];
  float num = 0.f, den = 0.f;
  for (int c0 = 0; c0 < used; c0 += kD) {
    const int n = min(kD, used - c0);
    __syncthreads();  // the previous chunk's weights are consumed
    if (tid < n) {
      const float* p = base + (c0 + tid) * stride;
      const float m = p[0];
      f_s[tid] = m == -INFINITY ? 0.f : __expf(m - M);
      l_s[tid] = p[1];
    }
    __syncthreads();
    const float* pd = base + c0 * stride + 2 + tid;
#pragma unroll 8
    for (int sp = 0; sp < n; ++sp) {
      const float f = f_s[sp];
      num += pd[sp * stride] * f;
      den += l_s[sp] * f;
    }
  }
  out[((int64_t)b * Hkv * G + h) * kD + tid] = __float2bfloat16_rn(den > 0.f ? num / den : 0.f);
}

}  // namespace

int attention_splits(int cap) { return (cap + kSplitKeys - 1) / kSplitKeys; }

cudaError_t launch_gqa_decode(const void* q, const void* k_new, const void* v_new, const void* cos, const void* sin,
                              const int32_t* positions, void* k_cache, void* v_cache, int64_t cb, int64_t ch,
                              const int32_t* lengths, const uint8_t* key_mask, int64_t mask_stride, void* out,
                              float* partial, int B, int Hq, int Hkv, int cap, float scale, int early,
                              cudaStream_t stream) {
  AttnArgs a;
  a.early = early;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k_new = static_cast<const __nv_bfloat16*>(k_new);
  a.v_new = static_cast<const __nv_bfloat16*>(v_new);
  a.cos = static_cast<const __nv_bfloat16*>(cos);
  a.sin = static_cast<const __nv_bfloat16*>(sin);
  a.positions = positions;
  a.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  a.cb = cb;
  a.ch = ch;
  a.lengths = lengths;
  a.key_mask = key_mask;
  a.mask_stride = mask_stride;
  a.partial = partial;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.B = B;
  a.Hq = Hq;
  a.Hkv = Hkv;
  a.G = Hq / Hkv;
  a.cap = cap;
  a.splits = attention_splits(cap);
  a.scale = scale;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.splits, Hkv, B);
  cfg.blockDim = dim3(kWarps * 32, 1, 1);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // Small grids (their time is one CTA's serial path): the splits of a
  // (sequence, KV head) as one cluster, merged in the kernel - no combine
  // launch. Up to 16 splits (1024 keys of capacity).
  if (a.splits <= kMaxClusterSplits && (int64_t)a.splits * Hkv * B <= 2 * (int64_t)sms) {
    static unsigned long long configured = 0;
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(configured & bit)) {
      cudaError_t e = cudaFuncSetAttribute(gqa_decode_kernel<true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return e;
      configured |= bit;
    }
    cudaLaunchAttribute cattr[2];
    cattr[0] = attr[0];
    cattr[1].id = cudaLaunchAttributeClusterDimension;
    cattr[1].val.clusterDim.x = (unsigned)a.splits;
    cattr[1].val.clusterDim.y = 1;
    cattr[1].val.clusterDim.z = 1;
    cfg.attrs = cattr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, gqa_decode_kernel<true>, a);
  }
  cudaError_t e = cudaLaunchKernelEx(&cfg, gqa_decode_kernel<false>, a);
  if (e != cudaSuccess) return e;
  cfg.gridDim = dim3(Hq, B, 1);
  cfg.blockDim = dim3(kD, 1, 1);
  return cudaLaunchKernelEx(&cfg, gqa_combine_kernel, static_cast<const float*>(partial), lengths,
                            static_cast<__nv_bfloat16*>(out), Hkv, a.G, a.splits, cap);
}

int read_attention_error(cudaStream_t stream) {
  int v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, g_attention_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return -1;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return -1;
  if (v) {
    const int zero = 0;
    cudaMemcpyToSymbolAsync(g_attention_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    cudaStreamSynchronize(stream);
  }
  return v;
}

}  // namespace qi4

namespace qi4 {
namespace {

size_t attention_workspace_bytes(int64_t B, int64_t Hq, int64_t Hkv, int64_t cap) {
  const int splits = attention_splits((int)std::min<int64_t>(cap, 1 << 24));
  return (size_t)B * Hkv * splits * (Hq / Hkv) * (kD + 2) * sizeof(float);
}

int attention_impl(const void* q, const void* k_new, const void* v_new, const void* cos, const void* sin,
                   const int32_t* positions, void* k_cache, void* v_cache, int64_t cache_batch_stride,
                   int64_t cache_head_stride, int64_t cache_capacity, const int32_t* lengths, const uint8_t* key_mask,
                   int64_t mask_stride, void* out, int64_t B, int64_t Hq, int64_t Hkv, int64_t head_dim, float scale,
                   int flags, void* workspace, size_t workspace_bytes, void* stream_ptr) {
  clear_error();
  if (!q || !k_new || !v_new || !k_cache || !v_cache || !lengths || !out || (!cos != !sin)) {
    set_error("q, k_new, v_new, the caches, lengths and out must be non-null (cos and sin both or neither)");
    return QI4_ERR_ARGUMENT;
  }
  if (B <= 0 || Hkv <= 0 || Hq <= 0 || cache_capacity <= 0 || B > 65535 || Hkv > 65535) {
    set_error("B, Hq, Hkv and the cache capacity must be positive");
    return QI4_ERR_ARGUMENT;
  }
  if (head_dim != kD || Hq % Hkv || Hq / Hkv > kMaxGroup) {
    set_error("decode attention supports head_dim 128 and up to %d query heads per KV head (got %lld, %lld/%lld)",
              kMaxGroup, (long long)head_dim, (long long)Hq, (long long)Hkv);
    return QI4_ERR_SHAPE;
  }
  if (flags & ~QI4_ATTN_EARLY_CACHE_READ) {
    set_error("unknown decode attention flags 0x%x", flags);
    return QI4_ERR_ARGUMENT;
  }
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al16(k_cache) || !al16(v_cache) || cache_batch_stride % 8 || cache_head_stride % 8 || !al16(q) ||
      !al16(k_new) || !al16(v_new) || (cos && (!al16(cos) || !al16(sin)))) {
    set_error("caches, q/k/v and cos/sin must be 16-byte aligned with strides a multiple of 8 elements");
    return QI4_ERR_ALIGNMENT;
  }
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const size_t bytes = attention_workspace_bytes(B, Hq, Hkv, cache_capacity);
  void* partial = workspace;
  if (workspace) {
    if (workspace_bytes < bytes || !al16(workspace)) {
      set_error("decode attention workspace needs %zu bytes, 16-byte aligned (got %zu)", bytes, workspace_bytes);
      return QI4_ERR_ARGUMENT;
    }
  } else if (scratch_alloc(&partial, bytes, stream) != cudaSuccess) {
    cudaGetLastError();
    set_error("cannot allocate %zu bytes of attention scratch", bytes);
    return QI4_ERR_LAUNCH;
  }
  const cudaError_t e = launch_gqa_decode(q, k_new, v_new, cos, sin, positions, k_cache, v_cache, cache_batch_stride,
                                          cache_head_stride, lengths, key_mask, mask_stride, out,
                                          static_cast<float*>(partial), (int)B, (int)Hq, (int)Hkv,
                                          (int)cache_capacity, scale, (flags & QI4_ATTN_EARLY_CACHE_READ) ? 1 : 0,
                                          stream);
  if (!workspace) scratch_free(partial, stream);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("decode attention launch failed: %s", cudaGetErrorString(e));
    return QI4_ERR_LAUNCH;
  }
  return QI4_OK;
}

}  // namespace
}  // namespace qi4

extern "C" QI4_API int qi4_gqa_decode_attention(const void* q, const void* k_new, const void* v_new, const void* cos,
                                                const void* sin, const int32_t* positions, void* k_cache,
                                                void* v_cache, int64_t cache_batch_stride, int64_t cache_head_stride,
                                                int64_t cache_capacity, const int32_t* lengths,
                                                const uint8_t* key_mask, int64_t mask_stride, void* out, int64_t B,
                                                int64_t Hq, int64_t Hkv, int64_t head_dim, float scale,
                                                void* stream_ptr) {
  return qi4::attention_impl(q, k_new, v_new, cos, sin, positions, k_cache, v_cache, cache_batch_stride,
                             cache_head_stride, cache_capacity, lengths, key_mask, mask_stride, out, B, Hq, Hkv,
                             head_dim, scale, 0, nullptr, 0, stream_ptr);
}

extern "C" QI4_API size_t qi4_gqa_decode_attention_workspace(int64_t B, int64_t Hq, int64_t Hkv,
                                                             int64_t cache_capacity) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || cache_capacity <= 0 || Hq % Hkv) return 0;
  return qi4::attention_workspace_bytes(B, Hq, Hkv, cache_capacity);
}

extern "C" QI4_API int qi4_gqa_decode_attention_ex(const void* q, const void* k_new, const void* v_new,
                                                   const void* cos, const void* sin, const int32_t* positions,
                                                   void* k_cache, void* v_cache, int64_t cache_batch_stride,
                                                   int64_t cache_head_stride, int64_t cache_capacity,
                                                   const int32_t* lengths, const uint8_t* key_mask,
                                                   int64_t mask_stride, void* out, int64_t B, int64_t Hq, int64_t Hkv,
                                                   int64_t head_dim, float scale, int flags, void* workspace,
                                                   size_t workspace_bytes, void* stream_ptr) {
  return qi4::attention_impl(q, k_new, v_new, cos, sin, positions, k_cache, v_cache, cache_batch_stride,
                             cache_head_stride, cache_capacity, lengths, key_mask, mask_stride, out, B, Hq, Hkv,
                             head_dim, scale, flags, workspace, workspace_bytes, stream_ptr);
}
