// Prefill dequant-GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// out[M, N] = x[M, K] @ deq(W)^T (+ bias), W4G64 canonical packing. Replaces
// the fp32 `tl.dot` of _linear_canonical_w4g64_kernel (reference
// src/qwen_int4/triton_kernels.py:66-116) for large M; numerics follow
// torch_reference_linear (src/qwen_int4/backends.py:73-98) up to the bf16 (or
// fp16) rounding of the dequantised weight fed to the tensor core.
//
// Tile: 128 weight rows (UMMA M) x BN tokens (UMMA N <= 256) x one 64-wide
// group per pipeline stage, i.e. the product is computed as D^T = W x^T with
// the dequantised weight as the 128-row A operand (dequant work per FLOP is
// 1/BN) and the activations as the B operand; the FP32 accumulator lives in
// TMEM (128 lanes x BN columns).
//
// Warp roles (10 warps):
//   warp 0     TMA producer: packed-weight boxes [128 rows x 128 B] (4 groups)
//              and activation tiles [BN rows x 64 elements], both with 128-byte
//              swizzle, into shared-memory rings completing on mbarriers. The
//              weight boxes are issued before griddepcontrol.wait.
//   warp 1     allocates TMEM, then one lane issues 4 tcgen05.mma (K = 16 each)
//              per stage and tcgen05.commit's the stage back to the producers.
//   warps 2-9  dequantise: per stage each thread expands 32 codes of one row
//              (exact FP32 w = (c - z) * s via the 1 + (c+8)/16 trick, one
//              rounding to bf16/fp16) and stores them in the UMMA canonical
//              K-major SW128 layout (16-byte chunk j of row r at j ^ (r % 8));
//              then, after the last MMA, the same warps are the epilogue:
//              tcgen05.ld 32 lanes x 32 columns, + bias (FP32), cast, store.
// Small M (fewer tiles than SMs): the grid's z dimension splits K over a
// thread-block cluster of up to 8 CTAs, each running its share of the packed
// boxes through the same pipeline; their FP32 partial tiles are parked in
// shared memory and summed over distributed shared memory, each CTA finishing
// 128 / ksplit rows of the tile (+ bias, cast, store).
// Every mbarrier wait is bounded (tma_util.cuh); every CTA loads its own tiles.
#include <cooperative_groups.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "gemm_tc.cuh"
#include "qi4_common.cuh"
#include "tma_util.cuh"

namespace qi4 {

__device__ int g_gemm_tc_error;

namespace {

// A (dequantised, in TMEM) + B (activations, in shared memory) stages in
// flight, by the activation tile's width (x_tiles = 2 for FP32 activations,
// carried as bf16 hi + lo). Measured on B200 at M = 2048 over the seven Qwen2
// shapes with 256-token tiles: 3 stages 700 TFLOP/s aggregate, 4 stages 734,
// 5 stages 717. Narrow tiles compute little per stage, so the round trip
// dequantise -> MMA -> commit -> dequantise the next use of the slot bounds
// them; they take more slots (the TMEM columns and shared memory are there:
// 64 + 12 x 32 columns at 64 tokens).
__host__ __device__ constexpr int a_stages(int x_tiles, int bn) {
  return x_tiles * bn <= 64 ? 12 : x_tiles * bn <= 128 ? 6 : 4;
}
// Packed-weight boxes (4 groups, 16 KB each) in flight: what shared memory
// leaves beside the activation stages (and the K split's partial tile). At
// least ~45 KB per SM covers the HBM latency (Little's law: ~1 us x the SM's
// share of the bandwidth); wide tiles compute long enough per box for two.
__host__ __device__ constexpr int p_stages(int x_tiles, int bn) {
  return x_tiles * bn <= 64 ? 5 : x_tiles * bn <= 128 ? 3 : x_tiles * bn <= 192 ? 4 : 2;
}
constexpr int kTileN = 128;     // weight rows per tile (UMMA M)
constexpr int kMaxKSplit = 8;   // CTAs per cluster along K (portable cluster size)
// Dequantise/epilogue warps per CTA: 16 (one CTA per SM, tiles up to 256
// tokens) or 8 (128-token tiles, two CTAs per SM, so that one CTA's prologue
// and epilogue overlap the other's main loop). Threads: producer + MMA warps
// plus these.
__host__ __device__ constexpr int gemm_threads(int dw) { return 64 + 32 * dw; }

// Tensor-memory columns: the FP32 accumulator (BN) plus the A stages of 32
// columns (64 bf16 K elements of 128 rows), rounded up to a power of two.
__host__ __device__ constexpr uint32_t tmem_cols(int bn, int stages) {
  return bn + 32 * stages <= 128 ? 128u : (bn + 32 * stages <= 256 ? 256u : 512u);
}
constexpr int kABytes = kTileN * 128;   // one group of 128 rows in bf16: 16 KB
constexpr int kPBytes = kTileN * 128;   // one packed box: 128 rows x 128 B

constexpr int kMaxMats = 3;  // weight matrices sharing the activations in one launch (q/k/v, gate/up)

// One weight matrix of a launch.
struct Mat {
  int64_t N;
  const __half* scales;
  const uint8_t* zeros;
  const void* bias;
  void* out;
};

struct Args {
  int M;
  int64_t K;
  Mat mat[kMaxMats];
  int tiles_end[kMaxMats];  // cumulative 128-row tiles: matrix m owns tiles [tiles_end[m-1], tiles_end[m])
  int nmats;
  int bias_dtype;
  int out_dtype;
  int BN;
  int tma_out;  // 1: output tile staged in shared memory and written by one TMA store
  int dw;       // dequantise/epilogue warps per CTA (16; the kernel also compiles for 8)
  int ksplit;   // CTAs per cluster along K (grid z); > 1 reduces FP32 partial tiles over DSMEM
  int bps;      // packed 128-byte boxes (4 groups) per K split
};

// The tensor maps of a launch: packed weights and outputs per matrix, activations (and their lo half).
struct Maps {
  CUtensorMap w[kMaxMats];
  CUtensorMap x, x_lo;
  CUtensorMap o[kMaxMats];
};

// ---- tcgen05 wrappers ------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Same, with the A operand read from tensor memory (lane = row, 32-bit column =
// two consecutive K elements).
__device__ __forceinline__ void tc_mma_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns, waiting until the writes complete.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint4& a, const uint4& b, const uint4& c,
                                          const uint4& d) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w), "r"(c.x), "r"(c.y), "r"(c.z),
      "r"(c.w), "r"(d.x), "r"(d.y), "r"(d.z), "r"(d.w)
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 8 consecutive 32-bit columns from registers into tensor memory,
// waiting until the writes have completed.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint4& a, const uint4& b) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), "r"(a.x),
      "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Arrive on `bar` once every tcgen05 operation issued so far by this thread completes.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), start address in 16-byte units.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;             // leading-byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;   // stride-byte offset
  d |= (uint64_t)1 << 46;             // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;             // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: D = F32, A = B = bf16 (1) or f16 (0),
// both K-major, N = bn, M = 128.
__host__ __device__ constexpr uint32_t make_idesc(int ab_bf16, int bn) {
  return (1u << 4) | ((uint32_t)ab_bf16 << 7) | ((uint32_t)ab_bf16 << 10) | ((uint32_t)(bn >> 3) << 17) |
         ((uint32_t)(kTileN >> 4) << 24);
}

// 8 codes (one packed word) -> 8 dequantised values packed as 4 x bf16x2/f16x2.
// (a * s + c, b * s + c) with one packed FP32 FMA (sm_100a f32x2: each lane
// rounded once, as two fmaf would be).
__device__ __forceinline__ void fma2(float a, float b, float s, float c, float& ra, float& rb) {
  asm("{\n\t.reg .b64 x, m, d, r;\n\t"
      "mov.b64 x, {%2, %3};\n\t"
      "mov.b64 m, {%4, %4};\n\t"
      "mov.b64 d, {%5, %5};\n\t"
      "fma.rn.f32x2 r, x, m, d;\n\t"
      "mov.b64 {%0, %1}, r;\n\t}"
      : "=f"(ra), "=f"(rb)
      : "f"(a), "f"(b), "f"(s), "f"(c));
}

template <int XT>
__device__ __forceinline__ uint4 dequant_word(uint32_t word, float s16, float nz) {
  uint32_t lo, hi;
  expand_nibbles(word, lo, hi);
  float w0, w1, w2, w3, w4, w5, w6, w7;
  fma2(nibble_float<0>(lo), nibble_float<0>(hi), s16, nz, w0, w1);
  fma2(nibble_float<1>(lo), nibble_float<1>(hi), s16, nz, w2, w3);
  fma2(nibble_float<2>(lo), nibble_float<2>(hi), s16, nz, w4, w5);
  fma2(nibble_float<3>(lo), nibble_float<3>(hi), s16, nz, w6, w7);
  uint4 r;
  if constexpr (XT == QI4_DTYPE_F16) {
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r.x) : "f"(w1), "f"(w0));
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r.y) : "f"(w3), "f"(w2));
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r.z) : "f"(w5), "f"(w4));
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r.w) : "f"(w7), "f"(w6));
  } else {
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r.x) : "f"(w1), "f"(w0));
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r.y) : "f"(w3), "f"(w2));
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r.z) : "f"(w5), "f"(w4));
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r.w) : "f"(w7), "f"(w6));
  }
  return r;
}

template <int XT, int BN, int DW>
__global__ void __launch_bounds__(gemm_threads(DW), DW == 8 ? 2 : 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap wmap0, const __grid_constant__ CUtensorMap wmap1,
                   const __grid_constant__ CUtensorMap wmap2, const __grid_constant__ CUtensorMap xmap,
                   const __grid_constant__ CUtensorMap xmap_lo, const __grid_constant__ CUtensorMap omap0,
                   const __grid_constant__ CUtensorMap omap1, const __grid_constant__ CUtensorMap omap2,
                   const Args a) {
  extern __shared__ uint8_t smem_raw[];
  // Offset from the shared array itself (not an integer round trip), so that
  // every pointer derived from it stays in the shared address space.
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  // FP32 activations arrive as two bf16 tiles (x = hi + lo), loaded together.
  constexpr int kXTiles = XT == QI4_DTYPE_F32 ? 2 : 1;
  constexpr int kBBytes = kXTiles * BN * 128;       // BN rows x 64 elements (2 bytes), per tile
  constexpr int kStages = a_stages(kXTiles, BN);
  constexpr int kPStages = p_stages(kXTiles, BN);
  constexpr uint32_t kTmemCols = tmem_cols(BN, kStages);  // D (BN columns) + A stages (32 columns each)
  static_assert(BN + 32 * kStages <= 512, "accumulator and A stages must fit tensor memory");
  uint8_t* sB = smem;                               // kStages x BN*128
  uint8_t* sP = sB + kStages * kBBytes;             // kPStages x 16 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + kPStages * kPBytes);
  uint64_t* b_full = bars;                  // [kStages]   TMA(x) -> MMA
  uint64_t* a_full = b_full + kStages;      // [kStages]   dequant -> MMA (DW arrivals)
  uint64_t* empty = a_full + kStages;       // [kStages]   MMA commit -> producers
  uint64_t* p_full = empty + kStages;       // [kPStages]  TMA(packed) -> dequant
  uint64_t* p_empty = p_full + kPStages;    // [kPStages]  dequant -> TMA(packed) (DW arrivals)
  uint64_t* acc_full = p_empty + kPStages;  // final commit -> epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

  // [BN][128] FP32 partial tile (K split only), 16-byte aligned for the cluster's vector reads.
  uint8_t* part_raw = reinterpret_cast<uint8_t*>(tmem_slot + 4);
  float* part = reinterpret_cast<float*>(part_raw + ((16u - (smem_addr(part_raw) & 15u)) & 15u));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // This CTA's matrix and its 128-row tile within that matrix.
  const int tile = blockIdx.x;
  const int mi = (a.nmats > 1 && tile >= a.tiles_end[0]) + (a.nmats > 2 && tile >= a.tiles_end[1]);
  const Mat& mt = mi == 0 ? a.mat[0] : (mi == 1 ? a.mat[1] : a.mat[2]);
  const CUtensorMap* wmap = mi == 0 ? &wmap0 : (mi == 1 ? &wmap1 : &wmap2);
  const CUtensorMap* omap = mi == 0 ? &omap0 : (mi == 1 ? &omap1 : &omap2);
  const int64_t N = mt.N;
  const int64_t n0 = (int64_t)(tile - (mi == 0 ? 0 : a.tiles_end[mi - 1])) * kTileN;
  const int m0 = blockIdx.y * BN;
  // This CTA's K range: boxes [box0, box0 + bps) of the row (4 groups each).
  const int KT_all = (int)(a.K / kGroup);
  const int box0 = blockIdx.z * a.bps;
  const int kb = box0 * 4;                                 // first group
  const int KT = max(0, min(KT_all - kb, a.bps * 4));     // pipeline steps (one group each)

  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&a_full[i], DW);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(&p_full[i], 1);
      mbar_init(&p_empty[i], DW);
    }
    mbar_init(acc_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;        // accumulator: columns [0, BN)
  const uint32_t tmem_a = tmem_d + BN;       // A stages: columns [BN + 32 s, BN + 32 s + 32)

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      prefetch_tensor_map(wmap);
      prefetch_tensor_map(&xmap);
      if constexpr (kXTiles == 2) prefetch_tensor_map(&xmap_lo);
      const int nbox = (KT + 3) / 4;
      // Weight boxes do not depend on the previous kernel: issue the first ones now.
      int pbox = 0;
      for (; pbox < kPStages && pbox < nbox; ++pbox) {
        mbar_arrive_expect_tx(&p_full[pbox], kPBytes);
        tma_load_2d(sP + pbox * kPBytes, wmap, (box0 + pbox) * 128, (int)n0, &p_full[pbox]);
      }
      pdl_wait();
      for (int k = 0; k < KT; ++k) {
        const int s = k % kStages;
        const uint32_t ph = (uint32_t)(k / kStages) & 1u;
        mbar_wait(&empty[s], ph ^ 1u, &g_gemm_tc_error);
        mbar_arrive_expect_tx(&b_full[s], kBBytes);
        tma_load_2d(sB + s * kBBytes, &xmap, (kb + k) * kGroup, m0, &b_full[s]);
        if constexpr (kXTiles == 2)
          tma_load_2d(sB + s * kBBytes + BN * 128, &xmap_lo, (kb + k) * kGroup, m0, &b_full[s]);
        if ((k & 3) == 3 && pbox < nbox) {  // refill the packed ring
          const int p = pbox % kPStages;
          const uint32_t pph = (uint32_t)(pbox / kPStages) & 1u;
          mbar_wait(&p_empty[p], pph ^ 1u, &g_gemm_tc_error);
          mbar_arrive_expect_tx(&p_full[p], kPBytes);
          tma_load_2d(sP + p * kPBytes, wmap, (box0 + pbox) * 128, (int)n0, &p_full[p]);
          ++pbox;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = make_idesc(XT == QI4_DTYPE_F16 ? 0 : 1, BN);  // FP32 x: bf16 hi/lo
      for (int k = 0; k < KT; ++k) {
        const int s = k % kStages;
        const uint32_t ph = (uint32_t)(k / kStages) & 1u;
        mbar_wait(&a_full[s], ph, &g_gemm_tc_error);
        mbar_wait(&b_full[s], ph, &g_gemm_tc_error);
        tc_fence_after();
        const uint64_t bdesc = sw128_desc(smem_addr(sB + s * kBBytes));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)  // K = 16 per MMA: 8 TMEM columns of A, +32 bytes of B
          tc_mma_ta(tmem_d, tmem_a + 32 * s + 8 * kk, bdesc + 2 * kk, idesc, (k > 0 || kk > 0) ? 1u : 0u);
        if constexpr (kXTiles == 2) {  // + W x_lo: the low bf16 half of FP32 activations
          const uint64_t ldesc = sw128_desc(smem_addr(sB + s * kBBytes + BN * 128));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) tc_mma_ta(tmem_d, tmem_a + 32 * s + 8 * kk, ldesc + 2 * kk, idesc, 1u);
        }
        tc_commit(&empty[s]);
      }
      tc_commit(acc_full);
    }
  } else {
    // ---------------- dequantise (warps 2..) into tensor memory ----------------
    // A warp may only access the TMEM lanes of its quarter (warp % 4): warp w
    // dequantises rows 32 (w % 4) + lane and, of each group, the codes of
    // slice sub = (w - 2) / 4: 16 codes (8 packed bytes -> 8 TMEM columns) with
    // 16 such warps, 32 codes (16 bytes -> 16 columns) with 8.
    constexpr int kSpan = 16 / DW;  // 16-code slices per thread per group
    const int quarter = warp & 3;
    const int sub = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;  // tile row 0..127
    const int64_t row = n0 + r;
    const bool row_ok = row < N;
    const int64_t G = a.K / kGroup;
    const __half* srow = mt.scales + (row_ok ? row : 0) * G + kb;
    const int64_t zrow = (row_ok ? row : 0) * G + kb;
    const uint32_t sP_addr = smem_addr(sP);
    const uint32_t t_lane = (uint32_t)(quarter * 32) << 16;
    const int nbox = (KT + 3) / 4;
    // Scales / zero points of a whole box (4 groups) are prefetched one box ahead.
    float sc4[4], nsc4[4];
    int z4[4], nz4[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sc4[j] = (row_ok && j < KT) ? __half2float(__ldg(srow + j)) : 0.f;
      z4[j] = (row_ok && j < KT) ? load_zero(mt.zeros, zrow + j) : 0;
    }
    for (int pb = 0; pb < nbox; ++pb) {
      const int p = pb % kPStages;
      const uint32_t pph = (uint32_t)(pb / kPStages) & 1u;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int kn = (pb + 1) * 4 + j;
        nsc4[j] = (row_ok && kn < KT) ? __half2float(__ldg(srow + kn)) : 0.f;
        nz4[j] = (row_ok && kn < KT) ? load_zero(mt.zeros, zrow + kn) : 0;
      }
      mbar_wait(&p_full[p], pph, &g_gemm_tc_error);
      uint4 q[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if constexpr (kSpan == 1) {
          const uint2 h =
              lds64(sP_addr + p * kPBytes + r * 128 + (((j * 2 + (sub >> 1)) ^ (r & 7)) << 4) + ((sub & 1) << 3));
          q[j] = make_uint4(h.x, h.y, 0u, 0u);
        } else {  // slices 2 sub and 2 sub + 1: the whole 16-byte chunk j * 2 + sub
          q[j] = lds128(sP_addr + p * kPBytes + r * 128 + (((j * 2 + sub) ^ (r & 7)) << 4));
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_empty[p]);  // box consumed into registers
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int k = pb * 4 + j;
        if (k >= KT) break;
        const int s = k % kStages;
        const uint32_t ph = (uint32_t)(k / kStages) & 1u;
        const float s16 = 16.0f * sc4[j], nz = -static_cast<float>(24 + z4[j]) * sc4[j];
        const uint4 d0 = dequant_word<XT>(q[j].x, s16, nz);
        const uint4 d1 = dequant_word<XT>(q[j].y, s16, nz);
        if constexpr (kSpan == 1) {
          mbar_wait(&empty[s], ph ^ 1u, &g_gemm_tc_error);
          tc_fence_after();
          tmem_st8(tmem_a + t_lane + (uint32_t)(32 * s + 8 * sub), d0, d1);
        } else {
          const uint4 d2 = dequant_word<XT>(q[j].z, s16, nz);
          const uint4 d3 = dequant_word<XT>(q[j].w, s16, nz);
          mbar_wait(&empty[s], ph ^ 1u, &g_gemm_tc_error);
          tc_fence_after();
          tmem_st16(tmem_a + t_lane + (uint32_t)(32 * s + 16 * sub), d0, d1, d2, d3);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[s]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sc4[j] = nsc4[j];
        z4[j] = nz4[j];
      }
    }

    // ---------------- epilogue ----------------
    mbar_wait(acc_full, 0, &g_gemm_tc_error);
    tc_fence_after();
    constexpr int kSlices = DW / 4;  // warps per lane quarter; warp `sub` takes 32-column blocks sub, sub + kSlices, ...
    const int er = quarter * 32 + lane;                            // tile row of this thread
    const int64_t orow = n0 + er;
    const float bv = (orow < N && mt.bias) ? load_as_f32(mt.bias, a.bias_dtype, orow) : 0.f;
    // Output: each warp stages its 32 rows x 32 tokens of a column block as a
    // contiguous [32 tokens][32 rows] box in the activation ring (which the
    // finished main loop no longer uses) and stores it with its own TMA store
    // at once, so staging, stores and the next block's TMEM loads overlap and
    // no CTA-wide barrier precedes the stores.
    constexpr int kOsz = XT == QI4_DTYPE_F32 ? 4 : 2;
#pragma unroll 1
    for (int c0 = sub * 32; c0 < BN; c0 += kSlices * 32) {
      uint8_t* box = sB + (size_t)((c0 >> 5) * 4 + quarter) * (32 * 32 * kOsz);
      uint16_t* sO = reinterpret_cast<uint16_t*>(box);
      float* sO32 = reinterpret_cast<float*>(box);
      uint32_t v[32];
      tmem_ld32(tmem_d + t_lane + (uint32_t)c0, v);
      if (a.ksplit > 1) {  // partial sums stay in shared memory for the cluster reduction
#pragma unroll
        for (int j = 0; j < 32; ++j) part[(c0 + j) * kTileN + er] = KT > 0 ? __uint_as_float(v[j]) : 0.f;
      } else if (a.tma_out) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float f = __uint_as_float(v[j]) + bv;
          if constexpr (XT == QI4_DTYPE_F32)
            sO32[j * 32 + lane] = f;
          else
            sO[j * 32 + lane] = XT == QI4_DTYPE_F16 ? __half_as_ushort(__float2half_rn(f))
                                                    : __bfloat16_as_ushort(__float2bfloat16_rn(f));
        }
        fence_proxy_async_smem();  // this thread's staged values -> visible to the TMA engine
        __syncwarp();
        // (a box wholly past the last row or token is not issued; partial boxes are clipped by the TMA)
        if (lane == 0 && n0 + quarter * 32 < N && m0 + c0 < a.M)
          tma_store_2d(omap, (int)n0 + quarter * 32, m0 + c0, box);
      } else if (orow < N) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int m = m0 + c0 + j;
          if (m < a.M) store_from_f32(mt.out, a.out_dtype, (int64_t)m * N + orow, __uint_as_float(v[j]) + bv);
        }
      }
    }
    if (a.tma_out && lane == 0) tma_store_commit_and_wait();  // the staged boxes were read
  }

  if (a.ksplit > 1) {
    // K split: the cluster's CTAs sum their partial tiles over distributed
    // shared memory; CTA z finishes rows [z * per, (z + 1) * per) of the tile
    // (per a multiple of 4). A thread takes 4 consecutive rows of one token:
    // it issues the 16-byte loads from every CTA of the cluster before
    // summing them in rank order.
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();  // every partial tile is written
    if (warp >= 2) {
      const int nranks = (int)cluster.num_blocks();
      const int per = ((kTileN + nranks - 1) / nranks + 3) & ~3;
      const int rlo = (int)cluster.block_rank() * per;
      const int rows4 = max(0, min(kTileN, rlo + per) - rlo) / 4;
      const float4* peer[kMaxKSplit];
#pragma unroll
      for (int q = 0; q < kMaxKSplit; ++q)
        peer[q] = reinterpret_cast<const float4*>(cluster.map_shared_rank(part, q < nranks ? q : 0));
      for (int i = (int)threadIdx.x - 64; i < rows4 * BN; i += 32 * DW) {
        const int c = i / rows4, r = rlo + 4 * (i - c * rows4);
        float4 v[kMaxKSplit];
#pragma unroll
        for (int q = 0; q < kMaxKSplit; ++q)
          if (q < nranks) v[q] = peer[q][(c * kTileN + r) >> 2];
        float sum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < kMaxKSplit; ++q)
          if (q < nranks) {
            sum[0] += v[q].x;
            sum[1] += v[q].y;
            sum[2] += v[q].z;
            sum[3] += v[q].w;
          }
        const int m = m0 + c;
        if (m < a.M) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int64_t n = n0 + r + e;
            if (n < N) {
              const float b = mt.bias ? load_as_f32(mt.bias, a.bias_dtype, n) : 0.f;
              store_from_f32(mt.out, a.out_dtype, (int64_t)m * N + n, sum[e] + b);
            }
          }
        }
      }
    }
    cluster.sync();  // no CTA leaves while a peer still reads its partials
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_d, kTmemCols);
  }
}

size_t smem_bytes(int BN, int x_tiles, int ksplit) {
  const int ps = p_stages(x_tiles, BN), st = a_stages(x_tiles, BN);
  return 1024 + (size_t)st * x_tiles * BN * 128 + (size_t)ps * kPBytes +
         (3 * st + 2 * ps + 1) * sizeof(uint64_t) + 16 +
         (ksplit > 1 ? (size_t)BN * kTileN * sizeof(float) + 16 : 0);
}

template <int XT, int BN, int DW>
cudaError_t launch_bn(const Maps& mp, const Args& a, cudaStream_t stream, bool pdl) {
  const size_t smem = smem_bytes(BN, XT == QI4_DTYPE_F32 ? 2 : 1, a.ksplit);
  auto kernel = gemm_tc_kernel<XT, BN, DW>;
  static unsigned long long configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(configured & bit)) {
    // Room for the K split's partial tile where one is planned (tiles <= 128 wide).
    const size_t max_smem = smem_bytes(BN, XT == QI4_DTYPE_F32 ? 2 : 1, BN <= 128 ? 2 : 1);
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)max_smem);
    if (e != cudaSuccess) return e;
    configured |= bit;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.tiles_end[a.nmats - 1], (unsigned)((a.M + BN - 1) / BN), (unsigned)a.ksplit);
  cfg.blockDim = dim3(gemm_threads(DW), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int n = 0;
  if (pdl) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (a.ksplit > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = 1;
    attrs[n].val.clusterDim.y = 1;
    attrs[n].val.clusterDim.z = (unsigned)a.ksplit;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, mp.w[0], mp.w[1], mp.w[2], mp.x, mp.x_lo, mp.o[0], mp.o[1], mp.o[2], a);
}

template <int XT>
cudaError_t launch_x(const Maps& mp, const Args& a, cudaStream_t s, bool pdl) {
  switch (a.BN) {
    case 32: return launch_bn<XT, 32, 16>(mp, a, s, pdl);
    case 64: return launch_bn<XT, 64, 16>(mp, a, s, pdl);
    case 128: return launch_bn<XT, 128, 16>(mp, a, s, pdl);
    default:
      if constexpr (XT == QI4_DTYPE_F32) {
        return cudaErrorInvalidValue;  // FP32 tiles are <= 128 wide
      } else {
        if (a.BN == 192) return launch_bn<XT, 192, 16>(mp, a, s, pdl);
        return launch_bn<XT, 256, 16>(mp, a, s, pdl);
      }
  }
}

thread_local int g_override_bn = 0, g_override_ks = 0;

// Estimated time (microseconds) of a plan: waves of CTAs x per-CTA time, the
// per-CTA time being its packed boxes (4 groups of K each) x (an MMA cost per
// token present in the tile plus a per-box dequantisation cost that does not
// shrink with the tile) plus a fixed pipeline fill, and, when K is split over
// a cluster, the reduction of the FP32 partial tiles. The constants are a
// least-squares fit to sweeps on B200 of tile widths 64..256 and splits 1..8
// over the Qwen2-1.5B shapes at M = 32, 64, 128, 512 and 2048.
double plan_cost(int64_t M, int64_t N, int nbox, int bn, int ks, int num_sms) {
  const int bps = (nbox + ks - 1) / ks;
  ks = (nbox + bps - 1) / bps;
  const int64_t ctas = ((N + kTileN - 1) / kTileN) * ((M + bn - 1) / bn) * ks;
  const double waves = (double)((ctas + num_sms - 1) / num_sms);
  const double tokens = (double)std::min<int64_t>(M, bn);
  return waves * (bps * (1.619e-3 * tokens + 1.503) + 3.38 + (ks > 1 ? 0.03864 * bn + 2.45 : 0.0));
}

// Token-tile width and K split: the cheapest plan by plan_cost over widths
// 256, 128 and 64 (wider tiles need M above half their width; FP32
// activations, two tiles per stage, at most 128) and clusters of 1, 2, 4 or 8
// CTAs along K. A split needs partial tiles of at most 128 tokens and
// M <= 512 (at larger M the per-CTA work already hides the pipeline latency),
// and its grid at most 0.65 x the SM count: larger cluster grids were
// measured to run well below the estimate (clusters of one-CTA-per-SM
// kernels do not pack every SM).
void plan_tiles(Args& a, int x_dtype, int num_sms) {
  const int nbox = (int)((a.K / kGroup + 3) / 4);
  const int64_t ntiles = a.tiles_end[a.nmats - 1];
  double best = 1e30;
  a.BN = 64;
  int ks_best = 1;
  for (int bn : {256, 128, 64}) {
    if (bn > 64 && a.M <= bn / 2) continue;
    if (bn > 128 && x_dtype == QI4_DTYPE_F32) continue;
    for (int ks : {1, 2, 4, 8}) {
      const int bps = (nbox + ks - 1) / ks, kse = (nbox + bps - 1) / bps;
      if (kse > 1 && (bn > 128 || a.M > 512 ||
                      (double)(ntiles * ((a.M + bn - 1) / bn) * kse) > 0.65 * num_sms))
        continue;
      const double t = plan_cost(a.M, ntiles * kTileN, nbox, bn, ks, num_sms);
      if (t < best) {
        best = t;
        a.BN = bn;
        ks_best = kse;
      }
    }
  }
  int ks = ks_best;
  if (g_override_bn) {
    a.BN = g_override_bn;
    ks = a.BN <= 128 ? std::min(g_override_ks, nbox) : 1;
  }
  a.bps = (nbox + ks - 1) / ks;
  a.ksplit = (nbox + a.bps - 1) / a.bps;  // every CTA of the cluster gets at least one box
}

// FP32 activations -> two bf16 arrays with x = hi + lo (hi = bf16(x),
// lo = bf16(x - hi)): 16 significant bits, the rest below 2^-17 |x|.
__global__ void __launch_bounds__(256) split_f32_kernel(const float4* __restrict__ x, uint2* __restrict__ hi,
                                                        uint2* __restrict__ lo, int64_t n4) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 v = __ldg(x + i);
    uint32_t h0, h1, l0, l1;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(h0) : "f"(v.y), "f"(v.x));
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(h1) : "f"(v.w), "f"(v.z));
    const float r0 = v.x - __uint_as_float(h0 << 16), r1 = v.y - __uint_as_float(h0 & 0xFFFF0000u);
    const float r2 = v.z - __uint_as_float(h1 << 16), r3 = v.w - __uint_as_float(h1 & 0xFFFF0000u);
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(l0) : "f"(r1), "f"(r0));
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(l1) : "f"(r3), "f"(r2));
    hi[i] = make_uint2(h0, h1);
    lo[i] = make_uint2(l0, l1);
  }
}

// Fills the per-matrix part of `a` and the weight / output tensor maps; false
// if a tensor map cannot describe a buffer. The output is written by TMA
// stores when every matrix's row pitch allows it (a multiple of 16 bytes,
// 16-byte-aligned base), else by direct stores.
bool set_mats(Args& a, Maps& mp, int count, const uint8_t* const* qweights, const uint16_t* const* scales,
              const uint8_t* const* zeros, const void* const* biases, void* const* outs, const int64_t* Ns) {
  if (count < 1 || count > kMaxMats) return false;
  int64_t tiles = 0;
  bool tma_ok = true;
  const int osz = a.out_dtype == QI4_DTYPE_F32 ? 4 : 2;
  for (int i = 0; i < kMaxMats; ++i) {
    const int j = i < count ? i : count - 1;  // unused slots repeat the last matrix
    if (i < count) {
      if (!tensor_map_2d(&mp.w[i], qweights[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, (uint64_t)(a.K / 2), (uint64_t)Ns[i],
                         (uint64_t)(a.K / 2), 128, kTileN, CU_TENSOR_MAP_SWIZZLE_128B))
        return false;
      tiles += (Ns[i] + kTileN - 1) / kTileN;
      tma_ok = tma_ok && (Ns[i] * osz) % 16 == 0 && reinterpret_cast<uintptr_t>(outs[i]) % 16 == 0;
    } else {
      mp.w[i] = mp.w[j];
    }
    a.mat[i].N = Ns[j];
    a.mat[i].scales = reinterpret_cast<const __half*>(scales[j]);
    a.mat[i].zeros = zeros ? zeros[j] : nullptr;
    a.mat[i].bias = biases ? biases[j] : nullptr;
    a.mat[i].out = outs[j];
    if (tiles > (1 << 30)) return false;
    a.tiles_end[i] = (int)tiles;
  }
  a.nmats = count;
  a.tma_out = 0;
  if (tma_ok) {
    const CUtensorMapDataType ot = a.out_dtype == QI4_DTYPE_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : a.out_dtype == QI4_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                  : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    a.tma_out = 1;
    for (int i = 0; i < count && a.tma_out; ++i)
      a.tma_out = tensor_map_2d(&mp.o[i], outs[i], ot, (uint64_t)Ns[i], (uint64_t)a.M, (uint64_t)Ns[i] * osz, 32, 32,
                                CU_TENSOR_MAP_SWIZZLE_NONE);
    for (int i = count; i < kMaxMats; ++i) mp.o[i] = mp.o[count - 1];
  }
  return true;
}

}  // namespace

void set_gemm_tc_override(int bn, int ksplit) {
  g_override_bn = bn;
  g_override_ks = bn ? ksplit : 0;
}

bool tc_supported(int64_t M, int64_t N, int64_t K, int x_dtype) {
  (void)N;
  return M >= 1 && K >= kGroup && K % kGroup == 0 &&
         (x_dtype == QI4_DTYPE_BF16 || x_dtype == QI4_DTYPE_F16 || x_dtype == QI4_DTYPE_F32);
}

cudaError_t launch_gemm_tc_multi(const void* x, int x_dtype, int64_t M, int64_t K, int count,
                                 const uint8_t* const* qweights, const uint16_t* const* scales,
                                 const uint8_t* const* zeros, const void* const* biases, int bias_dtype,
                                 void* const* outs, const int64_t* Ns, cudaStream_t stream, bool pdl, int num_sms) {
  Args a{};
  Maps mp;
  memset(&mp, 0, sizeof(mp));
  a.M = (int)M;
  a.K = K;
  a.bias_dtype = bias_dtype;
  a.out_dtype = x_dtype;
  if (!set_mats(a, mp, count, qweights, scales, zeros, biases, outs, Ns)) return cudaErrorInvalidValue;
  plan_tiles(a, x_dtype, num_sms);
  if (a.ksplit > 1) a.tma_out = 0;  // split tiles are finished by direct stores after the cluster reduction
  // 16 dequantise warps, one CTA per SM: measured faster at M = 2048 than
  // 128-token tiles with 8 warps and two CTAs per SM (700 vs 595 TFLOP/s).
  a.dw = 16;
  // FP32 activations: split into bf16 hi / lo arrays in stream-ordered scratch.
  void* scratch = nullptr;
  const void* x_hi = x;
  const void* x_lo = nullptr;
  if (x_dtype == QI4_DTYPE_F32) {
    const size_t half_bytes = (size_t)M * (size_t)K * 2;
    cudaError_t e = scratch_alloc(&scratch, 2 * half_bytes, stream);
    if (e != cudaSuccess) return e;
    const int64_t n4 = M * K / 4;
    const int blocks = (int)std::min<int64_t>((n4 + 255) / 256, (int64_t)num_sms * 8);
    split_f32_kernel<<<blocks, 256, 0, stream>>>(static_cast<const float4*>(x), static_cast<uint2*>(scratch),
                                                  reinterpret_cast<uint2*>(static_cast<char*>(scratch) + half_bytes),
                                                  n4);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
      scratch_free(scratch, stream);
      return e;
    }
    x_hi = scratch;
    x_lo = static_cast<char*>(scratch) + half_bytes;
  }
  const CUtensorMapDataType xt = x_dtype == QI4_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  bool ok = tensor_map_2d(&mp.x, x_hi, xt, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, kGroup, (uint32_t)a.BN,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (ok && x_lo)
    ok = tensor_map_2d(&mp.x_lo, x_lo, xt, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, kGroup, (uint32_t)a.BN,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  cudaError_t e = cudaErrorInvalidValue;
  if (ok) {
    e = x_dtype == QI4_DTYPE_F16   ? launch_x<QI4_DTYPE_F16>(mp, a, stream, pdl)
        : x_dtype == QI4_DTYPE_F32 ? launch_x<QI4_DTYPE_F32>(mp, a, stream, pdl)
                                   : launch_x<QI4_DTYPE_BF16>(mp, a, stream, pdl);
  }
  scratch_free(scratch, stream);
  return e;
}

cudaError_t launch_gemm_tc(const void* x, int x_dtype, int64_t M, int64_t K, const uint8_t* qweight,
                           const uint16_t* scales, const uint8_t* zeros, const void* bias, int bias_dtype, void* out,
                           int64_t N, cudaStream_t stream, bool pdl, int num_sms) {
  return launch_gemm_tc_multi(x, x_dtype, M, K, 1, &qweight, &scales, &zeros, &bias, bias_dtype, &out, &N, stream,
                              pdl, num_sms);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of the FP32-activation path
// ---------------------------------------------------------------------------
// The FP32-activation path above needs scratch for the bf16 hi/lo copies of
// x and gets it from the library's scratch pool. Some callers cannot allocate device
// memory at call time: engines that plan every byte of device memory up
// front and run under a hard memory cap, hosts that reach this library over a
// plain C FFI and manage no CUDA allocator of their own, and latency-critical
// loops that must not enter the allocator. For them the scratch below is a
// fixed array in the module's global memory, reserved once on every GPU that
// loads the library and held until the process exits.
namespace {

constexpr size_t kStaticScratchBytes = 32u << 20;  // 32 MiB: hi + lo bf16 copies of x, M * K <= 8 Mi elements
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch on the current device. The name is only
// a host-side handle; the address comes from cudaGetSymbolAddress, done once
// per device with that device current (the first call on a device). The
// cached address belongs to the device context that was current then: after
// cudaDeviceReset the module is loaded again and the array may move, so a
// process that resets a device must not call the allocation-free entry point
// on it again.
cudaError_t static_scratch_address(void** out) {
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return e;
    addr[dev] = p;
  }
  *out = addr[dev];
  return cudaSuccess;
}

}  // namespace

size_t static_scratch_bytes() { return kStaticScratchBytes; }

cudaError_t launch_gemm_tc_f32_static(const float* x, int64_t M, int64_t K, const uint8_t* qweight,
                                      const uint16_t* scales, const uint8_t* zeros, const void* bias, int bias_dtype,
                                      float* out, int64_t N, cudaStream_t stream, int num_sms) {
  const size_t half_bytes = (size_t)M * (size_t)K * 2;
  if (2 * half_bytes > kStaticScratchBytes) return cudaErrorInvalidValue;  // callers check first
  void* scratch = nullptr;
  cudaError_t e = static_scratch_address(&scratch);
  if (e != cudaSuccess) return e;
  Args a{};
  Maps mp;
  memset(&mp, 0, sizeof(mp));
  a.M = (int)M;
  a.K = K;
  a.bias_dtype = bias_dtype;
  a.out_dtype = QI4_DTYPE_F32;
  void* outp = out;
  if (!set_mats(a, mp, 1, &qweight, &scales, &zeros, &bias, &outp, &N)) return cudaErrorInvalidValue;
  plan_tiles(a, QI4_DTYPE_F32, num_sms);
  if (a.ksplit > 1) a.tma_out = 0;
  a.dw = 16;
  // Every element of the hi / lo arrays that the GEMM reads is written by the
  // split pass of the same call, so nothing left from an earlier call is used.
  const int64_t n4 = M * K / 4;
  const int blocks = (int)std::min<int64_t>((n4 + 255) / 256, (int64_t)num_sms * 8);
  uint2* hi = static_cast<uint2*>(scratch);
  uint2* lo = reinterpret_cast<uint2*>(static_cast<char*>(scratch) + half_bytes);
  split_f32_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<const float4*>(x), hi, lo, n4);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (!tensor_map_2d(&mp.x, hi, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2, kGroup,
                     (uint32_t)a.BN, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !tensor_map_2d(&mp.x_lo, lo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)K, (uint64_t)M, (uint64_t)K * 2,
                     kGroup, (uint32_t)a.BN, CU_TENSOR_MAP_SWIZZLE_128B))
    return cudaErrorInvalidValue;
  return launch_x<QI4_DTYPE_F32>(mp, a, stream, false);
}

int read_gemm_tc_error(cudaStream_t stream) {
  int v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, g_gemm_tc_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return -1;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return -1;
  if (v) {
    const int zero = 0;
    cudaMemcpyToSymbolAsync(g_gemm_tc_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    cudaStreamSynchronize(stream);
  }
  return v;
}

}  // namespace qi4
