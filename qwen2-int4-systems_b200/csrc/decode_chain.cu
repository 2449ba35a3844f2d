// Persistent decode chain (M <= 8 tokens): a sequence of W4G64 linear stages,
// each consuming the output of an earlier stage, run by ONE cooperative
// launch with one CTA per SM. sm_100a.
//
// Why a chain: at decode sizes one linear moves 0.2-7 MB of weights, 0.03-1.1
// us of HBM time at the measured copy bandwidth, while a dependent kernel
// launch costs 2-4 us of structure (CTA turnover behind the previous grid,
// dependency release). A decoder layer is four dependent steps (q/k/v, o,
// gate/up, down), so per-launch kernels leave HBM idle most of the time. Here
// the weights of every stage are streamed by one producer warp per SM into a
// shared-memory ring, running ahead across stage boundaries (weights do not
// depend on activations); only the math of a stage waits for its input.
//
// Weights are read from a load-time prepacked copy ("tile-major W4G64",
// qi4_chain_create): a tile is 16 output rows x one 64-wide K group, 512
// bytes of codes in exactly the order of a warp's m16n8k16 A fragments (lane
// l holds 16 bytes: four 32-bit words, one per 16-wide k step, whose nibbles
// i and i+4 are the (k, k+1) pair of fragment register i), followed by the
// tile's 16 fp16 scales in lane-pair order and, for asymmetric weights, its 16
// zero-point nibbles (544 or 560 bytes a tile). A stage's tiles are one
// contiguous range in (unit, matrix-in-unit, group) order - a unit is one
// 16-row block, or a gate and an up block for the fused SwiGLU stage - so a
// CTA's share is a contiguous byte range fetched by untiled bulk copies, one
// per ring slot: no tensor maps, no swizzle, no bank conflicts.
//
// Each CTA owns whole units (CTA c: units [c U / P, (c+1) U / P)), so every
// output element is summed inside one CTA, in a fixed order: no cross-CTA
// partial sums, deterministic results. Its 15 consumer warps take contiguous
// equal shares of its tiles; a warp expands each tile's codes into exact
// biased integers B + c in bf16/f16 pairs (one LOP3 per register for mask,
// XOR and magic exponent), runs the tile's MMAs in two independent chains (two
// tiles at a time where a row block allows), removes (B + z) times the group's
// activation sum and adds scale * D to FP32 accumulators,
// parking them in shared memory at each row-block boundary; the CTA then sums
// the warps' parts per row block and stores the outputs (+ bias, cast).
//
// Dependencies are carried by the data: an output that a later stage reads is
// also stored in a mailbox word that pairs the value with a per-launch tag
// (16-bit values with a 16-bit tag in 32 bits, FP32 values with a 32-bit tag
// in 64 bits). The consumer stages its input by polling those words until
// every tag is the current launch's: one L2 round trip after the last write,
// no fences, counters or grid barriers. The grid is a cooperative launch, so
// all CTAs are co-resident and every wait ends; each wait is also limited by
// the global timer (2 s), after which the kernel records an error code and
// gives up instead of hanging.
#include <algorithm>
#include <cstring>
#include <vector>

#include "qi4_common.cuh"
#include "tma_util.cuh"

namespace qi4 {

__device__ int g_chain_error;

namespace {

constexpr int kTileBytes = 512;  // 16 rows x 64 codes
constexpr int kPieceTiles = 32;  // tiles per ring slot
constexpr int kMetaMax = 48;     // scales (32 B) + zero points (8 B) + pad
constexpr int kSlotBytes = kPieceTiles * (kTileBytes + kMetaMax);  // a piece of the largest tile stride
constexpr int kConsumerWarps = 15;  // + the producer: 16 warps (128 registers each)
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;  // + one producer warp
constexpr int kMaxMats = 3;
constexpr int kMaxM = 8;
constexpr int kEntryFloats = 16 * 8;  // one partial: 16 rows x 8 token columns
constexpr int kConsumerBar = 1;       // named barrier id of the consumer warps

// How a stage's input arrives.
constexpr int kInExt16 = 0;  // 16-bit tensor written before the launch
constexpr int kInTag16 = 1;  // mailbox, u32 words: 16-bit value | tag << 16
constexpr int kInTag32 = 2;  // mailbox, u64 words: FP32 value | tag << 32
constexpr int kInExt32 = 3;  // FP32 tensor written before the launch

struct alignas(16) ChainStage {
  const uint8_t* tiles;  // [T][tile_stride] prepacked: 512 B of codes, then the meta bytes
  const void* x;         // [M][K] external input (kInExt16 / kInExt32)
  const void* in_mb;     // [M][K] producer's mailbox (otherwise)
  const float* bias_f32;  // [units][16] FP32 biases in row-block order (null: no bias)
  void* out[kMaxMats];
  void* out_mb[kMaxMats];  // mailbox of each output read by a later stage (or null)
  long long N[kMaxMats];
  int unit_end[kMaxMats];  // cumulative units per matrix
  int T, G, K, U, units;
  int tile_stride, x_dtype, in_fmt, bias_dtype, out_dtype, nmats, swiglu, has_zeros;
};

// The descriptor in 16-byte words (copied into shared memory for each stage).
constexpr int kDescWords = (int)((sizeof(ChainStage) + 15) / 16);

struct ChainParams {
  const ChainStage* stages;
  int nstages;
  int M;
  int nslot;
  int xs_stride;  // bytes per token row of the staged activations
  int xs_bytes;
  int emax;       // partial entries per warp
  int units_max;  // units per CTA, at most
  unsigned* epoch;
  int* exit_cnt;
};

template <int XT>
struct Fmt;
template <>
struct Fmt<QI4_DTYPE_BF16> {
  static constexpr uint32_t kMagic = 0x43004300u;  // 0x4300 | v == 128 + v
};
template <>
struct Fmt<QI4_DTYPE_F16> {
  static constexpr uint32_t kMagic = 0x64006400u;  // 0x6400 | v == 1024 + v
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

// Nibbles i and i+4 of w (w pre-shifted by 4i) -> (magic + c + 8) pair: the
// mask, the XOR 8 that turns a two's-complement nibble into c + 8 and the
// magic exponent in one LOP3 ((a & b) ^ c).
template <int XT>
__device__ __forceinline__ uint32_t nibble_pair(uint32_t w_shifted) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(w_shifted), "r"(0x000F000Fu), "r"(Fmt<XT>::kMagic | 0x00080008u));
  return d;
}

template <int XT>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  if constexpr (XT == QI4_DTYPE_F16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t lds8(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ void sts32(uint32_t a, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}

// Bounded wait for an mbarrier phase, kept compact (one loop, not unrolled:
// the kernel's code must stay small enough for the instruction cache, as every
// stage walks through all of it once). Gives up, recording the error, after
// kWaitLimitNs or once an earlier wait has timed out.
__device__ __forceinline__ void chain_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t start = global_timer_ns();
#pragma unroll 1
  for (;;) {
    if (mbar_try_wait(bar, parity)) return;
    __nanosleep(64);  // a waiting warp leaves the issue slots to the working ones
    if (*reinterpret_cast<volatile int*>(&g_chain_error) != 0) return;
    if (global_timer_ns() - start > kWaitLimitNs) {
      atomicOr(&g_chain_error, kErrWaitTimeout);
      return;
    }
  }
}

// Mailbox stores: morally strong (relaxed, GPU scope), single-copy atomic
// words, so that a reader on another SM sees either the old or the new word.
__device__ __forceinline__ void st_relaxed_u32(void* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_u64(void* p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}


// Staging of a stage's input into shared memory, in the fragment order: per
// token row, per 64-group, the 32 words (element pairs) in the order
// tq * 8 + j <- word 4 j + tq, so that lane tq reads its eight B-fragment
// words of a group as 32 contiguous bytes. FP32 activations: a bf16 hi plane,
// then a lo plane (x - hi, rounded) K * 2 bytes further.
//
// The input - an external tensor, or the producer stage's mailbox - is
// fetched by bulk copies in chunks of kRawHalf bytes into a double-buffered
// raw area (the next chunk in flight while one is converted; no registers
// held across the round trip). A mailbox chunk is checked in shared memory:
// if any word's tag is not this launch's, the chunk is fetched again
// (bounded by the global timer).
constexpr int kRawHalf = 16384;

// Shared-memory offset of the pair word holding elements (e, e + 1), e even.
__device__ __forceinline__ uint32_t pair_offset(int e) {
  const int g = e >> 6, wi = (e & 63) >> 1;
  return (uint32_t)(g * 128 + (((wi & 3) << 3) | (wi >> 2)) * 4);
}

__device__ __forceinline__ void store_pair_f32(uint32_t row, int e, int K, float a, float b) {
  const uint32_t hi = pack_bf16x2(a, b);
  const uint32_t lo = pack_bf16x2(a - __uint_as_float(hi << 16), b - __uint_as_float(hi & 0xFFFF0000u));
  const uint32_t off = pair_offset(e);
  sts32(row + off, hi);
  sts32(row + (uint32_t)(K * 2) + off, lo);
}

// All consumer threads: true if every thread's `ok` is true.
__device__ __forceinline__ bool consumers_all(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)ok), "n"(kConsumerBar), "n"(kConsumers)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// This thread's 16-byte units of chunk c (unit u = tid + k * kConsumers) into
// raw half c % 2, as one async-copy group. Every chunk maps units to threads
// the same way, so a thread only ever reads, checks and converts its own copies.
__device__ __forceinline__ void issue_chunk(uint32_t raw, const uint8_t* src, int c, uint32_t nunits, int tid) {
  const uint32_t dst = raw + (uint32_t)((c & 1) * kRawHalf);
  const uint8_t* from = src + (size_t)c * kRawHalf;
#pragma unroll 1
  for (uint32_t u = tid; u < nunits; u += kConsumers) cp_async16(dst + u * 16, from + u * 16);
  cp_async_commit();
}

// One 16-byte unit of the source at shared address a: false if it carries a
// mailbox tag other than this launch's.
__device__ __forceinline__ bool unit_ready(int fmt, uint32_t a, uint32_t tag16, uint32_t tag32) {
  if (fmt == kInTag16) {
    const uint4 v = lds128(a);
    const uint32_t t = tag16 << 16;
    return ((v.x & 0xFFFF0000u) == t) & ((v.y & 0xFFFF0000u) == t) & ((v.z & 0xFFFF0000u) == t) &
           ((v.w & 0xFFFF0000u) == t);
  }
  if (fmt == kInTag32) {
    const uint4 v = lds128(a);
    return (v.y == tag32) & (v.w == tag32);
  }
  return true;
}

// Converts one 16-byte unit (first element e of token row `row`) into the
// fragment order.
__device__ __forceinline__ void store_unit(int fmt, uint32_t a, uint32_t row, int e, int K) {
  const uint4 v = lds128(a);
  switch (fmt) {
    case kInTag32:
      store_pair_f32(row, e, K, __uint_as_float(v.x), __uint_as_float(v.z));
      break;
    case kInTag16:
      sts32(row + pair_offset(e), (v.x & 0xFFFFu) | (v.y << 16));
      sts32(row + pair_offset(e + 2), (v.z & 0xFFFFu) | (v.w << 16));
      break;
    case kInExt32:
      store_pair_f32(row, e, K, __uint_as_float(v.x), __uint_as_float(v.y));
      store_pair_f32(row, e + 2, K, __uint_as_float(v.z), __uint_as_float(v.w));
      break;
    default:
      sts32(row + pair_offset(e), v.x);
      sts32(row + pair_offset(e + 2), v.y);
      sts32(row + pair_offset(e + 4), v.z);
      sts32(row + pair_offset(e + 6), v.w);
  }
}

// The input - an external tensor, or the producer stage's mailbox - comes in
// chunks of kRawHalf bytes through asynchronous 16-byte copies (the load/store
// path through L2; not the bulk-copy unit, which streams the weights) into a
// double-buffered raw area, the next chunk in flight while one is converted.
// A mailbox unit whose tag is not this launch's is fetched again (bounded).
__device__ __forceinline__ void stage_activations(const ChainStage& st, int M, uint32_t xs, int xs_stride, int tid,
                                               uint32_t raw, uint32_t tag16, uint32_t tag32) {
  const int fmt = st.in_fmt;
  const int E = fmt == kInTag32 ? 2 : (fmt == kInExt16 ? 8 : 4);  // elements per 16-byte unit
  const int EB = 16 / E;                                          // source bytes per element
  const int K = st.K;
  const uint8_t* src = static_cast<const uint8_t*>(fmt == kInExt16 || fmt == kInExt32 ? st.x : st.in_mb);
  const int64_t total = (int64_t)M * K * EB;
  const int nchunks = (int)((total + kRawHalf - 1) / kRawHalf);
  auto chunk_units = [&](int c) {
    const int64_t left = total - (int64_t)c * kRawHalf;
    return (uint32_t)((left < kRawHalf ? left : kRawHalf) / 16);
  };
  issue_chunk(raw, src, 0, chunk_units(0), tid);
#pragma unroll 1
  for (int c = 0; c < nchunks; ++c) {
    if (c + 1 < nchunks)
      issue_chunk(raw, src, c + 1, chunk_units(c + 1), tid);
    else
      cp_async_commit();  // empty group: the wait below still leaves one group pending
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    const uint32_t nunits = chunk_units(c);
    const uint32_t base = raw + (uint32_t)((c & 1) * kRawHalf);
    bool ok = true;
#pragma unroll 1
    for (uint32_t u = tid; u < nunits; u += kConsumers) ok = ok & unit_ready(fmt, base + u * 16, tag16, tag32);
    if (!consumers_all(ok)) {
      // Some word is not written yet: fetch this chunk again (bounded).
      const uint64_t start = global_timer_ns();
#pragma unroll 1
      for (;;) {
        issue_chunk(raw, src, c, nunits, tid);
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        ok = true;
#pragma unroll 1
        for (uint32_t u = tid; u < nunits; u += kConsumers) ok = ok & unit_ready(fmt, base + u * 16, tag16, tag32);
        if (consumers_all(ok)) break;
        const bool give_up = *reinterpret_cast<volatile int*>(&g_chain_error) != 0 ||
                             global_timer_ns() - start > kWaitLimitNs;
        if (!consumers_all(!give_up)) {
          if (tid == 0) atomicOr(&g_chain_error, kErrWaitTimeout);
          break;
        }
      }
    }
    const int64_t e0 = (int64_t)c * kRawHalf / EB;  // first element of the chunk
#pragma unroll 1
    for (uint32_t u = tid; u < nunits; u += kConsumers) {
      const int64_t e = e0 + (int64_t)u * E;
      const int t = (int)(e / K);
      store_unit(fmt, base + u * 16, xs + (uint32_t)(t * xs_stride), (int)(e - (int64_t)t * K), K);
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// A tile's contribution to acc (rows gq / gq + 8 of the tile, tokens 2 tq,
// 2 tq + 1): scale * sum_k (c - z) x over the tile's 64 k. One LOP3 per
// register pair gives (magic + 8 + c) (mask, XOR 8 of the two's-complement
// nibble, magic exponent), one packed subtract of (magic + 8 + z) leaves the
// exact integer c - z; products with the activations are exact and sums FP32.
// Two independent MMA chains per tile (even / odd k steps, or the bf16 hi / lo
// planes of FP32 activations).
struct TileOps {
  uint4 cw;
  uint32_t sc, zl, zh;
  uint4 x0, x1, l0, l1;
};

template <int MT, bool TWO>
__device__ __forceinline__ void tile_load(TileOps& o, uint32_t codes, uint32_t meta, int has_zeros, uint32_t xg,
                                          uint32_t lo_off, int lane) {
  const int gq = lane >> 2;
  o.cw = lds128(codes + lane * 16);
  o.sc = lds32(meta + gq * 4);
  o.zl = o.zh = Fmt<MT>::kMagic + 0x00080008u;  // magic + 8 + z, z = 0
  if (has_zeros) {
    const uint32_t zb = lds8(meta + 32 + gq);
    o.zl = Fmt<MT>::kMagic + ((zb & 0xFu) ^ 0x8u) * 0x00010001u;
    o.zh = Fmt<MT>::kMagic + (((zb >> 4) & 0xFu) ^ 0x8u) * 0x00010001u;
  }
  o.x0 = lds128(xg);
  o.x1 = lds128(xg + 16);
  if constexpr (TWO) {
    o.l0 = lds128(xg + lo_off);
    o.l1 = lds128(xg + lo_off + 16);
  }
}

// TWO: FP32 activations (bf16 hi and lo planes, one MMA chain each).
template <int MT, bool TWO>
__device__ __forceinline__ void tile_math(float (&acc)[4], const TileOps& o) {
  const uint32_t words[4] = {o.cw.x, o.cw.y, o.cw.z, o.cw.w};
  const uint32_t xw[8] = {o.x0.x, o.x0.y, o.x0.z, o.x0.w, o.x1.x, o.x1.y, o.x1.z, o.x1.w};
  float da[4] = {0.f, 0.f, 0.f, 0.f}, db[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const uint32_t w = words[s];
    const uint32_t a0 = sub2<MT>(nibble_pair<MT>(w), o.zl);
    const uint32_t a1 = sub2<MT>(nibble_pair<MT>(w >> 4), o.zh);
    const uint32_t a2 = sub2<MT>(nibble_pair<MT>(w >> 8), o.zl);
    const uint32_t a3 = sub2<MT>(nibble_pair<MT>(w >> 12), o.zh);
    if constexpr (TWO) {
      const uint32_t lw[8] = {o.l0.x, o.l0.y, o.l0.z, o.l0.w, o.l1.x, o.l1.y, o.l1.z, o.l1.w};
      mma16816<MT>(da, a0, a1, a2, a3, xw[2 * s], xw[2 * s + 1]);
      mma16816<MT>(db, a0, a1, a2, a3, lw[2 * s], lw[2 * s + 1]);
    } else if (s & 1) {
      mma16816<MT>(db, a0, a1, a2, a3, xw[2 * s], xw[2 * s + 1]);
    } else {
      mma16816<MT>(da, a0, a1, a2, a3, xw[2 * s], xw[2 * s + 1]);
    }
  }
  const float2 sc = __half22float2(*reinterpret_cast<const __half2*>(&o.sc));
  acc[0] = fmaf(sc.x, da[0] + db[0], acc[0]);
  acc[1] = fmaf(sc.x, da[1] + db[1], acc[1]);
  acc[2] = fmaf(sc.y, da[2] + db[2], acc[2]);
  acc[3] = fmaf(sc.y, da[3] + db[3], acc[3]);
}

__device__ __forceinline__ void store_value(void* out, int dtype, int64_t i, float v, void* mb, uint32_t tag16,
                                            uint32_t tag32) {
  if (dtype == QI4_DTYPE_F32) {
    static_cast<float*>(out)[i] = v;
    if (mb) st_relaxed_u64(static_cast<uint64_t*>(mb) + i, (uint64_t)__float_as_uint(v) | ((uint64_t)tag32 << 32));
  } else {
    const uint16_t bits = dtype == QI4_DTYPE_BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                                  : __half_as_ushort(__float2half_rn(v));
    static_cast<uint16_t*>(out)[i] = bits;
    if (mb) st_relaxed_u32(static_cast<uint32_t*>(mb) + i, (uint32_t)bits | (tag16 << 16));
  }
}

template <int MT, bool TWO>
__device__ __forceinline__ int compute_tiles(int t0, int t1, int aw, int bw, int G, int tile_stride, int has_zeros,
                                          int nslot, int pc, uint32_t ring, uint64_t* full, uint64_t* empty,
                                          uint32_t xrow, uint32_t lo_off, uint32_t red_w, int lane) {
  const int n = t1 - t0;
  const int npieces = (n + kPieceTiles - 1) / kPieceTiles;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int seg0 = aw / G;
  int seg = seg0, g = aw - seg0 * G;
  const int gq = lane >> 2, tq = lane & 3;
  const uint32_t e_lo = (uint32_t)((gq * 8 + 2 * tq) * 4), e_hi = (uint32_t)(((gq + 8) * 8 + 2 * tq) * 4);
#pragma unroll 1
  for (int pi = 0; pi < npieces; ++pi, ++pc) {
    const int slot = pc % nslot;
    const int pbeg = t0 + pi * kPieceTiles;
    const int lo = max(aw, pbeg), hi = min(bw, pbeg + kPieceTiles);
    // Every warp waits for every piece of the stage before releasing it, even
    // one with none of its tiles: an arrival for a slot's next use must not
    // land before the arrivals of its current use are complete.
    chain_wait(full + slot, (uint32_t)((pc / nslot) & 1));
    const uint32_t piece = ring + (uint32_t)slot * kSlotBytes;
#pragma unroll 1
    for (int t = lo; t < hi; ++t) {
      if (g == G) {  // next row block: park this one's sums ([row][token])
        const uint32_t e = red_w + (uint32_t)((seg - seg0) * kEntryFloats * 4);
        asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(e + e_lo), "f"(acc[0]), "f"(acc[1]));
        asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(e + e_hi), "f"(acc[2]), "f"(acc[3]));
        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
        ++seg;
        g = 0;
      }
      const int i = t - pbeg;
      TileOps o;
      const uint32_t tile = piece + (uint32_t)(i * tile_stride);
      tile_load<MT, TWO>(o, tile, tile + kTileBytes, has_zeros, xrow + (uint32_t)(g * 128), lo_off, lane);
      tile_math<MT, TWO>(acc, o);
      ++g;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty + slot);
  }
  if (aw < bw) {
    const uint32_t e = red_w + (uint32_t)((seg - seg0) * kEntryFloats * 4);
    asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(e + e_lo), "f"(acc[0]), "f"(acc[1]));
    asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(e + e_hi), "f"(acc[2]), "f"(acc[3]));
  }
  return pc;
}

__device__ __forceinline__ float round_to(int dtype, float v) {
  if (dtype == QI4_DTYPE_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == QI4_DTYPE_F16) return __half2float(__float2half_rn(v));
  return v;
}

__device__ __forceinline__ void reduce_store(const ChainStage& st, int ua, int ub, int t0, int n, int M, int emax,
                                             const float* red,
                                          const float* bias_s, const int* wseg, uint32_t tag16, uint32_t tag32) {
  const int items = (ub - ua) * 16 * M;
  for (int it = threadIdx.x; it < items; it += kConsumers) {
    const int ul = it / (16 * M), rem = it - ul * 16 * M;
    const int r = rem / M, tok = rem - r * M;
    const int u = ua + ul;
    // Only the warps whose contiguous share overlaps the unit (two or three)
    // contributed: the warp of tile t is ((t - t0 + 1) W - 1) / n. Scalars,
    // not a runtime-indexed local array.
    const int tf = u * st.U * st.G - t0, tl = tf + st.U * st.G - 1;
    const int w0 = min(kConsumerWarps - 1, ((tf + 1) * kConsumerWarps - 1) / n);
    const int w1 = min(kConsumerWarps - 1, ((tl + 1) * kConsumerWarps - 1) / n);
    const int sg0 = u * st.U, sg1 = sg0 + st.U - 1;
    float v0 = 0.f, v1 = 0.f;
#pragma unroll 1
    for (int w = w0; w <= w1; ++w) {
      const int s0 = wseg[2 * w], s1 = wseg[2 * w + 1];
      const float* e = red + (size_t)w * emax * kEntryFloats + r * 8 + tok;
      if (s0 <= sg0 && sg0 <= s1) v0 += e[(size_t)(sg0 - s0) * kEntryFloats];
      if (sg1 != sg0 && s0 <= sg1 && sg1 <= s1) v1 += e[(size_t)(sg1 - s0) * kEntryFloats];
    }
    const float v[2] = {v0, v1};  // constant indices only
    if (st.swiglu) {
      const int64_t row = (int64_t)u * 16 + r;
      if (row < st.N[0]) {
        const float gv = round_to(st.x_dtype, v[0]), up = round_to(st.x_dtype, v[1]);
        store_value(st.out[0], QI4_DTYPE_F32, (int64_t)tok * st.N[0] + row, gv / (1.0f + expf(-gv)) * up,
                    st.out_mb[0], tag16, tag32);
      }
    } else {
      const int m = (st.nmats > 1 && u >= st.unit_end[0]) + (st.nmats > 2 && u >= st.unit_end[1]);
      const int64_t row = (int64_t)(u - (m ? st.unit_end[m - 1] : 0)) * 16 + r;
      if (row < st.N[m])
        store_value(st.out[m], st.out_dtype, (int64_t)tok * st.N[m] + row,
                    v[0] + (st.bias_f32 ? bias_s[ul * 16 + r] : 0.f), st.out_mb[m], tag16, tag32);
    }
  }
}

// The consumer warps' part of one stage.
template <int MT>
__device__ void consume_stage(const ChainStage& st, const ChainParams& p, uint8_t* ring, uint64_t* full,
                              uint64_t* empty, uint32_t xs, float* red, float* bias_s, int* wseg,
                              int& pc, uint32_t raw, uint32_t tag16, uint32_t tag32) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int M = p.M;
  const int P = (int)gridDim.x, c = (int)blockIdx.x;
  const int ua = (int)((int64_t)c * st.units / P), ub = (int)((int64_t)(c + 1) * st.units / P);
  if (ua == ub) return;  // no row block of this stage here
  const int G = st.G, UG = st.U * G;
  const int t0 = ua * UG, t1 = ub * UG, n = t1 - t0;

  // 1. Biases of this CTA's rows (constant: fetched asynchronously, waited for
  // with the input copies), then the input, polled from the producer's mailbox.
  if (st.bias_f32 && tid < (ub - ua) * 4)
    cp_async16(smem_addr(bias_s) + tid * 16, st.bias_f32 + (size_t)ua * 16 + tid * 4);
  cp_async_commit();
  stage_activations(st, M, xs, p.xs_stride, tid, raw, tag16, tag32);
  named_barrier(kConsumerBar, kConsumers);  // every thread's units are staged
  const uint32_t lo_off = st.x_dtype == QI4_DTYPE_F32 ? (uint32_t)(st.K * 2) : 0u;

  // 2. This warp's contiguous share of the CTA's tiles.
  const int aw = t0 + (n * warp) / kConsumerWarps, bw = t0 + (n * (warp + 1)) / kConsumerWarps;
  if (lane == 0) {
    wseg[2 * warp] = aw < bw ? aw / G : 1;
    wseg[2 * warp + 1] = aw < bw ? (bw - 1) / G : 0;
  }
  const int gq = lane >> 2, tq = lane & 3;
  const uint32_t xrow = xs + (uint32_t)(min(gq, M - 1) * p.xs_stride + tq * 32);
  const uint32_t red_w = smem_addr(red + (size_t)warp * p.emax * kEntryFloats);
  if (lo_off)
    pc = compute_tiles<MT, true>(t0, t1, aw, bw, G, st.tile_stride, st.has_zeros, p.nslot, pc, smem_addr(ring), full,
                                 empty, xrow, lo_off, red_w, lane);
  else
    pc = compute_tiles<MT, false>(t0, t1, aw, bw, G, st.tile_stride, st.has_zeros, p.nslot, pc, smem_addr(ring), full,
                                  empty, xrow, 0u, red_w, lane);
  named_barrier(kConsumerBar, kConsumers);

  // 3. Outputs.
  reduce_store(st, ua, ub, t0, n, M, p.emax, red, bias_s, wseg, tag16, tag32);
}

// MT: the MMA operand type of the 16-bit stages (bf16, or f16); FP32 stages
// run as bf16 hi / lo planes and need MT = bf16.
template <int MT>
__global__ void __launch_bounds__(kThreads, 1) decode_chain_kernel(const ChainParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u);
  uint8_t* ring = smem;
  uint8_t* xs = ring + (size_t)p.nslot * kSlotBytes;
  uint8_t* raw = xs + p.xs_bytes;  // 2 x kRawHalf
  float* red = reinterpret_cast<float*>(raw + 2 * kRawHalf);
  float* bias_s = red + (size_t)kConsumerWarps * p.emax * kEntryFloats;
  int* wseg = reinterpret_cast<int*>(bias_s + (size_t)p.units_max * 16);
  uint64_t* full = reinterpret_cast<uint64_t*>(wseg + 2 * kConsumerWarps);
  uint64_t* empty = full + p.nslot;
  uint8_t* after_bars = reinterpret_cast<uint8_t*>(empty + p.nslot);
  ChainStage* sdesc = reinterpret_cast<ChainStage*>(after_bars + ((16u - (smem_addr(after_bars) & 15u)) & 15u));  // [2]
  unsigned* epoch_s = reinterpret_cast<unsigned*>(sdesc + 2);
  const int tid = threadIdx.x;
  if (tid == 0) {
    for (int i = 0; i < p.nslot; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, kConsumerWarps);
    }
    fence_barrier_init();
    *epoch_s = *reinterpret_cast<volatile unsigned*>(p.epoch);
  }
  __syncthreads();
  const unsigned epoch = *epoch_s;
  const uint32_t tag16 = epoch % 65535u + 1u, tag32 = epoch + 1u;

  if (tid >= kConsumers) {
    // Producer: one thread streams this CTA's units of every stage into the
    // ring, as far ahead as free slots allow.
    if (tid == kConsumers) {
      const uint64_t policy = l2_evict_first_policy();
      int pc = 0;
      const int P = (int)gridDim.x, c = (int)blockIdx.x;
      for (int s = 0; s < p.nstages; ++s) {
        const ChainStage& st = p.stages[s];
        const int ua = (int)((int64_t)c * st.units / P), ub = (int)((int64_t)(c + 1) * st.units / P);
        const int UG = st.U * st.G, t0 = ua * UG, t1 = ub * UG;
        for (int t = t0; t < t1; t += kPieceTiles, ++pc) {
          const int nt = min(kPieceTiles, t1 - t);
          const int slot = pc % p.nslot;
          chain_wait(empty + slot, (uint32_t)(((pc / p.nslot) & 1) ^ 1));
          uint8_t* dst = ring + (size_t)slot * kSlotBytes;
          // One copy per piece: the bulk-copy unit's cost is per copy (about
          // 0.3 us per SM up to 16 KB), so tiles and their meta are one range.
          const uint32_t bytes = (uint32_t)(nt * st.tile_stride);
          mbar_arrive_expect_tx(full + slot, bytes);
          bulk_load_1d(dst, st.tiles + (size_t)t * st.tile_stride, bytes, full + slot, policy);
        }
      }
      // Every copy issued has landed before the CTA may exit (normally the
      // consumers have seen them all already).
      for (int i = max(0, pc - p.nslot); i < pc; ++i)
        chain_wait(full + (i % p.nslot), (uint32_t)((i / p.nslot) & 1));
    }
  } else {
    int pc = 0;
    const uint32_t xsa = smem_addr(xs);
    const uint32_t rawa = smem_addr(raw);
    // Stage descriptors are read from shared memory: the next one is copied
    // in (async) while a stage runs. Read from global memory, every field of a
    // descriptor not in L1 (which is small with this much shared memory) is an
    // L2 round trip on the critical path of the stage.
    const uint4* gdesc = reinterpret_cast<const uint4*>(p.stages);
    if (tid < kDescWords) reinterpret_cast<uint4*>(sdesc)[tid] = gdesc[tid];
    named_barrier(kConsumerBar, kConsumers);
    for (int s = 0; s < p.nstages; ++s) {
      const ChainStage& st = sdesc[s & 1];
      if (tid < kDescWords && s + 1 < p.nstages) {
        cp_async16(smem_addr(sdesc + ((s + 1) & 1)) + tid * 16, gdesc + (size_t)(s + 1) * kDescWords + tid);
      }
      cp_async_commit();
      consume_stage<MT>(st, p, ring, full, empty, xsa, red, bias_s, wseg, pc, rawa, tag16, tag32);
      asm volatile("cp.async.wait_group 0;" ::: "memory");
      named_barrier(kConsumerBar, kConsumers);  // next descriptor visible; this one no longer read
    }
  }

  // The last CTA to leave advances the launch epoch (every CTA read it at its
  // start), so the next launch's mailbox tags differ from this one's.
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(p.exit_cnt, 1) == (int)gridDim.x - 1) {
      *p.exit_cnt = 0;
      atomicAdd(p.epoch, 1u);
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------------------
// Load-time prepack: canonical W4G64 -> tile-major
// ---------------------------------------------------------------------------
// Tile (rb, g) of one matrix becomes stage tile ((unit0 + rb) * U + j) * G + g.
// One thread per (tile, lane): the lane's 16 bytes of codes; lanes with
// tq == 0 also write the scale pair (and zero-point byte) of rows gq, gq + 8.
__global__ void prepack_kernel(const uint8_t* __restrict__ qweight, const __half* __restrict__ scales,
                               const uint8_t* __restrict__ zeros, int64_t N, int K, int nb, int U, int j,
                               int unit0, uint8_t* __restrict__ tiles, int tile_stride) {
  const int G = K >> 6;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t tile = idx >> 5;
  if (tile >= (int64_t)nb * G) return;
  const int lane = (int)(idx & 31), gq = lane >> 2, tq = lane & 3;
  const int rb = (int)(tile / G), g = (int)(tile - (int64_t)rb * G);
  const int64_t t = ((int64_t)(unit0 + rb) * U + j) * G + g;
  const int64_t r0 = (int64_t)rb * 16 + gq, r1 = r0 + 8;
  auto byte_at = [&](int64_t r, int k) -> uint32_t {
    return r < N ? (uint32_t)__ldg(qweight + ((r * K + k) >> 1)) : 0u;
  };
  uint32_t w[4];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const int k0 = g * 64 + 16 * s + 2 * tq;
    const uint32_t b00 = byte_at(r0, k0), b01 = byte_at(r0, k0 + 8), b10 = byte_at(r1, k0), b11 = byte_at(r1, k0 + 8);
    // nibble i holds the even k of fragment register i, nibble i + 4 the odd k.
    w[s] = (b00 & 0xF) | ((b10 & 0xF) << 4) | ((b01 & 0xF) << 8) | ((b11 & 0xF) << 12) | ((b00 >> 4) << 16) |
           ((b10 >> 4) << 20) | ((b01 >> 4) << 24) | ((b11 >> 4) << 28);
  }
  *reinterpret_cast<uint4*>(tiles + t * tile_stride + lane * 16) = make_uint4(w[0], w[1], w[2], w[3]);
  if (tq == 0) {
    uint8_t* m = tiles + t * tile_stride + kTileBytes;
    const __half s0 = r0 < N ? scales[r0 * G + g] : __float2half(0.f);
    const __half s1 = r1 < N ? scales[r1 * G + g] : __float2half(0.f);
    *reinterpret_cast<__half2*>(m + gq * 4) = __halves2half2(s0, s1);
    if (tile_stride > kTileBytes + 32) {
      auto znib = [&](int64_t r) -> uint32_t {
        if (r >= N || zeros == nullptr) return 0u;
        const int64_t zi = r * G + g;
        return (uint32_t)(zeros[zi >> 1] >> ((zi & 1) * 4)) & 0xFu;
      };
      m[32 + gq] = (uint8_t)(znib(r0) | (znib(r1) << 4));
      m[40 + gq] = 0;
    }
  }
}

// Biases of one matrix into FP32 row-block order (rows past N are 0).
__global__ void prepack_bias_kernel(const void* __restrict__ bias, int dtype, int64_t N, int nb, int unit0,
                                    float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nb * 16) return;
  const int64_t row = i;
  out[(size_t)unit0 * 16 + i] = (bias && row < N) ? load_as_f32(bias, dtype, row) : 0.f;
}

}  // namespace

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

struct Chain {
  int device = -1;
  int M = 0;
  int nstages = 0;
  ChainParams params{};
  size_t smem = 0;
  int grid = 0;
  std::vector<ChainStage> host_stages;
  std::vector<void*> allocations;
  int mma_type = QI4_DTYPE_BF16;  // kernel instance: MMA operand type of the 16-bit stages
  int64_t weight_bytes = 0;  // prepacked bytes streamed per run
  int64_t alg_bytes = 0;     // algorithmic bytes per run (canonical formula)
};

namespace {

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

void free_chain(Chain* c) {
  for (void* p : c->allocations) cudaFree(p);
  delete c;
}

bool act_dtype(int d) { return d == QI4_DTYPE_BF16 || d == QI4_DTYPE_F16 || d == QI4_DTYPE_F32; }

}  // namespace

}  // namespace qi4

using qi4::Chain;

extern "C" {

QI4_API int qi4_chain_create(const qi4_chain_stage* stages, int n_stages, int64_t M, void* stream_ptr,
                             qi4_chain** out) {
  using namespace qi4;
  clear_error();
  if (!stages || !out || n_stages <= 0) {
    set_error("stages and out must be non-null and n_stages positive");
    return QI4_ERR_ARGUMENT;
  }
  *out = nullptr;
  if (M < 1 || M > kMaxM) {
    set_error("the decode chain takes 1 <= M <= %d tokens (got %lld)", kMaxM, (long long)M);
    return QI4_ERR_SHAPE;
  }
  // Validate every stage, and find the stage (and matrix) that produces each
  // stage's input, before touching the device.
  std::vector<int> src_stage(n_stages, -1), src_mat(n_stages, -1);
  for (int s = 0; s < n_stages; ++s) {
    const qi4_chain_stage& d = stages[s];
    const bool sw = (d.flags & QI4_CHAIN_SWIGLU) != 0;
    if (d.nmats < 1 || d.nmats > kMaxMats || (sw && d.nmats != 2) || (d.flags & ~QI4_CHAIN_SWIGLU)) {
      set_error("stage %d: nmats must be 1..3 (2 for a SwiGLU stage) and flags known", s);
      return QI4_ERR_ARGUMENT;
    }
    if (!d.x) {
      set_error("stage %d: x must be non-null", s);
      return QI4_ERR_ARGUMENT;
    }
    if (d.K <= 0 || d.K % 64 || d.K > (1 << 20)) {
      set_error("stage %d: K must be a positive multiple of 64 (got %lld)", s, (long long)d.K);
      return QI4_ERR_SHAPE;
    }
    if (!act_dtype(d.x_dtype) || (!sw && !act_dtype(d.out_dtype))) {
      set_error("stage %d: activation / output dtype is not F16, BF16 or F32", s);
      return QI4_ERR_DTYPE;
    }
    if (reinterpret_cast<uintptr_t>(d.x) % 16) {
      set_error("stage %d: x must be 16-byte aligned", s);
      return QI4_ERR_ALIGNMENT;
    }
    for (int m = 0; m < d.nmats; ++m) {
      if (!d.qweight[m] || !d.scales_f16[m] || (!d.out[m] && !(sw && m == 1)) || d.N[m] <= 0 || d.N[m] > (1 << 24)) {
        set_error("stage %d matrix %d: qweight, scales and out must be non-null and N positive", s, m);
        return QI4_ERR_ARGUMENT;
      }
      if (d.bias[m] && !act_dtype(d.bias_dtype)) {
        set_error("stage %d: bias dtype %d is not F16, BF16 or F32", s, d.bias_dtype);
        return QI4_ERR_DTYPE;
      }
      if (sw && d.bias[m]) {
        set_error("stage %d: the SwiGLU stage takes no bias", s);
        return QI4_ERR_ARGUMENT;
      }
    }
    if (sw && d.N[0] != d.N[1]) {
      set_error("stage %d: gate and up must have the same N", s);
      return QI4_ERR_SHAPE;
    }
    // Producer of x: an output of an earlier stage (same pointer), else external.
    for (int q = 0; q < n_stages; ++q) {
      const qi4_chain_stage& e = stages[q];
      const bool esw = (e.flags & QI4_CHAIN_SWIGLU) != 0;
      for (int m = 0; m < (esw ? 1 : e.nmats); ++m) {
        if (e.out[m] != d.x) continue;
        if (q >= s) {
          set_error("stage %d reads the output of stage %d, which does not come before it", s, q);
          return QI4_ERR_ARGUMENT;
        }
        const int64_t n = e.N[m];
        const int odt = esw ? QI4_DTYPE_F32 : e.out_dtype;
        if (odt != d.x_dtype || n != d.K) {
          set_error("stage %d reads stage %d's output: dtype and width must match (K %lld vs N %lld)", s, q,
                    (long long)d.K, (long long)n);
          return QI4_ERR_SHAPE;
        }
        src_stage[s] = q;
        src_mat[s] = m;
      }
    }
  }
  // One kernel instance per MMA operand type: bf16 (bf16 and FP32 stages) or
  // f16 (f16 stages only: FP32 inputs run as bf16 hi / lo planes).
  bool has_f16 = false, has_f32 = false;
  for (int s = 0; s < n_stages; ++s) {
    has_f16 = has_f16 || stages[s].x_dtype == QI4_DTYPE_F16;
    has_f32 = has_f32 || stages[s].x_dtype == QI4_DTYPE_F32;
  }
  if (has_f16 && has_f32) {
    set_error("a decode chain cannot mix float16 and float32 activations (float32 runs as bfloat16 planes)");
    return QI4_ERR_DTYPE;
  }
  // Outputs must be distinct buffers (a run writes each once).
  for (int s = 0; s < n_stages; ++s)
    for (int m = 0; m < stages[s].nmats; ++m)
      for (int q = s; q < n_stages; ++q)
        for (int k = (q == s ? m + 1 : 0); k < stages[q].nmats; ++k)
          if (stages[s].out[m] && stages[s].out[m] == stages[q].out[k]) {
            set_error("stages %d and %d write the same output buffer", s, q);
            return QI4_ERR_ARGUMENT;
          }

  int dev = 0, sms = 0, major = 0, smem_optin = 0, coop = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess) {
    cudaGetLastError();
    set_error("no usable CUDA device");
    return QI4_ERR_DEVICE;
  }
  if (major != 10) {
    set_error("device %d has compute capability %d.x; this library is built for sm_100a (B200)", dev, major);
    return QI4_ERR_DEVICE;
  }
  if (!coop) {
    set_error("device %d does not support cooperative launches", dev);
    return QI4_ERR_DEVICE;
  }
  // Shared-memory plan: staged activations, warp partials, biases, ring.
  int64_t max_xs = 0, emax = 1, units_max = 1;
  for (int s = 0; s < n_stages; ++s) {
    const qi4_chain_stage& d = stages[s];
    const bool sw = (d.flags & QI4_CHAIN_SWIGLU) != 0;
    const int64_t G = d.K / 64, U = sw ? 2 : 1;
    int64_t units = 0;
    for (int m = 0; m < (sw ? 1 : d.nmats); ++m) units += ceil_div(d.N[m], 16);
    if (units * U * G > (int64_t)1 << 30) {
      set_error("stage %d is too large for the decode chain", s);
      return QI4_ERR_SHAPE;
    }
    const int64_t per_cta = ceil_div(units, sms);
    units_max = std::max<int64_t>(units_max, per_cta);
    max_xs = std::max<int64_t>(max_xs, M * (d.K * (d.x_dtype == QI4_DTYPE_F32 ? 4 : 2) + 16));
    emax = std::max<int64_t>(emax, ceil_div(ceil_div(per_cta * U * G, kConsumerWarps), G) + 1);
  }
  const size_t fixed = 128 + (size_t)max_xs + 2 * kRawHalf + 16 + 2 * (size_t)kDescWords * 16 +
                       (size_t)kConsumerWarps * emax * kEntryFloats * 4 +
                       (size_t)units_max * 16 * 4 + 2 * kConsumerWarps * 4 + 64;
  const int64_t nslot = ((int64_t)smem_optin - (int64_t)fixed) / (kSlotBytes + 16);
  if (nslot < 2) {
    set_error("the decode chain does not fit in shared memory at M=%lld (activations %lld bytes, %lld row "
              "blocks per CTA)", (long long)M, (long long)max_xs, (long long)units_max);
    return QI4_ERR_SHAPE;
  }

  Chain* c = new Chain();
  c->device = dev;
  c->M = (int)M;
  c->nstages = n_stages;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  auto alloc = [&](size_t bytes) -> void* {
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
    c->allocations.push_back(p);
    return p;
  };
  int rc = QI4_OK;
  // Mailboxes for every output that a later stage reads.
  std::vector<std::vector<void*>> mbox(n_stages, std::vector<void*>(kMaxMats, nullptr));
  for (int s = 0; s < n_stages && rc == QI4_OK; ++s) {
    if (src_stage[s] < 0) continue;
    const int q = src_stage[s], m = src_mat[s];
    if (mbox[q][m]) continue;
    const bool f32 = (stages[q].flags & QI4_CHAIN_SWIGLU) || stages[q].out_dtype == QI4_DTYPE_F32;
    const size_t bytes = (size_t)M * stages[q].N[m] * (f32 ? 8 : 4);
    mbox[q][m] = alloc(bytes);
    if (!mbox[q][m]) {
      rc = QI4_ERR_LAUNCH;
      break;
    }
    cudaMemsetAsync(mbox[q][m], 0, bytes, stream);  // tag 0: never a launch's tag
  }
  for (int s = 0; s < n_stages && rc == QI4_OK; ++s) {
    const qi4_chain_stage& d = stages[s];
    const bool sw = (d.flags & QI4_CHAIN_SWIGLU) != 0;
    ChainStage st{};
    st.K = (int)d.K;
    st.G = (int)(d.K / 64);
    st.U = sw ? 2 : 1;
    st.swiglu = sw;
    st.nmats = d.nmats;
    st.x = d.x;
    st.x_dtype = d.x_dtype;
    st.out_dtype = sw ? QI4_DTYPE_F32 : d.out_dtype;
    st.bias_dtype = d.bias_dtype;
    if (src_stage[s] >= 0) {
      const int q = src_stage[s];
      st.in_mb = mbox[q][src_mat[s]];
      st.in_fmt = ((stages[q].flags & QI4_CHAIN_SWIGLU) || stages[q].out_dtype == QI4_DTYPE_F32) ? kInTag32 : kInTag16;
    } else {
      st.in_fmt = d.x_dtype == QI4_DTYPE_F32 ? kInExt32 : kInExt16;
    }
    bool zeros = false;
    for (int m = 0; m < d.nmats; ++m) zeros = zeros || d.zeros[m] != nullptr;
    st.has_zeros = zeros;
    st.tile_stride = kTileBytes + (zeros ? 48 : 32);
    int units = 0;
    bool any_bias = false;
    for (int m = 0; m < d.nmats; ++m) {
      st.N[m] = d.N[m];
      any_bias = any_bias || d.bias[m] != nullptr;
      st.out[m] = d.out[m];
      st.out_mb[m] = mbox[s][m];
      if (!sw || m == 0) units += (int)ceil_div(d.N[m], 16);
      st.unit_end[m] = units;
    }
    st.units = units;
    st.T = units * st.U * st.G;
    if (any_bias && !sw) {
      float* bf = static_cast<float*>(alloc((size_t)units * 16 * sizeof(float)));
      if (!bf) {
        rc = QI4_ERR_LAUNCH;
        break;
      }
      int u0 = 0;
      for (int m = 0; m < d.nmats; ++m) {
        const int nb = (int)ceil_div(d.N[m], 16);
        prepack_bias_kernel<<<(unsigned)ceil_div(nb * 16, 256), 256, 0, stream>>>(d.bias[m], d.bias_dtype, d.N[m],
                                                                                 nb, u0, bf);
        u0 += nb;
      }
      st.bias_f32 = bf;
    }
    uint8_t* tiles = static_cast<uint8_t*>(alloc((size_t)st.T * st.tile_stride));
    if (!tiles) {
      rc = QI4_ERR_LAUNCH;
      break;
    }
    st.tiles = tiles;
    int unit0 = 0;
    for (int m = 0; m < d.nmats; ++m) {
      const int nb = (int)ceil_div(d.N[m], 16);
      const int64_t threads = (int64_t)nb * st.G * 32;
      prepack_kernel<<<(unsigned)ceil_div(threads, 256), 256, 0, stream>>>(
          d.qweight[m], reinterpret_cast<const __half*>(d.scales_f16[m]), d.zeros[m], d.N[m], st.K, nb, st.U,
          sw ? m : 0, sw ? 0 : unit0, tiles, st.tile_stride);
      if (!sw) unit0 += nb;
      c->alg_bytes += d.N[m] * d.K / 2 + d.N[m] * st.G * 2 + (d.zeros[m] ? (d.N[m] * st.G + 1) / 2 : 0) +
                      (d.bias[m] ? d.N[m] * 2 : 0) + M * d.N[m] * 2;
    }
    c->alg_bytes += M * d.K * 2;
    c->weight_bytes += (int64_t)st.T * st.tile_stride;
    c->host_stages.push_back(st);
  }
  if (rc == QI4_OK && cudaGetLastError() != cudaSuccess) rc = QI4_ERR_LAUNCH;
  ChainStage* dstages = nullptr;
  int* counters = nullptr;
  if (rc == QI4_OK) {
    dstages = static_cast<ChainStage*>(alloc(sizeof(ChainStage) * n_stages));
    counters = static_cast<int*>(alloc(sizeof(int) * 2));
    if (!dstages || !counters) rc = QI4_ERR_LAUNCH;
  }
  if (rc == QI4_OK) {
    cudaMemcpyAsync(dstages, c->host_stages.data(), sizeof(ChainStage) * n_stages, cudaMemcpyHostToDevice, stream);
    cudaMemsetAsync(counters, 0, sizeof(int) * 2, stream);
    if (cudaStreamSynchronize(stream) != cudaSuccess) rc = QI4_ERR_LAUNCH;
  }
  if (rc != QI4_OK) {
    cudaGetLastError();
    set_error("decode chain set-up failed on the device (allocation, prepack or copy)");
    free_chain(c);
    return rc;
  }
  ChainParams& p = c->params;
  p.stages = dstages;
  p.nstages = n_stages;
  p.M = (int)M;
  p.nslot = (int)std::min<int64_t>(nslot, 64);
  p.xs_bytes = (int)((max_xs + 15) / 16 * 16);
  p.xs_stride = (int)(max_xs / M);
  p.emax = (int)emax;
  p.units_max = (int)units_max;
  p.epoch = reinterpret_cast<unsigned*>(counters);
  p.exit_cnt = counters + 1;
  c->smem = 128 + (size_t)p.nslot * kSlotBytes + p.xs_bytes + 2 * kRawHalf +
            (size_t)kConsumerWarps * p.emax * kEntryFloats * 4 + (size_t)p.units_max * 16 * 4 + 2 * kConsumerWarps * 4 +
            (size_t)p.nslot * 16 + 16 + 2 * (size_t)kDescWords * 16 + 16;
  c->grid = sms;
  c->mma_type = has_f16 ? QI4_DTYPE_F16 : QI4_DTYPE_BF16;
  auto kernel = has_f16 ? decode_chain_kernel<QI4_DTYPE_F16> : decode_chain_kernel<QI4_DTYPE_BF16>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)c->smem) !=
      cudaSuccess) {
    cudaGetLastError();
    set_error("cannot reserve %zu bytes of shared memory for the decode chain", c->smem);
    free_chain(c);
    return QI4_ERR_LAUNCH;
  }
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, kThreads, c->smem) != cudaSuccess ||
      blocks < 1) {
    cudaGetLastError();
    set_error("the decode chain kernel cannot be resident (one CTA per SM needed)");
    free_chain(c);
    return QI4_ERR_LAUNCH;
  }
  *out = reinterpret_cast<qi4_chain*>(c);
  return QI4_OK;
}

QI4_API int qi4_chain_run(qi4_chain* chain, void* stream_ptr) {
  using namespace qi4;
  clear_error();
  Chain* c = reinterpret_cast<Chain*>(chain);
  if (!c) {
    set_error("chain is null");
    return QI4_ERR_ARGUMENT;
  }
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != c->device) {
    cudaGetLastError();
    set_error("the chain was created on device %d; current device is %d", c->device, dev);
    return QI4_ERR_DEVICE;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)c->grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = c->smem;
  cfg.stream = static_cast<cudaStream_t>(stream_ptr);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = c->mma_type == QI4_DTYPE_F16 ? cudaLaunchKernelEx(&cfg, decode_chain_kernel<QI4_DTYPE_F16>, c->params)
                                                     : cudaLaunchKernelEx(&cfg, decode_chain_kernel<QI4_DTYPE_BF16>, c->params);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error("decode chain launch failed: %s", cudaGetErrorString(e));
    return QI4_ERR_LAUNCH;
  }
  return QI4_OK;
}

QI4_API int qi4_chain_info(const qi4_chain* chain, int64_t* info) {
  using namespace qi4;
  const Chain* c = reinterpret_cast<const Chain*>(chain);
  if (!c || !info) {
    set_error("chain and info must be non-null");
    return QI4_ERR_ARGUMENT;
  }
  info[0] = c->grid;
  info[1] = c->params.nslot;
  info[2] = (int64_t)c->smem;
  info[3] = c->weight_bytes;
  info[4] = c->alg_bytes;
  info[5] = c->nstages;
  return QI4_OK;
}

QI4_API int qi4_chain_destroy(qi4_chain* chain) {
  using namespace qi4;
  Chain* c = reinterpret_cast<Chain*>(chain);
  if (!c) return QI4_OK;
  const int owner = c->device;
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != owner) cudaSetDevice(owner);
  free_chain(c);
  if (cur >= 0 && cur != owner) cudaSetDevice(cur);
  return QI4_OK;
}

}  // extern "C"

namespace qi4 {

int read_chain_error(cudaStream_t stream) {
  int v = 0;
  if (cudaMemcpyFromSymbolAsync(&v, g_chain_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return -1;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return -1;
  if (v) {
    const int zero = 0;
    cudaMemcpyToSymbolAsync(g_chain_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    cudaStreamSynchronize(stream);
  }
  return v;
}

}  // namespace qi4
