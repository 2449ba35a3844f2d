// Shared device helpers for the W4G64 kernels (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qi4_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "qi4_b200 kernels target sm_100a only"
#endif

namespace qi4 {

constexpr int kGroup = 64;     // K elements per scale / zero point
constexpr int kChunkCodes = 32;  // codes in one 16-byte load
constexpr int kChunkBytes = 16;

// ---------------------------------------------------------------------------
// Host-side error reporting (thread-local message, see qi4_last_error).
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);

// Stream-ordered scratch from a per-device pool of the library that keeps
// freed memory for reuse (release threshold at its maximum): repeated calls
// do not map fresh device memory each time the device synchronises, as the
// default pool does. Free with scratch_free on the same stream.
cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t stream);
void scratch_free(void* p, cudaStream_t stream);
void clear_error();
int launch_status(const char* what);  // checks cudaGetLastError after a launch

// ---------------------------------------------------------------------------
// Loads
// ---------------------------------------------------------------------------

// 16-byte streaming load of packed weights: read-only path, no L1 allocation,
// with a 256-byte L2 prefetch hint (weights are touched exactly once).
__device__ __forceinline__ uint4 ldg_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float ldg_scale(const __half* p) {
  return __half2float(__ldg(p));
}

// Signed INT4 zero point of (row, group) in the packed zero-point stream.
__device__ __forceinline__ int load_zero(const uint8_t* zeros, int64_t index) {
  if (zeros == nullptr) return 0;
  const int byte = __ldg(zeros + (index >> 1));
  const int nib = (byte >> ((index & 1) * 4)) & 0xF;
  return (nib ^ 8) - 8;
}

// Scalar load of one element of a F16/BF16/F32 array as float.
__device__ __forceinline__ float load_as_f32(const void* base, int dtype, int64_t i) {
  if (dtype == QI4_DTYPE_F32) return __ldg(static_cast<const float*>(base) + i);
  const unsigned short raw = __ldg(static_cast<const unsigned short*>(base) + i);
  if (dtype == QI4_DTYPE_BF16) return __uint_as_float(static_cast<uint32_t>(raw) << 16);
  return __half2float(__ushort_as_half(raw));
}

// Four consecutive elements (16-byte aligned for F32, 8-byte for 16-bit types).
__device__ __forceinline__ float4 load4_as_f32(const void* base, int dtype, int64_t i) {
  if (dtype == QI4_DTYPE_F32) return __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(base) + i));
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(static_cast<const unsigned short*>(base) + i));
  float4 r;
  if (dtype == QI4_DTYPE_BF16) {
    r.x = __uint_as_float(raw.x << 16);
    r.y = __uint_as_float(raw.x & 0xFFFF0000u);
    r.z = __uint_as_float(raw.y << 16);
    r.w = __uint_as_float(raw.y & 0xFFFF0000u);
  } else {
    const __half2 a = *reinterpret_cast<const __half2*>(&raw.x);
    const __half2 b = *reinterpret_cast<const __half2*>(&raw.y);
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    r = make_float4(fa.x, fa.y, fb.x, fb.y);
  }
  return r;
}

// Store float as the output dtype (round to nearest even, as torch's .to()).
__device__ __forceinline__ void store_from_f32(void* base, int dtype, int64_t i, float v) {
  if (dtype == QI4_DTYPE_F32) {
    static_cast<float*>(base)[i] = v;
  } else if (dtype == QI4_DTYPE_BF16) {
    static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
  } else {
    static_cast<__half*>(base)[i] = __float2half_rn(v);
  }
}

// ---------------------------------------------------------------------------
// Nibble expansion
// ---------------------------------------------------------------------------
// For a 32-bit word holding 8 codes (element 2q in the low nibble of byte q,
// element 2q+1 in its high nibble), build two words whose byte q is
// 0x80 | ((code + 8) << 3), for the low and the high nibbles respectively.
// Placing such a byte at bits 16..23 under an 0x3F top byte gives the FP32
// number 1 + (code + 8) / 16, i.e. code = 16 * f - 24, exactly.
__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  // (a & b) ^ c : truth table 0xF0 & 0xCC ^ 0xAA = 0x6A
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ void expand_nibbles(uint32_t word, uint32_t& lo, uint32_t& hi) {
  lo = lop3_and_xor(word << 3, 0x78787878u, 0xC0C0C0C0u);
  hi = lop3_and_xor(word >> 1, 0x78787878u, 0xC0C0C0C0u);
}

// Byte q of `t` -> float 1 + (code + 8) / 16.
template <int Q>
__device__ __forceinline__ float nibble_float(uint32_t t) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(t), "r"(0x3F000000u), "n"(0x7044 | (Q << 8)));
  return __uint_as_float(d);
}

// Programmatic dependent launch controls (no-ops without the launch attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;");
}

}  // namespace qi4
