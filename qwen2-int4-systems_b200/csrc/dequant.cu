// Standalone format primitives: canonical INT4 unpack and W4G64 -> FP32
// dequantisation (bit-exact with the reference).
//
//   unpack   : reference src/qwen_int4/quantization.py:53-84 (CANONICAL) and
//              src/qwen_int4/triton_kernels.py:23-35,119-146
//   dequant  : reference src/qwen_int4/quantization.py:221-258 and
//              src/qwen_int4/triton_kernels.py:39-63,149-203
//
// Both are HBM-bound byte streams. One thread handles one 16-byte chunk of
// packed input (32 codes; a chunk never straddles a 64-group or a row because
// K/2 is a multiple of 32), reads it with one 128-bit load and writes its
// outputs with 128-bit stores. The grid is a multiple of the SM count and
// strides over the chunks.
#include "dequant.cuh"
#include "qi4_common.cuh"

namespace qi4 {

namespace {

// Byte -> two sign-extended nibbles packed as int8 in a 16-bit lane.
__device__ __forceinline__ uint32_t expand_pair_i8(uint32_t b) {
  const uint32_t lo = ((b & 0xF) ^ 8) - 8;
  const uint32_t hi = (((b >> 4) & 0xF) ^ 8) - 8;
  return (lo & 0xFF) | ((hi & 0xFF) << 8);
}

// 4 packed bytes -> 8 int8 codes in element order (two output words).
__device__ __forceinline__ uint2 expand_word_i8(uint32_t w) {
  uint2 r;
  r.x = expand_pair_i8(w & 0xFF) | (expand_pair_i8((w >> 8) & 0xFF) << 16);
  r.y = expand_pair_i8((w >> 16) & 0xFF) | (expand_pair_i8(w >> 24) << 16);
  return r;
}

__global__ void __launch_bounds__(256) unpack_kernel(const uint8_t* __restrict__ packed, int8_t* __restrict__ out,
                                                     int64_t elements) {
  const int64_t full_chunks = elements / kChunkCodes;  // chunks whose 32 outputs all exist
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < full_chunks; c += stride) {
    const uint4 q = ldg_stream16(packed + c * kChunkBytes);
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
    uint32_t o[8];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const uint2 e = expand_word_i8(words[w]);
      o[2 * w] = e.x;
      o[2 * w + 1] = e.y;
    }
    uint4* dst = reinterpret_cast<uint4*>(out + c * kChunkCodes);
    dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
    dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
  // Ragged tail (fewer than 32 trailing elements, e.g. an odd zero-point count).
  const int64_t tail0 = full_chunks * kChunkCodes;
  if (blockIdx.x == 0) {
    for (int64_t i = tail0 + threadIdx.x; i < elements; i += blockDim.x) {
      const int b = packed[i >> 1];
      const int nib = (b >> ((i & 1) * 4)) & 0xF;
      out[i] = (int8_t)((nib ^ 8) - 8);
    }
  }
}

__global__ void __launch_bounds__(256) dequant_f32_kernel(const uint8_t* __restrict__ qweight,
                                                          const __half* __restrict__ scales,
                                                          const uint8_t* __restrict__ zeros,
                                                          float* __restrict__ out, int64_t N, int64_t K) {
  const int64_t chunks_per_row = K / kChunkCodes;
  const int64_t total = N * chunks_per_row;
  const int64_t G = K / kGroup;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < total; c += stride) {
    const int64_t row = c / chunks_per_row;
    const int64_t cr = c - row * chunks_per_row;
    const int64_t gi = row * G + (cr >> 1);
    const float s = ldg_scale(scales + gi);
    const int z = load_zero(zeros, gi);
    const uint4 q = ldg_stream16(qweight + c * kChunkBytes);
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
    float4* dst = reinterpret_cast<float4*>(out + c * kChunkCodes);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int nib = (words[w] >> (4 * j)) & 0xF;
        // (code - zero) is a small integer and s an fp16 value: the FP32
        // product is exact, exactly as in the reference's FP32 expression.
        v[j] = static_cast<float>(((nib ^ 8) - 8) - z) * s;
      }
      dst[2 * w] = make_float4(v[0], v[1], v[2], v[3]);
      dst[2 * w + 1] = make_float4(v[4], v[5], v[6], v[7]);
    }
  }
}

int grid_for(int64_t work, int num_sms) {
  const int64_t per_block = 256;
  int64_t blocks = (work + per_block - 1) / per_block;
  const int64_t cap = (int64_t)num_sms * 8;  // 8 resident CTAs of 256 threads per SM
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return (int)blocks;
}

}  // namespace

cudaError_t launch_unpack(const uint8_t* packed, int8_t* out, int64_t elements, cudaStream_t stream,
                          int num_sms) {
  const int64_t chunks = elements / kChunkCodes;
  unpack_kernel<<<grid_for(chunks > 0 ? chunks : 1, num_sms), 256, 0, stream>>>(packed, out, elements);
  return cudaGetLastError();
}

cudaError_t launch_dequant_f32(const uint8_t* qweight, const uint16_t* scales, const uint8_t* zeros, float* out,
                               int64_t N, int64_t K, cudaStream_t stream, int num_sms) {
  const int64_t chunks = N * (K / kChunkCodes);
  dequant_f32_kernel<<<grid_for(chunks, num_sms), 256, 0, stream>>>(
      qweight, reinterpret_cast<const __half*>(scales), zeros, out, N, K);
  return cudaGetLastError();
}

}  // namespace qi4
