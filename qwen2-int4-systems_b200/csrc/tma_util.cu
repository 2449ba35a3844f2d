// Host side of tma_util.cuh: tensor-map encoding through the driver entry
// point (no link-time dependency on libcuda) and a small per-process cache.
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "qi4_common.cuh"
#include "tma_util.cuh"

namespace qi4 {

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct Key {
  int device;
  uintptr_t base;
  uint64_t inner, rows, stride;
  uint32_t box_inner, box_rows;
  int dtype, swizzle;
  uint64_t boxes;      // 3-D box-major maps: 128-byte boxes per row (0 for 2-D maps)
  uint32_t box_boxes;  // boxes per copy
  bool operator==(const Key& o) const { return memcmp(this, &o, sizeof(Key)) == 0; }
};

struct KeyHash {
  size_t operator()(const Key& k) const {
    const unsigned char* p = reinterpret_cast<const unsigned char*>(&k);
    size_t h = 1469598103934665603ull;
    for (size_t i = 0; i < sizeof(Key); ++i) h = (h ^ p[i]) * 1099511628211ull;
    return h;
  }
};

struct alignas(64) Entry {
  CUtensorMap map;
};

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
    cudaGetLastError();
  });
  return fn;
}

}  // namespace

namespace {

bool encode_cached(CUtensorMap* out, const Key& key, const void* base, CUtensorMapDataType dtype, int rank,
                   const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                   CUtensorMapSwizzle swizzle) {
  static std::mutex mu;
  static std::unordered_map<Key, Entry*, KeyHash> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second->map;
    return true;
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return false;
  }
  if (cache.size() > 4096) {  // bound the cache: drop everything (entries are cheap to rebuild)
    for (auto& kv : cache) delete kv.second;
    cache.clear();
  }
  Entry* e = new Entry;
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(&e->map, dtype, (cuuint32_t)rank, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    delete e;
    set_error("cuTensorMapEncodeTiled failed (%d) for a rank-%d map of %llu x %llu, box %u x %u", (int)r, rank,
              (unsigned long long)dims[1], (unsigned long long)dims[0], box[1], box[0]);
    return false;
  }
  cache.emplace(key, e);
  *out = e->map;
  return true;
}

Key make_key(const void* base, CUtensorMapDataType dtype, uint64_t inner, uint64_t rows, uint64_t stride,
             uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  int dev = 0;
  cudaGetDevice(&dev);
  Key key;
  memset(&key, 0, sizeof(key));
  key.device = dev;
  key.base = reinterpret_cast<uintptr_t>(base);
  key.inner = inner;
  key.rows = rows;
  key.stride = stride;
  key.box_inner = box_inner;
  key.box_rows = box_rows;
  key.dtype = (int)dtype;
  key.swizzle = (int)swizzle;
  return key;
}

}  // namespace

bool tensor_map_2d(CUtensorMap* out, const void* base, CUtensorMapDataType dtype, uint64_t inner, uint64_t rows,
                   uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  const Key key = make_key(base, dtype, inner, rows, row_stride_bytes, box_inner, box_rows, swizzle);
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  return encode_cached(out, key, base, dtype, 2, dims, strides, box, swizzle);
}

bool tensor_map_row_boxes(CUtensorMap* out, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_rows,
                          uint32_t boxes_per_copy) {
  Key key = make_key(base, CU_TENSOR_MAP_DATA_TYPE_UINT8, 128, rows, row_bytes, 128, box_rows,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  key.boxes = row_bytes / 128;
  key.box_boxes = boxes_per_copy;
  const cuuint64_t dims[3] = {128, rows, row_bytes / 128};
  const cuuint64_t strides[2] = {row_bytes, 128};
  const cuuint32_t box[3] = {128, box_rows, boxes_per_copy};
  return encode_cached(out, key, base, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace qi4
