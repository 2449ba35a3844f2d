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

bool tensor_map_2d(CUtensorMap* out, const void* base, CUtensorMapDataType dtype, uint64_t inner, uint64_t rows,
                   uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  static std::mutex mu;
  static std::unordered_map<Key, Entry*, KeyHash> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  Key key;
  memset(&key, 0, sizeof(key));
  key.device = dev;
  key.base = reinterpret_cast<uintptr_t>(base);
  key.inner = inner;
  key.rows = rows;
  key.stride = row_stride_bytes;
  key.box_inner = box_inner;
  key.box_rows = box_rows;
  key.dtype = (int)dtype;
  key.swizzle = (int)swizzle;
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
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {row_stride_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(&e->map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    delete e;
    set_error("cuTensorMapEncodeTiled failed (%d) for %llu x %llu, box %u x %u", (int)r,
              (unsigned long long)rows, (unsigned long long)inner, box_rows, box_inner);
    return false;
  }
  cache.emplace(key, e);
  *out = e->map;
  return true;
}

}  // namespace qi4
