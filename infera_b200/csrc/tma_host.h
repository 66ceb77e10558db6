// Host-side helpers: TMA tensor-map encoding through the driver entry point
// (no link against libcuda), device-property caching and a small
// tensor-map cache keyed by (address, shape, box).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>

namespace ib200 {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

inline int num_sms_for_current_device() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// 2-D row-major tensor [rows, cols] of `elem_bytes`-byte elements with a row
// pitch of `ld` elements; box = box_rows x box_cols with 128-byte swizzle
// (box_cols * elem_bytes must be 128). Returns false if encoding fails.
inline bool encode_2d_sw128(CUtensorMap* out, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                            uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows, uint32_t box_cols) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * static_cast<uint64_t>(elem_bytes)};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(out, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct TmapKey {
  uint64_t base, rows, cols, ld;
  uint32_t box_rows, box_cols, dtype, dev;
  bool operator==(const TmapKey& o) const { return std::memcmp(this, &o, sizeof(TmapKey)) == 0; }
};
struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    uint64_t h = 1469598103934665603ull;
    const unsigned char* p = reinterpret_cast<const unsigned char*>(&k);
    for (size_t i = 0; i < sizeof(TmapKey); ++i) h = (h ^ p[i]) * 1099511628211ull;
    return static_cast<size_t>(h);
  }
};

// Tensor maps are cheap to encode (~1 us) but the decode loop encodes the
// same handful hundreds of times a second; cache them.
inline bool cached_tmap_2d(CUtensorMap* out, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                           uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows, uint32_t box_cols) {
  static std::mutex mu;
  static std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  TmapKey key;
  std::memset(&key, 0, sizeof(key));
  key.base = reinterpret_cast<uint64_t>(base);
  key.rows = rows;
  key.cols = cols;
  key.ld = ld;
  key.box_rows = box_rows;
  key.box_cols = box_cols;
  key.dtype = static_cast<uint32_t>(dtype);
  key.dev = static_cast<uint32_t>(dev);
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return true;
  }
  if (!encode_2d_sw128(out, base, dtype, elem_bytes, rows, cols, ld, box_rows, box_cols)) return false;
  if (cache.size() > 8192) cache.clear();
  cache.emplace(key, *out);
  return true;
}

}  // namespace ib200
