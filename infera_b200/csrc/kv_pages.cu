// KV page gather / scatter between the paged cache and a contiguous chunk.
//
// Chunk layout (KV chunk blob v2 payload): [C, L, T, H] with C = 2 (K, V),
// or C = 1 for a latent (MLA) cache, whose one row per token holds the
// compressed KV and the rope key; L layers, T = n_pages * 16 tokens, H = kv
// elements per token.
// Cache layout: per channel [L, num_slots, H] (slot = page * 16 + offset), so
// one page of one layer is 16 * H contiguous elements: each CTA moves one
// (page, layer, channel) block with 16-byte vector accesses.
//
//   dir 0 (gather / save):  chunk[c, l, p*16 + i, :] = cache_c[l, pages[p]*16 + i, :]
//   dir 1 (scatter / load): cache_c[l, pages[p]*16 + i, :] = chunk[c, l, p*16 + i, :]
//   dir 2 / 3: the same with a page-major chunk [n_pages, C, L, 16, H], i.e.
//   one v2 payload per page back to back (the tier staging rings: each slot
//   is one page's blob payload).
//
// Reference parity: the reference implements this transfer as a Triton
// kernel (infera/engine/vllm/triton_kv_gather.py:82-220, with a Python loop
// oracle at :546-627); this is the CUDA counterpart for this cache layout.
#include <cuda_runtime.h>
#include <stdint.h>

namespace ib200 {
namespace kvp {

__global__ void page_copy_kernel(uint4* __restrict__ k_cache, uint4* __restrict__ v_cache, uint4* __restrict__ chunk,
                                 const int* __restrict__ pages, int n_pages, int L, long long slots_per_layer,
                                 int vec_per_token, int dir) {
  const int p = blockIdx.x, l = blockIdx.y, c = blockIdx.z;
  uint4* cache = c == 0 ? k_cache : v_cache;
  const long long page = pages[p];
  const long long tokens = static_cast<long long>(n_pages) * 16;
  const long long n = 16ll * vec_per_token;
  uint4* cbase = cache + (static_cast<long long>(l) * slots_per_layer + page * 16) * vec_per_token;
  const int C = gridDim.z;
  uint4* xbase = (dir & 2) ? chunk + (((static_cast<long long>(p) * C + c) * L + l) * 16) * vec_per_token
                           : chunk + ((static_cast<long long>(c) * L + l) * tokens + static_cast<long long>(p) * 16) *
                                         vec_per_token;
  if ((dir & 1) == 0) {
    for (long long i = threadIdx.x; i < n; i += blockDim.x) xbase[i] = cbase[i];
  } else {
    for (long long i = threadIdx.x; i < n; i += blockDim.x) cbase[i] = xbase[i];
  }
}

}  // namespace kvp
}  // namespace ib200

// k_cache / v_cache: [L, slots, H] of elem_bytes elements (v_cache unused when
// channels == 1); chunk: [channels, L, n_pages*16, H] (dir 0 / 1) or
// [n_pages, channels, L, 16, H] (dir 2 / 3).
// H * elem_bytes must be a multiple of 16.
extern "C" int ib_kv_page_copy(void* k_cache, void* v_cache, void* chunk, const int* pages, int n_pages, int L,
                               long long slots_per_layer, int H, int elem_bytes, int channels, int dir,
                               cudaStream_t stream) {
  if (n_pages <= 0) return 0;
  if ((H * elem_bytes) % 16 != 0 || dir < 0 || dir > 3 || (channels != 1 && channels != 2)) return -1;
  dim3 grid(n_pages, L, channels);
  ib200::kvp::page_copy_kernel<<<grid, 256, 0, stream>>>(
      static_cast<uint4*>(k_cache), static_cast<uint4*>(v_cache), static_cast<uint4*>(chunk), pages, n_pages, L,
      slots_per_layer, H * elem_bytes / 16, dir);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

// ---------------------------------------------------------------------------
// Prefill -> decode KV push (PD disaggregation over NVLink).
//
// Copies whole pages of layers [l0, l1) from this instance's caches into
// another instance's caches (dst_* are CUDA-IPC mappings of the decode
// instance's [L, slots, H] tensors on a peer GPU, or local pointers when both
// instances share a GPU): dst_c[l, dst_pages[p]*16 + i, :] =
// src_c[l, src_pages[p]*16 + i, :]. One CTA per (page, layer, channel);
// 16-byte loads from local HBM, 16-byte stores over NVLink (plain peer
// stores, no multicast). Called per layer as the prefill finishes it, or once
// for the whole range; channels = 1 pushes a latent cache (src_k / dst_k only).
namespace ib200 {
namespace kvp {

__global__ void __launch_bounds__(256) kv_push_kernel(const uint4* __restrict__ src_k, const uint4* __restrict__ src_v,
                                                      uint4* __restrict__ dst_k, uint4* __restrict__ dst_v,
                                                      const int* __restrict__ src_pages,
                                                      const int* __restrict__ dst_pages, int l0,
                                                      long long src_slots, long long dst_slots, int vec_per_token) {
  const int p = blockIdx.x, l = l0 + blockIdx.y, c = blockIdx.z;
  const uint4* src = c == 0 ? src_k : src_v;
  uint4* dst = c == 0 ? dst_k : dst_v;
  const long long n = 16ll * vec_per_token;
  const uint4* s = src + (static_cast<long long>(l) * src_slots + static_cast<long long>(src_pages[p]) * 16) *
                             vec_per_token;
  uint4* d = dst + (static_cast<long long>(l) * dst_slots + static_cast<long long>(dst_pages[p]) * 16) *
                       vec_per_token;
  // four independent 16-byte transfers in flight per thread
  long long i = threadIdx.x;
  for (; i + 3 * blockDim.x < n; i += 4 * blockDim.x) {
    const uint4 a = __ldg(s + i), b = __ldg(s + i + blockDim.x), e = __ldg(s + i + 2 * blockDim.x),
                f = __ldg(s + i + 3 * blockDim.x);
    d[i] = a;
    d[i + blockDim.x] = b;
    d[i + 2 * blockDim.x] = e;
    d[i + 3 * blockDim.x] = f;
  }
  for (; i < n; i += blockDim.x) d[i] = __ldg(s + i);
}

}  // namespace kvp
}  // namespace ib200

// src_*: this instance's caches [L, src_slots, H]; dst_*: the receiver's
// caches [L, dst_slots, H] (peer or local pointers); pages: int32 device
// arrays of n_pages each. Layers [l0, l1). H * elem_bytes % 16 == 0.
extern "C" int ib_kv_push_pages(const void* src_k, const void* src_v, void* dst_k, void* dst_v, const int* src_pages,
                                const int* dst_pages, int n_pages, int l0, int l1, long long src_slots,
                                long long dst_slots, int H, int elem_bytes, int channels, cudaStream_t stream) {
  if (n_pages <= 0 || l1 <= l0) return 0;
  if ((H * elem_bytes) % 16 != 0 || (channels != 1 && channels != 2)) return -1;
  dim3 grid(n_pages, l1 - l0, channels);
  ib200::kvp::kv_push_kernel<<<grid, 256, 0, stream>>>(
      static_cast<const uint4*>(src_k), static_cast<const uint4*>(src_v), static_cast<uint4*>(dst_k),
      static_cast<uint4*>(dst_v), src_pages, dst_pages, l0, src_slots, dst_slots, H * elem_bytes / 16);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}
