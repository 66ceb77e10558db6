// Paged decode attention for grouped-query attention (one new token per
// sequence), split along the KV length so that small batches still fill the
// 148 SMs, followed by a log-sum-exp combine.
//
// Decode attention reads every cached K/V byte once per step and does ~4
// FLOP per byte, so it is bound by HBM bandwidth, not by the tensor cores:
// the kernel streams 64-token tiles (4 pages) into shared memory with 16-byte
// cp.async (double buffered), and computes scores and P.V on the FP32 pipes
// from an XOR-swizzled tile.
//
// Layout: KV cache per layer [num_slots, Hkv * 128] bf16, slot = page*16+off.
//
// Reference parity: the reference's decode attention lives inside its
// engines (vLLM / SGLang / AITER); not in its tree.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "sm100.cuh"

namespace ib200 {
namespace dec {

constexpr int D = 128;
constexpr int TILE = 64;   // tokens per tile (4 pages)
constexpr int PAGE = 16;
constexpr int DYN_SMEM = 4 * TILE * 16 * 16;  // K and V, double buffered
constexpr int THREADS = 128;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 16-byte chunk c of row r lives at chunk (c ^ (r & 15)) -> conflict-free
// row-parallel 16-byte reads.
__device__ __forceinline__ int swz(int r, int c) { return r * 16 + (c ^ (r & 15)); }

struct Params {
  const __nv_bfloat16* q;   // [B, Hq*D] (row stride ldq)
  int ldq;
  const __nv_bfloat16* k;   // [slots, Hkv*D]
  const __nv_bfloat16* v;
  const int* block_table;   // [rows, max_pages]
  const int* bt_rows;       // [B] table row of each sequence (null: row b)
  const int* seq_lens;      // [B]
  int max_pages;
  int hq, hkv, splits;
  float scale_log2;
  float* o_part;            // [B, Hq, splits, D]
  float* lse_part;          // [B, Hq, splits]
  __nv_bfloat16* out;       // [B, Hq*D] when splits == 1
  int ldo;
};

template <int G>
__global__ void __launch_bounds__(THREADS) decode_kernel(const Params p) {
  extern __shared__ __align__(16) uint4 dyn_smem[];
  uint4 (*sK)[TILE * 16] = reinterpret_cast<uint4 (*)[TILE * 16]>(dyn_smem);
  uint4 (*sV)[TILE * 16] = reinterpret_cast<uint4 (*)[TILE * 16]>(dyn_smem + 2 * TILE * 16);
  __shared__ float sQ[G][D];
  __shared__ float sS[G][TILE];

  const int b = blockIdx.x;
  const int kvh = blockIdx.y;
  const int split = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int len = p.seq_lens[b];
  const int n_tiles_total = (len + TILE - 1) / TILE;
  const int tiles_per_split = (n_tiles_total + p.splits - 1) / p.splits;
  const int t_begin = split * tiles_per_split;
  const int t_end = min(n_tiles_total, t_begin + tiles_per_split);
  const int bt_row = p.bt_rows != nullptr ? p.bt_rows[b] : b;
  const int* bt = p.block_table + static_cast<size_t>(bt_row) * p.max_pages;
  const int kvw = p.hkv * D;

  for (int i = tid; i < G * D; i += THREADS) {
    int g = i / D, d = i % D;
    sQ[g][d] = __bfloat162float(p.q[static_cast<size_t>(b) * p.ldq + (kvh * G + g) * D + d]) * p.scale_log2;
  }

  auto load_tile = [&](int t, int buf) {
    // 64 tokens x 16 chunks of 16 B for K and V: 1024 chunks each, 8 per thread
#pragma unroll
    for (int i = 0; i < (TILE * 16) / THREADS; ++i) {
      int idx = i * THREADS + tid;
      int r = idx >> 4, c = idx & 15;
      int tok = t * TILE + r;
      int tok_c = tok < len ? tok : len - 1;
      int page = __ldg(bt + tok_c / PAGE);
      size_t slot = static_cast<size_t>(page) * PAGE + (tok_c % PAGE);
      const __nv_bfloat16* kp = p.k + slot * kvw + kvh * D + c * 8;
      const __nv_bfloat16* vp = p.v + slot * kvw + kvh * D + c * 8;
      cp_async16(&sK[buf][swz(r, c)], kp);
      cp_async16(&sV[buf][swz(r, c)], vp);
    }
    cp_async_commit();
  };

  // per-warp head ownership for softmax / PV: warp w owns heads w, w+4, ...
  float m_run[(G + 3) / 4], l_run[(G + 3) / 4];
  float acc[(G + 3) / 4][4];
#pragma unroll
  for (int i = 0; i < (G + 3) / 4; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.f;
    acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  }

  if (t_begin < t_end) load_tile(t_begin, 0);
  __syncthreads();
  for (int t = t_begin; t < t_end; ++t) {
    const int buf = (t - t_begin) & 1;
    if (t + 1 < t_end) {
      load_tile(t + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    // scores: TILE tokens x G heads over THREADS threads
    for (int pair = tid; pair < TILE * G; pair += THREADS) {
      const int r = pair % TILE;
      const int g = pair / TILE;
      float s = 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint4 kv = sK[buf][swz(r, c)];
        const float* qq = &sQ[g][c * 8];
        s += qq[0] * bf16_lo(kv.x) + qq[1] * bf16_hi(kv.x) + qq[2] * bf16_lo(kv.y) + qq[3] * bf16_hi(kv.y) +
             qq[4] * bf16_lo(kv.z) + qq[5] * bf16_hi(kv.z) + qq[6] * bf16_lo(kv.w) + qq[7] * bf16_hi(kv.w);
      }
      const int tok = t * TILE + r;
      sS[g][r] = tok < len ? s : -INFINITY;
    }
    __syncthreads();
    // softmax + PV: warp handles heads g = warp + 4*i; lane owns dims 4*lane..4*lane+3
#pragma unroll
    for (int i = 0; i < (G + 3) / 4; ++i) {
      const int g = warp + 4 * i;
      if (g >= G) break;
      float s0 = sS[g][lane], s1 = sS[g][lane + 32];
      float mx = fmaxf(s0, s1);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_new = fmaxf(m_run[i], mx);
      const float alpha = exp2f(m_run[i] - m_new);
      float e0 = exp2f(s0 - m_new), e1 = exp2f(s1 - m_new);
      float sum = e0 + e1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      l_run[i] = l_run[i] * alpha + sum;
      m_run[i] = m_new;
      acc[i][0] *= alpha;
      acc[i][1] *= alpha;
      acc[i][2] *= alpha;
      acc[i][3] *= alpha;
      __syncwarp();
      sS[g][lane] = e0;
      sS[g][lane + 32] = e1;
      __syncwarp();
      const int c = lane >> 1;          // 16-byte chunk holding dims 4*lane..
      const int half = lane & 1;        // which 8-byte half of the chunk
#pragma unroll 8
      for (int r = 0; r < TILE; ++r) {
        const float pr = sS[g][r];
        const uint2 vv = reinterpret_cast<const uint2*>(&sV[buf][swz(r, c)])[half];
        acc[i][0] += pr * bf16_lo(vv.x);
        acc[i][1] += pr * bf16_hi(vv.x);
        acc[i][2] += pr * bf16_lo(vv.y);
        acc[i][3] += pr * bf16_hi(vv.y);
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < (G + 3) / 4; ++i) {
    const int g = warp + 4 * i;
    if (g >= G) break;
    const int h = kvh * G + g;
    if (p.splits == 1) {
      const float inv = l_run[i] > 0.f ? 1.f / l_run[i] : 0.f;
      __nv_bfloat16* o = p.out + static_cast<size_t>(b) * p.ldo + h * D + lane * 4;
      uint2 w;
      w.x = pack_bf16(acc[i][0] * inv, acc[i][1] * inv);
      w.y = pack_bf16(acc[i][2] * inv, acc[i][3] * inv);
      *reinterpret_cast<uint2*>(o) = w;
    } else {
      const size_t base = (static_cast<size_t>(b) * p.hq + h) * p.splits + split;
      const float inv = l_run[i] > 0.f ? 1.f / l_run[i] : 0.f;
      float4 v = make_float4(acc[i][0] * inv, acc[i][1] * inv, acc[i][2] * inv, acc[i][3] * inv);
      *reinterpret_cast<float4*>(p.o_part + base * D + lane * 4) = v;
      if (lane == 0)
        p.lse_part[base] = (l_run[i] > 0.f) ? (m_run[i] + log2f(l_run[i])) : -INFINITY;
    }
  }
}

// Combine split partials. Each split stored its output normalised by its own
// softmax sum (o_s) and lse_s = m_s + log2(l_s) in log2 units, so
//   o = sum_s 2^(lse_s - M) o_s / sum_s 2^(lse_s - M),  M = max_s lse_s.
__global__ void combine_kernel(const Params p) {
  const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;  // blockDim = D
  const size_t base = (static_cast<size_t>(b) * p.hq + h) * p.splits;
  float mx = -INFINITY;
  for (int s = 0; s < p.splits; ++s) mx = fmaxf(mx, p.lse_part[base + s]);
  float num = 0.f, den = 0.f;
  for (int s = 0; s < p.splits; ++s) {
    const float lse = p.lse_part[base + s];
    if (lse == -INFINITY) continue;
    const float w = exp2f(lse - mx);
    den += w;
    num += p.o_part[(base + s) * D + d] * w;
  }
  const float out = den > 0.f ? num / den : 0.f;
  p.out[static_cast<size_t>(b) * p.ldo + h * D + d] = __float2bfloat16(out);
}

}  // namespace dec
}  // namespace ib200

using namespace ib200;

template <int G>
static void launch_decode(const dec::Params& p, int B, cudaStream_t stream) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(dec::decode_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, dec::DYN_SMEM);
    attr_set[dev] = true;
  }
  dim3 grid(B, p.hkv, p.splits);
  dec::decode_kernel<G><<<grid, dec::THREADS, dec::DYN_SMEM, stream>>>(p);
}

// q [B, ldq] bf16 (head h at h*128); out [B, ldo] bf16.
// o_part: fp32 [B*Hq*splits*128], lse_part: fp32 [B*Hq*splits] (scratch,
// only used when splits > 1).
extern "C" int ib_attn_decode(const void* q, int ldq, const void* k_cache, const void* v_cache,
                              const int* block_table, const int* bt_rows, const int* seq_lens, int max_pages, int B,
                              int hq, int hkv,
                              int splits, float scale, float* o_part, float* lse_part, void* out, int ldo,
                              cudaStream_t stream) {
  if (B <= 0) return 0;
  if (hq % hkv != 0 || splits < 1) return -1;
  const int G = hq / hkv;
  dec::Params p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.ldq = ldq;
  p.k = static_cast<const __nv_bfloat16*>(k_cache);
  p.v = static_cast<const __nv_bfloat16*>(v_cache);
  p.block_table = block_table;
  p.bt_rows = bt_rows;
  p.seq_lens = seq_lens;
  p.max_pages = max_pages;
  p.hq = hq;
  p.hkv = hkv;
  p.splits = splits;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o_part = o_part;
  p.lse_part = lse_part;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  switch (G) {
    case 1: launch_decode<1>(p, B, stream); break;
    case 2: launch_decode<2>(p, B, stream); break;
    case 4: launch_decode<4>(p, B, stream); break;
    case 8: launch_decode<8>(p, B, stream); break;
    default: return -1;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return static_cast<int>(e);
  if (splits > 1) {
    dim3 grid(B, hq);
    dec::combine_kernel<<<grid, dec::D, 0, stream>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return 0;
}

// ---------------------------------------------------------------------------
// Allocation-free entry point (declared, with its contract, in
// attn_decode_noalloc.h). Same kernels as ib_attn_decode; the split-KV
// partials live in file-scope device arrays instead of caller memory.
#include <mutex>

#include "attn_decode_noalloc.h"

namespace ib200 {
namespace dec_noalloc {

// Split-KV partial outputs and their log-sum-exp. In host code these names
// are host-side stand-ins, not device addresses: never hand them to a
// kernel; use the addresses looked up by device_scratch().
static __device__ __align__(256) float g_o_part[IB_DECODE_NOALLOC_MAX_ROWS * dec::D];
static __device__ __align__(256) float g_lse_part[IB_DECODE_NOALLOC_MAX_ROWS];

struct DeviceScratch {
  float* o = nullptr;
  float* lse = nullptr;
  bool ready = false;
};
constexpr int kMaxDevices = 64;
static DeviceScratch g_scratch[kMaxDevices];
static std::mutex g_mu;

// Device addresses of the arrays for the current device, looked up once per
// device (with that device current) and cached.
static int device_scratch(DeviceScratch** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return IB_DECODE_NOALLOC_SETUP_FAILED;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceScratch& s = g_scratch[dev];
  if (!s.ready) {
    void* o = nullptr;
    void* lse = nullptr;
    if (cudaGetSymbolAddress(&o, g_o_part) != cudaSuccess) return IB_DECODE_NOALLOC_SETUP_FAILED;
    if (cudaGetSymbolAddress(&lse, g_lse_part) != cudaSuccess) return IB_DECODE_NOALLOC_SETUP_FAILED;
    s.o = static_cast<float*>(o);
    s.lse = static_cast<float*>(lse);
    s.ready = true;
  }
  *out = &s;
  return 0;
}

}  // namespace dec_noalloc
}  // namespace ib200

extern "C" int ib_attn_decode_noalloc_max_rows(void) { return IB_DECODE_NOALLOC_MAX_ROWS; }

extern "C" int ib_attn_decode_noalloc(const void* q, int ldq, const void* k_cache, const void* v_cache,
                                      const int* block_table, const int* bt_rows, const int* seq_lens, int max_pages,
                                      int B, int hq, int hkv, int splits, float scale, void* out, int ldo,
                                      cudaStream_t stream) {
  if (B <= 0) return 0;
  if (hkv <= 0 || hq % hkv != 0 || splits < 1) return -1;
  const int G = hq / hkv;
  if (G != 1 && G != 2 && G != 4 && G != 8) return -1;
  float* o_part = nullptr;
  float* lse_part = nullptr;
  if (splits > 1) {
    if (static_cast<long long>(B) * hq * splits > IB_DECODE_NOALLOC_MAX_ROWS) return IB_DECODE_NOALLOC_TOO_BIG;
    dec_noalloc::DeviceScratch* s = nullptr;
    const int rc = dec_noalloc::device_scratch(&s);
    if (rc != 0) return rc;
    o_part = s->o;
    lse_part = s->lse;
  }
  dec::Params p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.ldq = ldq;
  p.k = static_cast<const __nv_bfloat16*>(k_cache);
  p.v = static_cast<const __nv_bfloat16*>(v_cache);
  p.block_table = block_table;
  p.bt_rows = bt_rows;
  p.seq_lens = seq_lens;
  p.max_pages = max_pages;
  p.hq = hq;
  p.hkv = hkv;
  p.splits = splits;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o_part = o_part;
  p.lse_part = lse_part;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  switch (G) {
    case 1: launch_decode<1>(p, B, stream); break;
    case 2: launch_decode<2>(p, B, stream); break;
    case 4: launch_decode<4>(p, B, stream); break;
    default: launch_decode<8>(p, B, stream); break;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return static_cast<int>(e);
  if (splits > 1) {
    dim3 grid(B, hq);
    dec::combine_kernel<<<grid, dec::D, 0, stream>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return 0;
}
