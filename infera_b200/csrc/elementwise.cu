// Memory-bound fused kernels of the decoder layer:
//   * RMSNorm and fused residual-add + RMSNorm (one CTA per token)
//   * RoPE on q/k (rotate-half convention) fused with the write of k and v
//     into their paged-cache slots
//   * embedding gather
//   * greedy / temperature sampling (Gumbel-max over a counter-based hash)
//
// All vectorised to 16-byte accesses; each reads its inputs and writes its
// outputs exactly once.
//
// Reference parity: these ops run inside the reference's engines (vLLM /
// SGLang); none has a source file in the reference tree.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "sm100.cuh"

namespace ib200 {
namespace ew {

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = lane < nw ? red[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  __syncthreads();
  return t;
}

// out = rmsnorm(x) * w ; optionally residual += delta first (x = residual).
// H must be a multiple of 8. Each thread owns up to 4 chunks of 8 elements.
template <bool ADD>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16* __restrict__ delta,
                                                      __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                                      __nv_bfloat16* __restrict__ out, int H, int ldx, int ldd,
                                                      int ldo, float eps) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  const int t = blockIdx.x;
  __nv_bfloat16* xr = x + static_cast<size_t>(t) * ldx;
  const int nchunk = H / 8;
  constexpr int MAXC = 4;
  float vals[MAXC][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nchunk) {
      uint4 a = reinterpret_cast<const uint4*>(xr)[c];
      float f[8] = {bf16_lo(a.x), bf16_hi(a.x), bf16_lo(a.y), bf16_hi(a.y),
                    bf16_lo(a.z), bf16_hi(a.z), bf16_lo(a.w), bf16_hi(a.w)};
      if (ADD) {
        uint4 d = reinterpret_cast<const uint4*>(delta + static_cast<size_t>(t) * ldd)[c];
        float g[8] = {bf16_lo(d.x), bf16_hi(d.x), bf16_lo(d.y), bf16_hi(d.y),
                      bf16_lo(d.z), bf16_hi(d.z), bf16_lo(d.w), bf16_hi(d.w)};
        uint4 s;
        s.x = pack_bf16(f[0] + g[0], f[1] + g[1]);
        s.y = pack_bf16(f[2] + g[2], f[3] + g[3]);
        s.z = pack_bf16(f[4] + g[4], f[5] + g[5]);
        s.w = pack_bf16(f[6] + g[6], f[7] + g[7]);
        reinterpret_cast<uint4*>(xr)[c] = s;
        // normalise the rounded residual so the stream stays self-consistent
        f[0] = bf16_lo(s.x); f[1] = bf16_hi(s.x); f[2] = bf16_lo(s.y); f[3] = bf16_hi(s.y);
        f[4] = bf16_lo(s.z); f[5] = bf16_hi(s.z); f[6] = bf16_lo(s.w); f[7] = bf16_hi(s.w);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        vals[i][j] = f[j];
        ss += f[j] * f[j];
      }
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / H + eps);
  __nv_bfloat16* orow = out + static_cast<size_t>(t) * ldo;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nchunk) {
      uint4 wv = reinterpret_cast<const uint4*>(w)[c];
      uint4 o;
      o.x = pack_bf16(vals[i][0] * inv * bf16_lo(wv.x), vals[i][1] * inv * bf16_hi(wv.x));
      o.y = pack_bf16(vals[i][2] * inv * bf16_lo(wv.y), vals[i][3] * inv * bf16_hi(wv.y));
      o.z = pack_bf16(vals[i][4] * inv * bf16_lo(wv.z), vals[i][5] * inv * bf16_hi(wv.z));
      o.w = pack_bf16(vals[i][6] * inv * bf16_lo(wv.w), vals[i][7] * inv * bf16_hi(wv.w));
      reinterpret_cast<uint4*>(orow)[c] = o;
    }
  }
}

// residual += delta; out = rmsnorm(residual) * w, with delta read from a
// split GEMM's fp32 workspace row [t, 0:H) (stride ldws) instead of a
// finalized bf16 output; the workspace row is zeroed for the next GEMM.
__global__ void __launch_bounds__(256) add_rmsnorm_ws_kernel(float* __restrict__ ws, int ldws,
                                                             __nv_bfloat16* __restrict__ x,
                                                             const __nv_bfloat16* __restrict__ w,
                                                             __nv_bfloat16* __restrict__ out, int H, int ldx, int ldo,
                                                             float eps) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  const int t = blockIdx.x;
  __nv_bfloat16* xr = x + static_cast<size_t>(t) * ldx;
  float* wr = ws + static_cast<size_t>(t) * ldws;
  const int nchunk = H / 8;
  constexpr int MAXC = 4;
  float vals[MAXC][8];
  float ss = 0.f;
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nchunk) {
      uint4 a = reinterpret_cast<const uint4*>(xr)[c];
      float4* d4 = reinterpret_cast<float4*>(wr + c * 8);
      const float4 d0 = __ldcg(d4), d1 = __ldcg(d4 + 1);
      __stcg(d4, zero);
      __stcg(d4 + 1, zero);
      // the delta rounded to bf16 first, as a finalized GEMM output would be
      auto rb = [](float v) { return __bfloat162float(__float2bfloat16(v)); };
      uint4 r;
      r.x = pack_bf16(bf16_lo(a.x) + rb(d0.x), bf16_hi(a.x) + rb(d0.y));
      r.y = pack_bf16(bf16_lo(a.y) + rb(d0.z), bf16_hi(a.y) + rb(d0.w));
      r.z = pack_bf16(bf16_lo(a.z) + rb(d1.x), bf16_hi(a.z) + rb(d1.y));
      r.w = pack_bf16(bf16_lo(a.w) + rb(d1.z), bf16_hi(a.w) + rb(d1.w));
      reinterpret_cast<uint4*>(xr)[c] = r;
      const float f[8] = {bf16_lo(r.x), bf16_hi(r.x), bf16_lo(r.y), bf16_hi(r.y),
                          bf16_lo(r.z), bf16_hi(r.z), bf16_lo(r.w), bf16_hi(r.w)};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        vals[i][j] = f[j];
        ss += f[j] * f[j];
      }
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(ss / H + eps);
  __nv_bfloat16* orow = out + static_cast<size_t>(t) * ldo;
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = threadIdx.x + i * blockDim.x;
    if (c < nchunk) {
      uint4 wv = reinterpret_cast<const uint4*>(w)[c];
      uint4 o;
      o.x = pack_bf16(vals[i][0] * inv * bf16_lo(wv.x), vals[i][1] * inv * bf16_hi(wv.x));
      o.y = pack_bf16(vals[i][2] * inv * bf16_lo(wv.y), vals[i][3] * inv * bf16_hi(wv.y));
      o.z = pack_bf16(vals[i][4] * inv * bf16_lo(wv.z), vals[i][5] * inv * bf16_hi(wv.z));
      o.w = pack_bf16(vals[i][6] * inv * bf16_lo(wv.w), vals[i][7] * inv * bf16_hi(wv.w));
      reinterpret_cast<uint4*>(orow)[c] = o;
    }
  }
}

// rope_kvwrite over a split GEMM's fp32 workspace row [t, 0:(hq+2hkv)*D)
// (stride ldws) instead of a finalized bf16 qkv row: the rotated q heads go
// to qkv (what attention reads), rotated k and v to the cache slot; the
// workspace row is zeroed (also when the token's indices are rejected).
__global__ void rope_kvwrite_ws_kernel(float* __restrict__ ws, int ldws, __nv_bfloat16* __restrict__ qkv,
                                       int ldqkv, const int* __restrict__ pos, const int* __restrict__ slots,
                                       const float2* __restrict__ cos_sin, int hq, int hkv, int D,
                                       __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc, int ldkv,
                                       long long num_slots, int max_pos, int* status) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int p = pos[t];
  long long slot = slots[t];
  float* wr = ws + static_cast<size_t>(t) * ldws;
  const int width = (hq + 2 * hkv) * D;
  const bool bad = p < 0 || p >= max_pos || slot >= num_slots;
  if (bad) {
    if (threadIdx.x == 0)
      record_status_detail(status, kStatusBadIndex, p < 0 || p >= max_pos ? 1 : 2, t,
                           p < 0 || p >= max_pos ? p : static_cast<int>(slot));
    for (int c = threadIdx.x; c < width; c += blockDim.x) wr[c] = 0.f;
    return;
  }
  __nv_bfloat16* row = qkv + static_cast<size_t>(t) * ldqkv;
  const int half = D / 2;
  const float2* cs = cos_sin + static_cast<size_t>(p) * half;
  const int pairs_per_head = half / 2;
  const int nheads = hq + hkv;
  for (int idx = threadIdx.x; idx < nheads * pairs_per_head; idx += blockDim.x) {
    const int hh = idx / pairs_per_head;
    const int i = (idx % pairs_per_head) * 2;
    float* hp = wr + hh * D;
    const float2 a = __ldcg(reinterpret_cast<const float2*>(hp + i));
    const float2 b = __ldcg(reinterpret_cast<const float2*>(hp + i + half));
    __stcg(reinterpret_cast<float2*>(hp + i), make_float2(0.f, 0.f));
    __stcg(reinterpret_cast<float2*>(hp + i + half), make_float2(0.f, 0.f));
    // round the projections to bf16 first, as the finalized path does
    const float a0 = __bfloat162float(__float2bfloat16(a.x)), a1 = __bfloat162float(__float2bfloat16(a.y));
    const float b0 = __bfloat162float(__float2bfloat16(b.x)), b1 = __bfloat162float(__float2bfloat16(b.y));
    const float2 c0 = cs[i], c1 = cs[i + 1];
    const __nv_bfloat162 na = __floats2bfloat162_rn(a0 * c0.x - b0 * c0.y, a1 * c1.x - b1 * c1.y);
    const __nv_bfloat162 nb = __floats2bfloat162_rn(b0 * c0.x + a0 * c0.y, b1 * c1.x + a1 * c1.y);
    if (hh < hq) {
      *reinterpret_cast<__nv_bfloat162*>(row + hh * D + i) = na;
      *reinterpret_cast<__nv_bfloat162*>(row + hh * D + i + half) = nb;
    } else if (slot >= 0) {
      __nv_bfloat16* kd = kc + slot * ldkv + (hh - hq) * D;
      *reinterpret_cast<__nv_bfloat162*>(kd + i) = na;
      *reinterpret_cast<__nv_bfloat162*>(kd + i + half) = nb;
    }
  }
  const int v0 = nheads * D;
  for (int c = threadIdx.x * 2; c < hkv * D; c += blockDim.x * 2) {
    float2* src = reinterpret_cast<float2*>(wr + v0 + c);
    const float2 v = __ldcg(src);
    __stcg(src, make_float2(0.f, 0.f));
    if (slot >= 0) *reinterpret_cast<__nv_bfloat162*>(vc + slot * ldkv + c) = __floats2bfloat162_rn(v.x, v.y);
  }
}

// qkv: [T, ldqkv] with q heads at [0, hq*D), k at [hq*D, (hq+hkv)*D), v after.
// Rotate q and k in place (rotate-half pairs (i, i + D/2)), then copy k, v
// into the cache slot of each token (slot < 0: skip the cache write).
// cos_sin: [max_pos, D/2, 2] fp32.
// Out-of-range positions or slots (bad host metadata) are recorded in the
// status word and skipped instead of touching memory outside the tables.
__global__ void rope_kvwrite_kernel(__nv_bfloat16* __restrict__ qkv, int ldqkv, const int* __restrict__ pos,
                                    const int* __restrict__ slots, const float2* __restrict__ cos_sin, int hq,
                                    int hkv, int D, __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc,
                                    int ldkv, long long num_slots, int max_pos, int* status) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int p = pos[t];
  long long slot = slots[t];
  if (p < 0 || p >= max_pos || slot >= num_slots) {
    if (threadIdx.x == 0)
      record_status_detail(status, kStatusBadIndex, p < 0 || p >= max_pos ? 1 : 2, t,
                           p < 0 || p >= max_pos ? p : static_cast<int>(slot));
    return;
  }
  __nv_bfloat16* row = qkv + static_cast<size_t>(t) * ldqkv;
  const int half = D / 2;
  const float2* cs = cos_sin + static_cast<size_t>(p) * half;
  // pairs of 2 adjacent i per thread: (i, i+1) with partners (i+half, i+1+half)
  const int pairs_per_head = half / 2;
  const int nheads = hq + hkv;
  for (int idx = threadIdx.x; idx < nheads * pairs_per_head; idx += blockDim.x) {
    const int hh = idx / pairs_per_head;
    const int i = (idx % pairs_per_head) * 2;
    __nv_bfloat16* hp = row + hh * D;
    __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(hp + i);
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(hp + i + half);
    const float2 c0 = cs[i], c1 = cs[i + 1];
    float a0 = __low2float(a), a1 = __high2float(a), b0 = __low2float(b), b1 = __high2float(b);
    float ra0 = a0 * c0.x - b0 * c0.y, rb0 = b0 * c0.x + a0 * c0.y;
    float ra1 = a1 * c1.x - b1 * c1.y, rb1 = b1 * c1.x + a1 * c1.y;
    __nv_bfloat162 na = __floats2bfloat162_rn(ra0, ra1), nb = __floats2bfloat162_rn(rb0, rb1);
    *reinterpret_cast<__nv_bfloat162*>(hp + i) = na;
    *reinterpret_cast<__nv_bfloat162*>(hp + i + half) = nb;
    if (hh >= hq && slot >= 0) {
      __nv_bfloat16* kd = kc + slot * ldkv + (hh - hq) * D;
      *reinterpret_cast<__nv_bfloat162*>(kd + i) = na;
      *reinterpret_cast<__nv_bfloat162*>(kd + i + half) = nb;
    }
  }
  if (slot >= 0) {
    const uint4* vs = reinterpret_cast<const uint4*>(row + (hq + hkv) * D);
    uint4* vd = reinterpret_cast<uint4*>(vc + slot * ldkv);
    for (int c = threadIdx.x; c < hkv * D / 8; c += blockDim.x) vd[c] = vs[c];
  }
}

// An id outside [0, vocab) is recorded in the status word and its row zeroed.
__global__ void embed_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                             __nv_bfloat16* __restrict__ out, int H, int vocab, int* status) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x;
  const int id = ids[t];
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H);
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) record_status_detail(status, kStatusBadIndex, 3, t, id);
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<size_t>(id) * H);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = src[c];
}

// splitmix64-style finaliser: a counter-based hash, not a cryptographic RNG.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// One CTA per row: argmax of logits / T + Gumbel noise (T == 0: argmax).
// Sampling from softmax(logits / T) by the Gumbel-max identity.
__global__ void __launch_bounds__(1024) sample_kernel(const __nv_bfloat16* __restrict__ logits, int ld, int V,
                                                      const float* __restrict__ temperature,
                                                      const long long* __restrict__ seeds, int* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  __shared__ float sv[32];
  __shared__ int si[32];
  const int b = blockIdx.x;
  const __nv_bfloat16* row = logits + static_cast<size_t>(b) * ld;
  const float T = temperature != nullptr ? temperature[b] : 0.f;
  const uint64_t seed = seeds != nullptr ? static_cast<uint64_t>(seeds[b]) : 0ull;
  float best = -INFINITY;
  int besti = 0;
  const float invT = T > 0.f ? 1.f / T : 0.f;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    float x = __bfloat162float(row[i]);
    if (T > 0.f) {
      uint64_t h = mix64(seed * 0x100000001B3ull ^ static_cast<uint64_t>(i));
      float u = (static_cast<float>(h >> 40) + 0.5f) * (1.0f / 16777216.0f);  // (0,1)
      x = x * invT - __logf(-__logf(u));
    }
    if (x > best) {
      best = x;
      besti = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, besti, o);
    if (ov > best || (ov == best && oi < besti)) {
      best = ov;
      besti = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = besti;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    besti = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, best, o);
      int oi = __shfl_xor_sync(0xffffffffu, besti, o);
      if (ov > best || (ov == best && oi < besti)) {
        best = ov;
        besti = oi;
      }
    }
    if (lane == 0) out[b] = besti;
  }
}

// Gather the rows `idx[i]` of src [*, ld] into dst [n, ld] (bf16, ld % 8 == 0).
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ src, const int* __restrict__ idx,
                                   __nv_bfloat16* __restrict__ dst, int ld) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x;
  const uint4* s = reinterpret_cast<const uint4*>(src + static_cast<size_t>(idx[i]) * ld);
  uint4* d = reinterpret_cast<uint4*>(dst + static_cast<size_t>(i) * ld);
  for (int c = threadIdx.x; c < ld / 8; c += blockDim.x) d[c] = s[c];
}

// dst[idx[i]] = val[i] for i < n (incremental block-table updates).
__global__ void scatter_i32_kernel(int* __restrict__ dst, const int* __restrict__ idx, const int* __restrict__ val,
                                   int n) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[idx[i]] = val[i];
}

}  // namespace ew
}  // namespace ib200

using namespace ib200;

static inline int ret_launch() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

extern "C" int ib_rmsnorm(const void* x, const void* w, void* out, int T, int H, int ldx, int ldo, float eps,
                          cudaStream_t stream) {
  if (T <= 0) return 0;
  if (H % 8 != 0 || H / 8 > 4 * 256) return -1;
  launch_pdl(ew::rmsnorm_kernel<false>, T, 256, 0, stream, nullptr, static_cast<__nv_bfloat16*>(const_cast<void*>(x)),
                                                    static_cast<const __nv_bfloat16*>(w),
                                                    static_cast<__nv_bfloat16*>(out), H, ldx, 0, ldo, eps);
  return ret_launch();
}

// residual += delta; out = rmsnorm(residual) * w
extern "C" int ib_add_rmsnorm(const void* delta, void* residual, const void* w, void* out, int T, int H, int ldd,
                              int ldr, int ldo, float eps, cudaStream_t stream) {
  if (T <= 0) return 0;
  if (H % 8 != 0 || H / 8 > 4 * 256) return -1;
  launch_pdl(ew::rmsnorm_kernel<true>, T, 256, 0, stream, static_cast<const __nv_bfloat16*>(delta),
                                                   static_cast<__nv_bfloat16*>(residual),
                                                   static_cast<const __nv_bfloat16*>(w),
                                                   static_cast<__nv_bfloat16*>(out), H, ldr, ldd, ldo, eps);
  return ret_launch();
}

// residual += ws[t, 0:H] (fp32 split-GEMM workspace, zeroed); out = rmsnorm(residual) * w
extern "C" int ib_add_rmsnorm_ws(void* ws, int ldws, void* residual, const void* w, void* out, int T, int H, int ldr,
                                 int ldo, float eps, cudaStream_t stream) {
  if (T <= 0) return 0;
  if (H % 8 != 0 || H / 8 > 4 * 256 || (ldws % 4) != 0) return -1;
  launch_pdl(ew::add_rmsnorm_ws_kernel, T, 256, 0, stream, static_cast<float*>(ws), ldws,
             static_cast<__nv_bfloat16*>(residual), static_cast<const __nv_bfloat16*>(w),
             static_cast<__nv_bfloat16*>(out), H, ldr, ldo, eps);
  return ret_launch();
}

// rope_kvwrite whose q / k / v come from the fp32 split-GEMM workspace
// [T, ldws] (zeroed); rotated q heads are written to qkv.
extern "C" int ib_rope_kvwrite_ws(void* ws, int ldws, void* qkv, int T, int ldqkv, const int* pos, const int* slots,
                                  const void* cos_sin, int hq, int hkv, int D, void* k_cache, void* v_cache,
                                  int ldkv, long long num_slots, int max_pos, int* status, cudaStream_t stream) {
  if (T <= 0) return 0;
  if (D % 4 != 0 || (ldws % 2) != 0) return -1;
  launch_pdl(ew::rope_kvwrite_ws_kernel, T, 256, 0, stream, static_cast<float*>(ws), ldws,
             static_cast<__nv_bfloat16*>(qkv), ldqkv, pos, slots, static_cast<const float2*>(cos_sin), hq, hkv, D,
             static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), ldkv, num_slots, max_pos,
             status);
  return ret_launch();
}

// num_slots: rows of each cache; max_pos: rows of the cos / sin table.
extern "C" int ib_rope_kvwrite(void* qkv, int T, int ldqkv, const int* pos, const int* slots, const void* cos_sin,
                               int hq, int hkv, int D, void* k_cache, void* v_cache, int ldkv, long long num_slots,
                               int max_pos, int* status, cudaStream_t stream) {
  if (T <= 0) return 0;
  if (D % 4 != 0) return -1;
  launch_pdl(ew::rope_kvwrite_kernel, T, 256, 0, stream, static_cast<__nv_bfloat16*>(qkv), ldqkv, pos, slots,
                                                  static_cast<const float2*>(cos_sin), hq, hkv, D,
                                                  static_cast<__nv_bfloat16*>(k_cache),
                                                  static_cast<__nv_bfloat16*>(v_cache), ldkv, num_slots, max_pos,
                                                  status);
  return ret_launch();
}

extern "C" int ib_embed(const int* ids, const void* table, void* out, int T, int H, int vocab, int* status,
                        cudaStream_t stream) {
  if (T <= 0) return 0;
  if (H % 8 != 0) return -1;
  launch_pdl(ew::embed_kernel, T, 256, 0, stream, ids, static_cast<const __nv_bfloat16*>(table),
                                           static_cast<__nv_bfloat16*>(out), H, vocab, status);
  return ret_launch();
}

extern "C" int ib_sample(const void* logits, int B, int ld, int V, const float* temperature, const long long* seeds,
                         int* out, cudaStream_t stream) {
  if (B <= 0) return 0;
  launch_pdl(ew::sample_kernel, B, 1024, 0, stream, static_cast<const __nv_bfloat16*>(logits), ld, V, temperature, seeds,
                                             out);
  return ret_launch();
}

extern "C" int ib_gather_rows(const void* src, const int* idx, void* dst, int n, int ld, cudaStream_t stream) {
  if (n <= 0) return 0;
  if (ld % 8 != 0) return -1;
  launch_pdl(ew::gather_rows_kernel, n, 128, 0, stream, static_cast<const __nv_bfloat16*>(src), idx,
                                                 static_cast<__nv_bfloat16*>(dst), ld);
  return ret_launch();
}

extern "C" int ib_scatter_i32(int* dst, const int* idx, const int* val, int n, cudaStream_t stream) {
  if (n <= 0) return 0;
  launch_pdl(ew::scatter_i32_kernel, (n + 255) / 256, 256, 0, stream, dst, idx, val, n);
  return ret_launch();
}
