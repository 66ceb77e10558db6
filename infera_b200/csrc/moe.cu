// Mixture-of-experts routing and data movement around the grouped GEMM
// (ib_gemm_grouped in gemm_bf16.cu):
//
//   ib_moe_topk     router scores -> top-k experts and weights per token.
//                   Grouped selection of DeepSeek-V3: score = sigmoid(logit)
//                   (or softmax), choice = score + bias; a group's rank is
//                   the sum of its two best choices; keep the best
//                   `topk_groups` groups, then the `top_k` best choices in
//                   them; weights = scores of the chosen experts,
//                   renormalised to sum 1 (optional), times `scaling`.
//                   One warp per token; n_groups = 1 gives plain top-k.
//   ib_moe_permute  counts tokens per expert, exclusive offsets, and the
//                   expert-sorted row of every (token, slot) pair, plus the
//                   sorted rows' token ids (for the activation gather).
//   ib_moe_tiles    the grouped GEMM's tile table from the offsets: for every
//                   expert, ceil(count / bn) token tiles x N/128 feature tiles.
//   ib_moe_combine  out[t] = sum_j weight[t, j] * rows[row_of(t, j)] (fp32).
//
// Semantics of the routing: the reference serves DeepSeek-V3 / Kimi through
// vLLM / SGLang's fused MoE (grouped top-k); this is this framework's own.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace ib200 {
namespace moe {

constexpr int kMaxExperts = 1024;
constexpr int kMaxTopK = 16;
constexpr int kMaxGroups = 32;

__device__ __forceinline__ float load_f(const void* p, int i, int is_bf16) {
  return is_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]) : static_cast<const float*>(p)[i];
}

// warp argmax over (value, index); ties to the lower index
__device__ __forceinline__ void warp_argmax(float& v, int& i) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (ov > v || (ov == v && oi < i)) {
      v = ov;
      i = oi;
    }
  }
}

// one warp per token; experts live in shared memory per warp
__global__ void __launch_bounds__(128) topk_kernel(const void* __restrict__ logits, int ld, int is_bf16,
                                                   const float* __restrict__ bias, int T, int E, int n_groups,
                                                   int topk_groups, int top_k, int use_softmax, int renorm,
                                                   float scaling, int* __restrict__ ids, float* __restrict__ wts) {
  extern __shared__ float sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + warp;
  float* score = sm + warp * 2 * E;   // scores (weights source)
  float* choice = score + E;          // selection keys
  if (t >= T) return;
  const long long row = static_cast<long long>(t) * ld;
  float mx = -INFINITY;
  for (int e = lane; e < E; e += 32) {
    const float x = load_f(logits, static_cast<int>(row + e), is_bf16);
    score[e] = x;
    mx = fmaxf(mx, x);
  }
  float denom = 0.f;
  if (use_softmax) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int e = lane; e < E; e += 32) denom += __expf(score[e] - mx);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) denom += __shfl_xor_sync(0xffffffffu, denom, o);
  }
  __syncwarp();
  for (int e = lane; e < E; e += 32) {
    const float s = use_softmax ? __expf(score[e] - mx) / denom : 1.f / (1.f + __expf(-score[e]));
    score[e] = s;
    choice[e] = s + (bias ? bias[e] : 0.f);
  }
  __syncwarp();
  // group ranks: lane g scores group g by its two best choices
  const int gsize = E / n_groups;
  float gscore = -INFINITY;
  if (lane < n_groups) {
    float b0 = -INFINITY, b1 = -INFINITY;
    for (int e = lane * gsize; e < (lane + 1) * gsize; ++e) {
      const float c = choice[e];
      if (c > b0) {
        b1 = b0;
        b0 = c;
      } else if (c > b1) {
        b1 = c;
      }
    }
    gscore = n_groups == 1 ? 0.f : b0 + (gsize > 1 ? b1 : 0.f);
  }
  unsigned keep = 0;  // bit g: group g selected
  for (int k = 0; k < topk_groups && k < n_groups; ++k) {
    float v = (lane < n_groups && !((keep >> lane) & 1u)) ? gscore : -INFINITY;
    int i = lane;
    warp_argmax(v, i);
    keep |= 1u << i;
  }
  // top-k experts within the kept groups
  float wsum = 0.f;
  float mine_w = 0.f;
  int mine_id = -1;
  for (int k = 0; k < top_k; ++k) {
    float v = -INFINITY;
    int i = E;
    for (int e = lane; e < E; e += 32) {
      if (!((keep >> (e / gsize)) & 1u)) continue;
      const float c = choice[e];
      if (c > v || (c == v && e < i)) {
        v = c;
        i = e;
      }
    }
    warp_argmax(v, i);
    if (i >= E) i = 0;  // fewer eligible experts than top_k (degenerate configs)
    const float w = score[i];
    if (lane == k) {
      mine_id = i;
      mine_w = w;
    }
    wsum += w;
    if (lane == 0) choice[i] = -INFINITY;
    __syncwarp();
  }
  if (lane < top_k) {
    const float w = renorm ? mine_w / fmaxf(wsum, 1e-20f) : mine_w;
    ids[t * top_k + lane] = mine_id;
    wts[t * top_k + lane] = w * scaling;
  }
}

__global__ void count_kernel(const int* __restrict__ ids, int n, int* __restrict__ counts) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) atomicAdd(counts + ids[i], 1);
}

// single block: exclusive scan of counts -> offsets[E+1]; resets the cursors
__global__ void scan_kernel(const int* __restrict__ counts, int E, int* __restrict__ offsets, int* __restrict__ cursor) {
  __shared__ int s[kMaxExperts];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s[e] = counts[e];
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = acc;
      acc += s[e];
    }
    offsets[E] = acc;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) cursor[e] = 0;
}

__global__ void scatter_kernel(const int* __restrict__ ids, int n, int top_k, const int* __restrict__ offsets,
                               int* __restrict__ cursor, int* __restrict__ row_of_slot, int* __restrict__ token_of_row) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int e = ids[i];
    const int r = offsets[e] + atomicAdd(cursor + e, 1);
    row_of_slot[i] = r;
    token_of_row[r] = i / top_k;
  }
}

// one block of E threads: tiles of expert e are written after the tiles of
// experts < e (exclusive scan of per-expert tile counts)
__global__ void tiles_kernel(const int* __restrict__ offsets, int E, int n_tiles, int bn, int4* __restrict__ tab,
                             int* __restrict__ num) {
  __shared__ int s[kMaxExperts + 1];
  const int e = threadIdx.x;
  int cnt = 0, q = 0;
  if (e < E) {
    cnt = offsets[e + 1] - offsets[e];
    q = (cnt + bn - 1) / bn;
    s[e] = q * n_tiles;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int i = 0; i < E; ++i) {
      const int v = s[i];
      s[i] = acc;
      acc += v;
    }
    s[E] = acc;
    *num = acc;
  }
  __syncthreads();
  if (e < E) {
    int w = s[e];
    const int m_end = offsets[e + 1];
    for (int qi = 0; qi < q; ++qi)
      for (int nt = 0; nt < n_tiles; ++nt) tab[w++] = make_int4(e, nt, offsets[e] + qi * bn, m_end);
  }
}

__global__ void combine_kernel(const __nv_bfloat16* __restrict__ rows, int ldr, const int* __restrict__ row_of_slot,
                               const float* __restrict__ wts, int top_k, int H, __nv_bfloat16* __restrict__ out,
                               int ldo) {
  const int t = blockIdx.x;
  for (int c = threadIdx.x * 2; c < H; c += blockDim.x * 2) {
    float a = 0.f, b = 0.f;
    for (int j = 0; j < top_k; ++j) {
      const int r = row_of_slot[t * top_k + j];
      const float w = wts[t * top_k + j];
      const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(rows + static_cast<size_t>(r) * ldr + c);
      a += w * __low2float(v);
      b += w * __high2float(v);
    }
    *reinterpret_cast<__nv_bfloat162*>(out + static_cast<size_t>(t) * ldo + c) = __floats2bfloat162_rn(a, b);
  }
}

}  // namespace moe
}  // namespace ib200

using namespace ib200::moe;

extern "C" int ib_moe_topk(const void* logits, int ld, int is_bf16, const float* bias, int T, int E, int n_groups,
                           int topk_groups, int top_k, int use_softmax, int renorm, float scaling, int* ids,
                           float* wts, cudaStream_t stream) {
  if (T <= 0) return 0;
  if (E > kMaxExperts || top_k > 32 || top_k > kMaxTopK || n_groups < 1 || n_groups > kMaxGroups ||
      E % n_groups != 0 || topk_groups < 1)
    return -1;
  const int warps = 4;
  const size_t smem = static_cast<size_t>(warps) * 2 * E * sizeof(float);
  topk_kernel<<<(T + warps - 1) / warps, warps * 32, smem, stream>>>(logits, ld, is_bf16, bias, T, E, n_groups,
                                                                       topk_groups, top_k, use_softmax, renorm, scaling,
                                                                       ids, wts);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

// counts / cursor: int32 workspaces of E (counts zeroed here); offsets: E+1
extern "C" int ib_moe_permute(const int* ids, int T, int top_k, int E, int* counts, int* cursor, int* offsets,
                              int* row_of_slot, int* token_of_row, cudaStream_t stream) {
  if (T <= 0) return 0;
  if (E > kMaxExperts) return -1;
  const int n = T * top_k;
  cudaMemsetAsync(counts, 0, sizeof(int) * E, stream);
  const int blocks = (n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024;
  count_kernel<<<blocks, 256, 0, stream>>>(ids, n, counts);
  scan_kernel<<<1, 256, 0, stream>>>(counts, E, offsets, cursor);
  scatter_kernel<<<blocks, 256, 0, stream>>>(ids, n, top_k, offsets, cursor, row_of_slot, token_of_row);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

extern "C" int ib_moe_tiles(const int* offsets, int E, int N, int bn, void* tab, int* num, cudaStream_t stream) {
  if (E > kMaxExperts || N % 128 != 0) return -1;
  tiles_kernel<<<1, E < 32 ? 32 : E, 0, stream>>>(offsets, E, N / 128, bn, static_cast<int4*>(tab), num);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

extern "C" int ib_moe_combine(const void* rows, int ldr, const int* row_of_slot, const float* wts, int T, int top_k,
                              int H, void* out, int ldo, cudaStream_t stream) {
  if (T <= 0) return 0;
  if (H % 2 != 0) return -1;
  combine_kernel<<<T, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(rows), ldr, row_of_slot, wts, top_k, H,
                                        static_cast<__nv_bfloat16*>(out), ldo);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}
