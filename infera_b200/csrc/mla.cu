// Multi-head latent attention (DeepSeek-V3 MLA), absorbed form, on tcgen05.
//
// The cache holds one 576-wide latent row per token: the RMS-normalised
// compressed KV c (512) followed by the rotated shared rope key (64). With
// the up-projections absorbed into the query and output sides, attention is
// multi-query attention with one 576-dim key / 512-dim value head:
//
//   S[h, t] = q[h] . cache[t]              (q = [W_UK^T q_nope | rope(q_pe)])
//   O[h]    = softmax_t(S[h, :] * scale) . cache[:, 0:512]
//
// One CTA handles one query (128 head rows; fewer heads leave the rest of
// the tile unused), one 256-dim half of the value dims and one split of the
// keys:
//   warp 0      TMA producer: the query's 9 x [128 x 64] blocks once, then
//               key tiles of two pages (32 tokens x 9 blocks of 64 dims) into
//               a 2-stage ring
//   warp 1      MMA issuer: S = Q K^T (M 128, N 32, K 576) into TMEM (double
//               buffered); O += P V (M 128, N 256, K 32) with P read from
//               TMEM and V = the tile's latent dims of this CTA's half, read
//               MN-major from the same ring stage
//   warps 2..5  softmax, thread = head row: running max with lazy O rescale
//               (only when the max grows by more than 2^8), P (bf16 pairs)
//               written back over the first 16 columns of the tile's own S,
//               final O / l epilogue or split partials with their
//               log-sum-exp
// The S MMAs cost about the same per instruction at N 16 and N 32 (issue-
// bound), so 32-key tiles halve their cost per key; 2 stages of 36 KiB keep
// the same key bytes in flight as 4 stages of one page did.
// TMEM: S 2 x 32 columns, O 256 columns. The 128 x 512 fp32 output of all
// heads would fill TMEM on its own, hence the value split over two CTAs (the
// two recompute S; they read the same key tiles, which L2 serves once).
// Prefill reuses the kernel with one "query" per prompt token (its own
// causal key count).
//
// Reference parity: the reference serves DeepSeek-V3 MLA through its
// engines (AITER MLA in vLLM / SGLang); none of that code is in its tree.
#include <cstdlib>

#include "sm100.cuh"
#include "tma_host.h"

namespace ib200 {
namespace mla {

inline int mla_key_tile() {
  static const int v = [] {
    const char* e = std::getenv("INFERA_MLA_TILE");
    return e != nullptr && std::atoi(e) == 32 ? 32 : 128;
  }();
  return v;
}

constexpr int DL = 512;
constexpr int DR = 64;
constexpr int DQK = DL + DR;
constexpr int NCH = DQK / 64;              // 9 blocks of 64 dims
constexpr int BT = 32;                     // keys per tile (two pages)
constexpr int PAGE = 16;
constexpr int STAGES = 2;
constexpr int QCH = 128 * 128;             // one [128 rows x 64 dims] bf16 block
constexpr int KCH = BT * 128;              // one [32 keys x 64 dims] block
constexpr int KV_STAGE = NCH * KCH;        // 36 KiB
constexpr int DV = 256;                    // value dims per CTA
constexpr int NUM_THREADS = 192;
// S of even / odd tiles (32 fp32 columns each; P of the tile, bf16 pairs,
// is written back over the first 16 of them), O 256 columns
constexpr uint32_t S_COL0 = 0, S_COL1 = 32, O_COL = 64;
constexpr int SMEM_BYTES = 1024 + NCH * QCH + STAGES * KV_STAGE + 256;

struct Params {
  const int* q_row;        // [nq] block-table row of each query
  const int* q_kvlen;      // [nq] keys visible to each query
  const int* block_table;  // [rows, max_pages]
  int max_pages;
  int hq;                  // head rows per query (<= 128)
  int splits;              // key splits per query (each covers ceil(tiles / splits) tiles)
  float scale_log2;
  __nv_bfloat16* out;      // [nq, hq, 512]
  float* o_part;           // [nq, splits, hq, 512]
  float* lse_part;         // [nq, splits, hq] (log2 units)
  int* status;
  long long* trace;        // optional: clock64 stamps of CTA (0,0,0)'s pipeline events (see TR_*)
  const __nv_bfloat16* cache;  // [num_slots, 576] (L2 prefetch of coming pages)
  int prefetch;            // tiles ahead whose pages are prefetched into L2 (0: none)
};

// pipeline event stamps (trace[event * kTraceTiles + tile]) for diagnosis
enum : int { TR_TMA = 0, TR_KVFULL, TR_SISSUE, TR_PFULL, TR_SFULL, TR_ODONE, TR_PARRIVE, kTraceEvents };
constexpr int kTraceTiles = 64;

__device__ __forceinline__ void stamp(const Params& p, bool cta0, int ev, int j) {
  if (p.trace != nullptr && cta0 && j < kTraceTiles) p.trace[ev * kTraceTiles + j] = clock64();
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    mla_decode_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                      const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + NCH * QCH;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + STAGES * KV_STAGE);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;          // [STAGES]
  uint64_t* kv_empty = kv_full + STAGES; // [STAGES]
  uint64_t* s_full = kv_empty + STAGES;  // [2]
  // [2] each: P written (128 arrivals) / PV done, for even and odd tiles: a
  // warp may run a tile ahead of the others, and its arrival must not count
  // toward the tile the slower warps are still writing.
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qi = blockIdx.x;
  const int half = blockIdx.y;
  const int sp = blockIdx.z;
  const int kvlen = p.q_kvlen[qi];
  const int n_tiles_all = (kvlen + BT - 1) / BT;
  const int tps = (n_tiles_all + p.splits - 1) / p.splits;
  const int tile0 = sp * tps;
  const int n_tiles = max(0, min(n_tiles_all - tile0, tps));
  const bool cta0 = blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(&p_full[0], 128);
    mbar_init(&p_full[1], 128);
    mbar_init(&o_done[0], 1);
    mbar_init(&o_done[1], 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmKV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && n_tiles > 0) {
      const uint64_t pol_q = policy_evict_first();
      const uint64_t pol_kv = policy_evict_last();  // the other value half reads the same tiles
      mbar_expect_tx(q_full, NCH * QCH);
      for (int c = 0; c < NCH; ++c) tma_load_2d(sQ + c * QCH, &tmQ, q_full, c * 64, qi * p.hq, pol_q);
      const int* bt = p.block_table + static_cast<size_t>(p.q_row[qi]) * p.max_pages;
      const int n_pages = (kvlen + PAGE - 1) / PAGE;
      // pages of tile t: 2t and 2t + 1 (past the sequence's last page: the
      // first again, its keys masked)
      auto pages_of = [&](int t, int& a, int& b) {
        a = __ldg(bt + 2 * t);
        b = 2 * t + 1 < n_pages ? __ldg(bt + 2 * t + 1) : a;
      };
      long long issued = 0;
      int na, nb;
      pages_of(tile0, na, nb);
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j % STAGES;
        const uint32_t ph = (j / STAGES) & 1;
        const int pa = na, pb = nb;
        if (j + 1 < n_tiles) pages_of(tile0 + j + 1, na, nb);  // in flight while we wait
        if (!mbar_wait(&kv_empty[st], ph ^ 1u, abort_flag, p.status, kStatusTimeoutEmpty)) break;
        uint8_t* base = sKV + st * KV_STAGE;
        mbar_expect_tx(&kv_full[st], KV_STAGE);
        for (int c = 0; c < NCH; ++c) {
          tma_load_2d(base + c * KCH, &tmKV, &kv_full[st], c * 64, pa * PAGE, pol_kv);
          tma_load_2d(base + c * KCH + PAGE * 128, &tmKV, &kv_full[st], c * 64, pb * PAGE, pol_kv);
        }
        stamp(p, cta0, TR_TMA, j);
        ++issued;
      }
      // drain: every issued copy must land before the CTA exits
      mbar_wait(q_full, 0, nullptr, nullptr, 0, kWaitLimitNs / 4);
      const long long first = issued > STAGES ? issued - STAGES : 0;
      for (long long i = first; i < issued; ++i)
        mbar_wait(&kv_full[i % STAGES], static_cast<uint32_t>((i / STAGES) & 1), nullptr, nullptr, 0,
                  kWaitLimitNs / 4);
    }
  } else if (warp == 1) {
    if (lane == 0 && n_tiles > 0) {
      const uint32_t idesc_qk = make_idesc_bf16(128, BT);
      const uint32_t idesc_pv = make_idesc_bf16(128, DV, true);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status, kStatusTimeoutFull);
      auto issue_pv = [&](int jj) -> bool {
        if (!mbar_wait(&p_full[jj & 1], static_cast<uint32_t>((jj >> 1) & 1), abort_flag, p.status,
                       kStatusTimeoutTmemEmpty))
          return false;
        stamp(p, cta0, TR_PFULL, jj);
        tc_fence_after();
        const int st = jj % STAGES;
        // V = latent dims [256*half, +256) of the tile: blocks 4*half .. 4*half+3;
        // P of this tile = the first 16 columns of its S (keys 16s.. are 8 columns)
        const uint32_t v_addr = smem_u32(sKV + st * KV_STAGE + half * 4 * KCH);
        const uint32_t p_col = (jj & 1) ? S_COL1 : S_COL0;
#pragma unroll
        for (int s = 0; s < BT / 16; ++s) {
          // MN-major V: LBO = distance between 64-dim blocks, SBO = 8 keys
          const uint64_t bd = make_sw128_desc(v_addr + s * 16 * 128, KCH, 1024);
          umma_bf16_ts(tmem + O_COL, tmem + p_col + s * 8, bd, idesc_pv, (jj > 0 || s > 0) ? 1u : 0u);
        }
        umma_commit(&o_done[jj & 1]);
        umma_commit(&kv_empty[st]);
        return true;
      };
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int st = j % STAGES;
        if (!mbar_wait(&kv_full[st], static_cast<uint32_t>((j / STAGES) & 1), abort_flag, p.status,
                       kStatusTimeoutFull)) {
          ok = false;
          break;
        }
        stamp(p, cta0, TR_KVFULL, j);
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sKV + st * KV_STAGE);
        const uint32_t s_col = (j & 1) ? S_COL1 : S_COL0;
        for (int c = 0; c < NCH; ++c) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = make_sw128_desc(q_addr + c * QCH + kk * 32, 16, 1024);
            const uint64_t bd = make_sw128_desc(k_addr + c * KCH + kk * 32, 16, 1024);
            umma_bf16(tmem + s_col, ad, bd, idesc_qk, (c > 0 || kk > 0) ? 1u : 0u);
          }
        }
        umma_commit(&s_full[j & 1]);
        stamp(p, cta0, TR_SISSUE, j);
        if (j > 0 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) issue_pv(n_tiles - 1);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, p.status, kStatusTimeoutFull);
    }
  } else {
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // head row
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles && ok; ++j) {
      if (!mbar_wait_warp(&s_full[j & 1], static_cast<uint32_t>((j >> 1) & 1), abort_flag, p.status,
                          kStatusTimeoutTmemFull)) {
        ok = false;
        break;
      }
      if (r == 0) stamp(p, cta0, TR_SFULL, j);
      tc_fence_after();
      uint32_t v[32];
      const uint32_t s_addr = lane_addr + ((j & 1) ? S_COL1 : S_COL0);
      tmem_ld32(s_addr, v);
      tmem_ld_wait();
      const int lim = kvlen - (tile0 + j) * BT;  // keys c < lim are valid
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (i >= lim) v[i] = __float_as_uint(-INFINITY);
        mx = fmaxf(mx, __uint_as_float(v[i]));
      }
      mx *= p.scale_log2;
      const float m_new = fmaxf(m_run, mx);
      const bool rescale = (j == 0) || (m_new > m_run + 8.0f);
      const float m_use = rescale ? m_new : m_run;
      const float alpha = (j == 0) ? 0.f : exp2f(m_run - m_use);
      const bool warp_rescale = __any_sync(0xffffffffu, rescale && j > 0);
      // P goes over S(j)'s own columns, which no MMA in flight touches (S(j+2)
      // reuses them and is issued after PV(j)); only a rescale of O waits for
      // every PV so far (tile j-1's)
      const int wait_tile = warp_rescale ? j - 1 : -1;
      if (wait_tile >= 0) {
        if (!mbar_wait_warp(&o_done[wait_tile & 1], static_cast<uint32_t>((wait_tile >> 1) & 1), abort_flag,
                            p.status, kStatusTimeoutTmemFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (r == 0) stamp(p, cta0, TR_ODONE, j);
      if (warp_rescale) {
#pragma unroll 1
        for (int c0 = 0; c0 < DV; c0 += 16) {
          uint32_t o[16];
          tmem_ld16(lane_addr + O_COL + c0, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st16(lane_addr + O_COL + c0, o);
        }
        tmem_st_wait();
      }
      float sum = 0.f;
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float e0 = exp2f(fmaf(__uint_as_float(v[i]), p.scale_log2, -m_use));
        const float e1 = exp2f(fmaf(__uint_as_float(v[i + 1]), p.scale_log2, -m_use));
        __nv_bfloat162 bb = __floats2bfloat162_rn(e0, e1);
        sum += __low2float(bb) + __high2float(bb);
        pk[i / 2] = *reinterpret_cast<uint32_t*>(&bb);
      }
      tmem_st16(s_addr, pk);
      l_run = l_run * alpha + sum;
      m_run = m_use;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
      if (r == 0) stamp(p, cta0, TR_PARRIVE, j);
    }
    ok = __all_sync(0xffffffffu, ok);
    const bool write = r < p.hq;
    const size_t row = static_cast<size_t>(qi) * p.hq + r;
    const int dv0 = half * DV;
    if (n_tiles == 0) {
      // no keys in this split: an empty partial (or zeros)
      if (write) {
        if (p.splits == 1) {
          for (int c = 0; c < DV; ++c) p.out[row * DL + dv0 + c] = __float2bfloat16(0.f);
        } else {
          const size_t prow = (static_cast<size_t>(qi) * p.splits + sp) * p.hq + r;
          for (int c = 0; c < DV; ++c) p.o_part[prow * DL + dv0 + c] = 0.f;
          if (half == 0) p.lse_part[prow] = -INFINITY;
        }
      }
    } else if (ok && mbar_wait_warp(&o_done[(n_tiles - 1) & 1], static_cast<uint32_t>(((n_tiles - 1) >> 1) & 1),
                                    abort_flag, p.status, kStatusTimeoutTmemFull)) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
      const size_t prow = (static_cast<size_t>(qi) * p.splits + sp) * p.hq + r;
#pragma unroll 1
      for (int c0 = 0; c0 < DV; c0 += 32) {
        uint32_t o[32];
        tmem_ld32(lane_addr + O_COL + c0, o);
        tmem_ld_wait();
        if (!write) continue;
        if (p.splits == 1) {
          __nv_bfloat16* dst = p.out + row * DL + dv0 + c0;
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            w.x = pack_bf16(__uint_as_float(o[i + 0]) * inv, __uint_as_float(o[i + 1]) * inv);
            w.y = pack_bf16(__uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
            w.z = pack_bf16(__uint_as_float(o[i + 4]) * inv, __uint_as_float(o[i + 5]) * inv);
            w.w = pack_bf16(__uint_as_float(o[i + 6]) * inv, __uint_as_float(o[i + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + i) = w;
          }
        } else {
          float* dst = p.o_part + prow * DL + dv0 + c0;
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(dst + i) =
                make_float4(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv,
                            __uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
        }
      }
      if (write && p.splits > 1 && half == 0) p.lse_part[prow] = m_run + log2f(l_run);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------
// 128-key tiles (eight pages): the S MMAs run at N = 128 (128 heads x 128
// keys x 16 dims each), where an MMA's math outlasts its fixed issue cost,
// instead of N = 32. A tile's 576 key dims no longer fit next to the
// resident Q, so keys stream through a 5-slot ring of [128 keys x 64 dims]
// chunks (16 KiB) in the order the MMA warp consumes them:
//   S chunks 0..8 of tile j, then V chunks 0..3 of tile j-1
// (V = this CTA's 256 latent dims, read again from L2: the S chunks of the
// same dims were released right after their MMAs).
//   warp 0      TMA producer (one lane)
//   warp 1      MMA issuer: S(j) = Q K^T into S buffer j&1 (9 x 4 MMAs,
//               M 128, N 128), then O[:, 64v:+64] += P(j-1) V_v
//               (4 x 8 MMAs, N 64, P from TMEM); S(j+1) overwrites P(j-1)
//               only after PV(j-1) was issued (tcgen05 MMAs run in order)
//   warps 2..5  softmax, thread = head row, 128 keys per tile; P as bf16
//               pairs over the first 64 columns of the tile's S
// TMEM: S 2 x 128 columns, O 256 columns.
constexpr int BT2 = 128;
constexpr int RING = 5;
constexpr int CH2 = BT2 * 128;                              // 16 KiB
constexpr int SMEM2 = 1024 + NCH * QCH + RING * CH2 + 256;
constexpr uint32_t S2_COL1 = 128, O2_COL = 256;

__device__ __forceinline__ uint64_t m2pack(float a, float b) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ void m2unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t m2fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    mla_decode128_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                         const __grid_constant__ CUtensorMap tmKV8, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sR = sQ + NCH * QCH;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sR + RING * CH2);
  uint64_t* q_full = bars;
  uint64_t* r_full = bars + 1;           // [RING]
  uint64_t* r_empty = r_full + RING;     // [RING]
  uint64_t* s_full = r_empty + RING;     // [2] by tile parity
  uint64_t* p_full = s_full + 2;         // [2]
  uint64_t* o_done = p_full + 2;         // [2]
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qi = blockIdx.x;
  const int half = blockIdx.y;
  const int sp = blockIdx.z;
  const int kvlen = p.q_kvlen[qi];
  const int n_tiles_all = (kvlen + BT2 - 1) / BT2;
  const int tps = (n_tiles_all + p.splits - 1) / p.splits;
  const int tile0 = sp * tps;
  const int n_tiles = max(0, min(n_tiles_all - tile0, tps));
  const bool cta0 = blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < RING; ++s) {
      mbar_init(&r_full[s], 1);
      mbar_init(&r_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 128);
      mbar_init(&o_done[b], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmKV);
    tma_prefetch_desc(&tmKV8);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && n_tiles > 0) {
      const uint64_t pol_q = policy_evict_first();
      const uint64_t pol_kv = policy_evict_last();  // V chunks and the other value half read the same rows
      mbar_expect_tx(q_full, NCH * QCH);
      for (int c = 0; c < NCH; ++c) tma_load_2d(sQ + c * QCH, &tmQ, q_full, c * 64, qi * p.hq, pol_q);
      const int* bt = p.block_table + static_cast<size_t>(p.q_row[qi]) * p.max_pages;
      const int n_pages = (kvlen + PAGE - 1) / PAGE;
      long long seq = 0;  // chunks issued so far (ring position)
      bool ok = true;
      int pg[8];
      auto load_chunk = [&](int col) -> bool {
        const int st = static_cast<int>(seq % RING);
        const uint32_t ph = static_cast<uint32_t>((seq / RING) & 1);
        if (!mbar_wait(&r_empty[st], ph ^ 1u, abort_flag, p.status, kStatusTimeoutEmpty)) return false;
        uint8_t* dst = sR + st * CH2;
        mbar_expect_tx(&r_full[st], CH2);
        bool run = true;
#pragma unroll
        for (int i = 1; i < 8; ++i) run = run && pg[i] == pg[0] + i;
        if (run) {
          tma_load_2d(dst, &tmKV8, &r_full[st], col, pg[0] * PAGE, pol_kv);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) tma_load_2d(dst + i * PAGE * 128, &tmKV, &r_full[st], col, pg[i] * PAGE, pol_kv);
        }
        ++seq;
        return true;
      };
      // pages of tile t (past the sequence's last page: its first page again,
      // those keys are masked)
      auto pages_of = [&](int t) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int lp = t * 8 + i;
          pg[i] = __ldg(bt + (lp < n_pages ? lp : t * 8));
        }
      };
      // INFERA_MLA_PREFETCH=n: pages of the tile n ahead go to L2 while this
      // one streams (a page is 16 rows x 576 dims, 18 KiB contiguous). Off
      // by default: 64 queries x 4096 keys ran 0.269 ms with n = 2 against
      // 0.247 ms without.
      const int kPrefetch = p.prefetch;
      auto prefetch_tile = [&](int t) {
        if (kPrefetch <= 0 || t >= tile0 + n_tiles) return;
        for (int i = 0; i < 8; ++i) {
          const int lp = t * 8 + i;
          if (lp >= n_pages) break;
          l2_prefetch_bulk(p.cache + static_cast<size_t>(__ldg(bt + lp)) * PAGE * DQK, PAGE * DQK * 2);
        }
      };
      for (int t = 0; t < kPrefetch; ++t) prefetch_tile(tile0 + t);
      for (int j = 0; j <= n_tiles && ok; ++j) {
        if (j < n_tiles) {
          prefetch_tile(tile0 + j + kPrefetch);
          pages_of(tile0 + j);
          for (int c = 0; c < NCH && ok; ++c) ok = load_chunk(c * 64);
          stamp(p, cta0, TR_TMA, j);
        }
        if (j >= 1 && ok) {
          pages_of(tile0 + j - 1);
          for (int v = 0; v < 4 && ok; ++v) ok = load_chunk(half * DV + v * 64);
        }
      }
      // drain: every issued copy must land before the CTA exits
      mbar_wait(q_full, 0, nullptr, nullptr, 0, kWaitLimitNs / 4);
      const long long first = seq > RING ? seq - RING : 0;
      for (long long i = first; i < seq; ++i)
        mbar_wait(&r_full[i % RING], static_cast<uint32_t>((i / RING) & 1), nullptr, nullptr, 0, kWaitLimitNs / 4);
    }
  } else if (warp == 1) {
    if (lane == 0 && n_tiles > 0) {
      const uint32_t idesc_qk = make_idesc_bf16(128, BT2);
      const uint32_t idesc_pv = make_idesc_bf16(128, 64, true);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status, kStatusTimeoutFull);
      long long seq = 0;
      auto take = [&](uint32_t& addr) -> bool {
        const int st = static_cast<int>(seq % RING);
        if (!mbar_wait(&r_full[st], static_cast<uint32_t>((seq / RING) & 1), abort_flag, p.status,
                       kStatusTimeoutFull))
          return false;
        tc_fence_after();
        addr = smem_u32(sR + st * CH2);
        return true;
      };
      auto release = [&]() {
        umma_commit(&r_empty[seq % RING]);
        ++seq;
      };
      for (int j = 0; j <= n_tiles && ok; ++j) {
        if (j < n_tiles) {
          const uint32_t s_col = (j & 1) ? S2_COL1 : 0u;
          for (int c = 0; c < NCH && ok; ++c) {
            uint32_t k_addr;
            if (!(ok = take(k_addr))) break;
            if (c == 0) stamp(p, cta0, TR_KVFULL, j);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t ad = make_sw128_desc(q_addr + c * QCH + kk * 32, 16, 1024);
              const uint64_t bd = make_sw128_desc(k_addr + kk * 32, 16, 1024);
              umma_bf16(tmem + s_col, ad, bd, idesc_qk, (c > 0 || kk > 0) ? 1u : 0u);
            }
            release();
          }
          if (!ok) break;
          umma_commit(&s_full[j & 1]);
          stamp(p, cta0, TR_SISSUE, j);
        }
        if (j >= 1) {
          const int jj = j - 1;
          if (!mbar_wait(&p_full[jj & 1], static_cast<uint32_t>((jj >> 1) & 1), abort_flag, p.status,
                         kStatusTimeoutTmemEmpty)) {
            ok = false;
            break;
          }
          stamp(p, cta0, TR_PFULL, jj);
          tc_fence_after();
          const uint32_t p_col = (jj & 1) ? S2_COL1 : 0u;
          for (int v = 0; v < 4 && ok; ++v) {
            uint32_t v_addr;
            if (!(ok = take(v_addr))) break;
#pragma unroll
            for (int s = 0; s < BT2 / 16; ++s) {
              // MN-major V chunk: keys 16s.. start 16 rows (2 KiB) further; SBO = 8 keys
              const uint64_t bd = make_sw128_desc(v_addr + s * 16 * 128, CH2, 1024);
              umma_bf16_ts(tmem + O2_COL + v * 64, tmem + p_col + s * 8, bd, idesc_pv,
                           (jj > 0 || s > 0) ? 1u : 0u);
            }
            release();
          }
          if (!ok) break;
          umma_commit(&o_done[jj & 1]);
        }
      }
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, p.status, kStatusTimeoutFull);
    }
  } else {
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // head row
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const float sl = p.scale_log2;
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles && ok; ++j) {
      if (!mbar_wait_warp(&s_full[j & 1], static_cast<uint32_t>((j >> 1) & 1), abort_flag, p.status,
                          kStatusTimeoutTmemFull)) {
        ok = false;
        break;
      }
      if (r == 0) stamp(p, cta0, TR_SFULL, j);
      tc_fence_after();
      const uint32_t s_addr = lane_addr + ((j & 1) ? S2_COL1 : 0u);
      const int lim = kvlen - (tile0 + j) * BT2;  // keys c < lim are valid
      uint32_t v[128];
      tmem_ld32(s_addr + 0, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tmem_ld32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tmem_ld32(s_addr + 64, *reinterpret_cast<uint32_t(*)[32]>(&v[64]));
      tmem_ld32(s_addr + 96, *reinterpret_cast<uint32_t(*)[32]>(&v[96]));
      tmem_ld_wait();
      if (lim < BT2) {
#pragma unroll
        for (int i = 0; i < BT2; ++i)
          if (i >= lim) v[i] = __float_as_uint(-INFINITY);
      }
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int i = 0; i < BT2; i += 2) {
        mx0 = fmaxf(mx0, __uint_as_float(v[i]));
        mx1 = fmaxf(mx1, __uint_as_float(v[i + 1]));
      }
      const float mx = fmaxf(mx0, mx1) * sl;
      const float m_new = fmaxf(m_run, mx);
      const bool rescale = (j == 0) || (m_new > m_run + 8.0f);
      const float m_use = rescale ? m_new : m_run;
      const float alpha = (j == 0) ? 0.f : exp2f(m_run - m_use);
      const bool warp_rescale = __any_sync(0xffffffffu, rescale && j > 0);
      // P goes over S(j)'s own columns, which no MMA in flight touches; only
      // a rescale of O waits for every PV so far (tile j-1's)
      if (warp_rescale) {
        if (!mbar_wait_warp(&o_done[(j - 1) & 1], static_cast<uint32_t>(((j - 1) >> 1) & 1), abort_flag, p.status,
                            kStatusTimeoutTmemFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (r == 0) stamp(p, cta0, TR_ODONE, j);
      // P = 2^(s*scale - m): pairs scaled with one f32x2 FMA, exponentials on MUFU
      const uint64_t sl2 = m2pack(sl, sl), nm2 = m2pack(-m_use, -m_use);
      float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
      for (int i = 0; i < BT2; i += 2) {
        float x0, x1;
        m2unpack(m2fma(m2pack(__uint_as_float(v[i]), __uint_as_float(v[i + 1])), sl2, nm2), x0, x1);
        const float e0 = exp2f(x0), e1 = exp2f(x1);
        sum0 += e0;
        sum1 += e1;
        v[i / 2] = pack_bf16(e0, e1);
      }
      tmem_st32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tmem_st32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      if (warp_rescale) {
#pragma unroll 1
        for (int c0 = 0; c0 < DV; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(lane_addr + O2_COL + c0, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(lane_addr + O2_COL + c0, o);
        }
      }
      l_run = l_run * alpha + (sum0 + sum1);
      m_run = m_use;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
      if (r == 0) stamp(p, cta0, TR_PARRIVE, j);
    }
    ok = __all_sync(0xffffffffu, ok);
    const bool write = r < p.hq;
    const size_t row = static_cast<size_t>(qi) * p.hq + r;
    const int dv0 = half * DV;
    if (n_tiles == 0) {
      if (write) {
        if (p.splits == 1) {
          for (int c = 0; c < DV; ++c) p.out[row * DL + dv0 + c] = __float2bfloat16(0.f);
        } else {
          const size_t prow = (static_cast<size_t>(qi) * p.splits + sp) * p.hq + r;
          for (int c = 0; c < DV; ++c) p.o_part[prow * DL + dv0 + c] = 0.f;
          if (half == 0) p.lse_part[prow] = -INFINITY;
        }
      }
    } else if (ok && mbar_wait_warp(&o_done[(n_tiles - 1) & 1], static_cast<uint32_t>(((n_tiles - 1) >> 1) & 1),
                                    abort_flag, p.status, kStatusTimeoutTmemFull)) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
      const size_t prow = (static_cast<size_t>(qi) * p.splits + sp) * p.hq + r;
#pragma unroll 1
      for (int c0 = 0; c0 < DV; c0 += 32) {
        uint32_t o[32];
        tmem_ld32(lane_addr + O2_COL + c0, o);
        tmem_ld_wait();
        if (!write) continue;
        if (p.splits == 1) {
          __nv_bfloat16* dst = p.out + row * DL + dv0 + c0;
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 w;
            w.x = pack_bf16(__uint_as_float(o[i + 0]) * inv, __uint_as_float(o[i + 1]) * inv);
            w.y = pack_bf16(__uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
            w.z = pack_bf16(__uint_as_float(o[i + 4]) * inv, __uint_as_float(o[i + 5]) * inv);
            w.w = pack_bf16(__uint_as_float(o[i + 6]) * inv, __uint_as_float(o[i + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + i) = w;
          }
        } else {
          float* dst = p.o_part + prow * DL + dv0 + c0;
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(dst + i) =
                make_float4(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv,
                            __uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
        }
      }
      if (write && p.splits > 1 && half == 0) p.lse_part[prow] = m_run + log2f(l_run);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, 512);
  }
}

// out[row] = sum_s 2^(lse_s - m) o_s / sum_s 2^(lse_s - m); one CTA per
// (query, head) row, 128 threads x 4 dims.
__global__ void __launch_bounds__(128) mla_combine_kernel(const float* __restrict__ o_part,
                                                          const float* __restrict__ lse_part, int hq, int splits,
                                                          __nv_bfloat16* __restrict__ out) {
  const int row = blockIdx.x;  // qi * hq + h
  const int qi = row / hq;
  const int h = row - qi * hq;
  float m = -INFINITY;
  for (int s = 0; s < splits; ++s) m = fmaxf(m, lse_part[(static_cast<size_t>(qi) * splits + s) * hq + h]);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float wsum = 0.f;
  if (m > -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      const size_t prow = (static_cast<size_t>(qi) * splits + s) * hq + h;
      const float w = exp2f(lse_part[prow] - m);
      if (w == 0.f) continue;
      const float4 o = *reinterpret_cast<const float4*>(o_part + prow * DL + threadIdx.x * 4);
      acc[0] += w * o.x;
      acc[1] += w * o.y;
      acc[2] += w * o.z;
      acc[3] += w * o.w;
      wsum += w;
    }
  }
  const float inv = wsum > 0.f ? 1.0f / wsum : 0.f;
  uint2 v;
  v.x = pack_bf16(acc[0] * inv, acc[1] * inv);
  v.y = pack_bf16(acc[2] * inv, acc[3] * inv);
  *reinterpret_cast<uint2*>(out + static_cast<size_t>(row) * DL + threadIdx.x * 4) = v;
}

// One CTA per token: c = rmsnorm(kva[0:512]) * w, k_pe = rope(kva[512:576]),
// cache[slot] = [c | k_pe] (slot < 0: no write), and every head's rope part
// of q (columns 512..575 of each 576-wide head row) rotated in place.
// Rotation pairs (i, i + 32) ("rotate half"); cos_sin [max_pos, 32, 2].
__global__ void __launch_bounds__(256) mla_rope_kvwrite_kernel(__nv_bfloat16* __restrict__ q, int hq,
                                                               const __nv_bfloat16* __restrict__ kva, int ldkva,
                                                               const int* __restrict__ pos,
                                                               const int* __restrict__ slots,
                                                               const float2* __restrict__ cos_sin,
                                                               const __nv_bfloat16* __restrict__ w, float eps,
                                                               __nv_bfloat16* __restrict__ cache) {
  __shared__ float red[8];
  const int t = blockIdx.x;
  const __nv_bfloat16* kr = kva + static_cast<size_t>(t) * ldkva;
  const int slot = slots[t];
  const int ps = pos[t];
  // RMSNorm of the 512 latent dims: 2 per thread
  const __nv_bfloat162 c2 = reinterpret_cast<const __nv_bfloat162*>(kr)[threadIdx.x];
  const float c0 = __low2float(c2), c1 = __high2float(c2);
  float ss = c0 * c0 + c1 * c1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = rsqrtf(tot / DL + eps);
  const __nv_bfloat162 w2 = reinterpret_cast<const __nv_bfloat162*>(w)[threadIdx.x];
  __nv_bfloat16* crow = slot >= 0 ? cache + static_cast<size_t>(slot) * DQK : nullptr;
  if (crow != nullptr)
    reinterpret_cast<__nv_bfloat162*>(crow)[threadIdx.x] =
        __floats2bfloat162_rn(c0 * inv * __low2float(w2), c1 * inv * __high2float(w2));
  const float2* cs = cos_sin + static_cast<size_t>(ps) * (DR / 2);
  // shared rope key
  if (threadIdx.x < DR / 2 && crow != nullptr) {
    const int i = threadIdx.x;
    const float a = __bfloat162float(kr[DL + i]), b = __bfloat162float(kr[DL + i + DR / 2]);
    const float2 c = cs[i];
    crow[DL + i] = __float2bfloat16(a * c.x - b * c.y);
    crow[DL + i + DR / 2] = __float2bfloat16(b * c.x + a * c.y);
  }
  // every head's rope query
  for (int k = threadIdx.x; k < hq * (DR / 2); k += blockDim.x) {
    const int h = k / (DR / 2);
    const int i = k - h * (DR / 2);
    __nv_bfloat16* qr = q + (static_cast<size_t>(t) * hq + h) * DQK + DL;
    const float a = __bfloat162float(qr[i]), b = __bfloat162float(qr[i + DR / 2]);
    const float2 c = cs[i];
    qr[i] = __float2bfloat16(a * c.x - b * c.y);
    qr[i + DR / 2] = __float2bfloat16(b * c.x + a * c.y);
  }
}

}  // namespace mla
}  // namespace ib200

using namespace ib200;

// q: [nq * hq, 576] bf16 (absorbed queries, rope part already rotated);
// cache: [num_slots, 576] bf16; q_row / q_kvlen: [nq] device int32; out:
// [nq, hq, 512] bf16. splits > 1 needs o_part [nq, splits, hq, 512] and
// lse_part [nq, splits, hq] fp32 scratch.
static long long* g_mla_trace = nullptr;

// Keys per tile of the decode kernel: 128 (default) or 32 (INFERA_MLA_TILE=32).
extern "C" int ib_mla_key_tile() { return mla::mla_key_tile(); }

// Diagnostics: the next launches stamp CTA (0,0,0)'s pipeline events into
// trace[7 * 64] (clock64), or stop when trace is null.
extern "C" void ib_mla_set_trace(long long* trace) { g_mla_trace = trace; }

extern "C" int ib_mla_decode(const void* q, int nq, int hq, const void* cache, long long num_slots,
                             const int* q_row, const int* q_kvlen, const int* block_table, int max_pages,
                             int splits, float scale, void* out, float* o_part, float* lse_part,
                             int* status, cudaStream_t stream) {
  using namespace ib200::mla;
  if (nq <= 0) return 0;
  if (hq < 1 || hq > 128 || splits < 1 || (splits > 1 && (o_part == nullptr || lse_part == nullptr))) return -1;
  CUtensorMap tq, tkv, tkv8;
  if (!cached_tmap_2d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, static_cast<long long>(nq) * hq, DQK, DQK, 128,
                      64))
    return -2;
  if (!cached_tmap_2d(&tkv, cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, num_slots, DQK, DQK, PAGE, 64)) return -2;
  const bool wide = mla_key_tile() == BT2;
  if (wide && !cached_tmap_2d(&tkv8, cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, num_slots, DQK, DQK, BT2, 64))
    return -2;
  Params p;
  p.q_row = q_row;
  p.q_kvlen = q_kvlen;
  p.block_table = block_table;
  p.max_pages = max_pages;
  p.hq = hq;
  p.splits = splits;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.o_part = o_part;
  p.lse_part = lse_part;
  p.status = status;
  p.trace = g_mla_trace;
  p.cache = static_cast<const __nv_bfloat16*>(cache);
  static const int prefetch = [] {
    const char* e = std::getenv("INFERA_MLA_PREFETCH");
    return e != nullptr && *e ? std::atoi(e) : 0;
  }();
  p.prefetch = prefetch;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(mla_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    cudaFuncSetAttribute(mla_decode128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2);
    attr_set[dev] = true;
  }
  dim3 grid(nq, 2, splits);
  if (wide)
    mla_decode128_kernel<<<grid, NUM_THREADS, SMEM2, stream>>>(tq, tkv, tkv8, p);
  else
    mla_decode_kernel<<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(tq, tkv, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return static_cast<int>(e);
  if (splits > 1) {
    mla_combine_kernel<<<nq * hq, 128, 0, stream>>>(o_part, lse_part, hq, splits, static_cast<__nv_bfloat16*>(out));
    e = cudaGetLastError();
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return 0;
}

extern "C" int ib_mla_rope_kvwrite(void* q, int T, int hq, const void* kva, int ldkva, const int* pos,
                                   const int* slots, const void* cos_sin, const void* norm_w, float eps, void* cache,
                                   cudaStream_t stream) {
  using namespace ib200::mla;
  if (T <= 0) return 0;
  if ((ldkva % 2) != 0) return -1;
  mla_rope_kvwrite_kernel<<<T, 256, 0, stream>>>(
      static_cast<__nv_bfloat16*>(q), hq, static_cast<const __nv_bfloat16*>(kva), ldkva, pos, slots,
      static_cast<const float2*>(cos_sin), static_cast<const __nv_bfloat16*>(norm_w), eps,
      static_cast<__nv_bfloat16*>(cache));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}
