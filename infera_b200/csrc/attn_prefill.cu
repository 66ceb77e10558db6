// Causal flash attention over a paged KV cache on tcgen05 tensor cores.
//
// One CTA computes 128 query rows of one query head:
//   warp 0      TMA producer: Q tile once, then K/V tiles of 128 keys
//               (8 pages of 16 tokens, two 64-dim halves each)
//   warp 1      MMA issuer: S = Q K^T into TMEM (double buffered),
//               O += P V into TMEM
//   warps 2..9  softmax, two warpgroups per query tile: warps w and w+4
//               share a TMEM lane quadrant (the same 32 rows) and each
//               handles half of the 128 keys of S / P and half of the 128
//               dims of O, exchanging only per-row maxima (bounded mbarrier
//               pair barrier); P (bf16 pairs) is written back into the
//               tile's own S columns of TMEM and the PV MMA reads its A
//               operand from there, so P never touches shared memory and
//               the softmax of tile j does not wait for PV(j-1) unless O
//               must be rescaled; O is rescaled in TMEM only when the
//               running max grows by more than 2^8 (lazy rescale); final
//               O / l epilogue.
//               Half of the exponentials run on the FMA pipe (polynomial).
//
// KV cache layout (per layer): [num_slots, Hkv * 128] bf16 with slot =
// page * 16 + offset, i.e. a page is 16 tokens x Hkv heads x 128 dims.
// V tiles are consumed MN-major (dims contiguous) as the B operand.
//
// The EXT variant scores over 192 query / key dims (MLA prefill: 128
// "nope" dims per head plus 64 rope dims that come from separate tensors,
// the rope key shared by every head) and still accumulates 128-dim values;
// every operand has its own row stride and per-head column stride, so the
// up-projected [k_nope | v] rows and the latent cache's rope columns are
// read in place.
//
// Reference parity: the reference runs prefill attention inside vLLM /
// SGLang / AITER (not in its tree); this is this framework's own kernel.
#include <cstdlib>

#include "sm100.cuh"
#include "tma_host.h"

namespace ib200 {
namespace fa {

constexpr int D = 128;
constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int PAGE = 16;
constexpr int BLK = 128 * 128;        // bytes of one 128-row x 64-col bf16 block (16 KiB)
constexpr int KV_STAGES = 2;
constexpr int NUM_THREADS = 320;  // producer, MMA, 8 softmax warps
// 64-dim blocks of Q / K: 2, or 3 with the extra rope dims
__host__ __device__ constexpr int qk_blocks(bool ext) { return ext ? 3 : 2; }
// smem: Q blocks + KV_STAGES x (K blocks + V 2 blocks)
__host__ __device__ constexpr int smem_bytes(bool ext) {
  return 1024 + (qk_blocks(ext) + KV_STAGES * (qk_blocks(ext) + 2)) * BLK + 4096;
}
constexpr uint32_t S_COL0 = 0, S_COL1 = 128, O_COL = 256;

struct Params {
  const int* tiles;        // [num_tiles * 2]: (seq, q_block)
  const int* q_start;      // [num_seqs] first row of the sequence in Q / O
  const int* q_len;        // [num_seqs]
  const int* ctx_len;      // [num_seqs] keys visible after this chunk
  const int* block_table;  // [rows, max_pages]
  const int* bt_rows;      // [num_seqs] table row of each sequence (null: row = seq)
  int max_pages;
  int num_heads, num_kv_heads;
  int q_hs, k_hs, v_hs;    // column stride between heads of Q / K / V (elements)
  int qe_hs, ke_hs;        // EXT: the same for the rope Q / K columns (0: shared)
  float scale_log2;        // softmax scale * log2(e)
  __nv_bfloat16* out;      // [T, num_heads * 128]
  int ldo;
  int* status;
  long long* trace;        // optional: clock64 stamps of CTA (0,0)'s pipeline events (FTR_*)
  int kv_splits;           // > 1: blockIdx.z takes one contiguous share of the key tiles
  float* o_part;           // kv_splits > 1: [T][num_heads][kv_splits][128] O / l of each share
  float* lse_part;         // kv_splits > 1: [T][num_heads][kv_splits] m + log2(l) (scaled log2 units)
};

// pipeline event stamps (trace[event * kFTraceTiles + tile]) for diagnosis
enum : int { FTR_TMA = 0, FTR_KFULL, FTR_SISSUE, FTR_PVISSUE, FTR_SFULL, FTR_PAIR, FTR_SOFTMAX, FTR_PARRIVE,
             kFTraceEvents };
constexpr int kFTraceTiles = 64;

__device__ __forceinline__ void fstamp(const Params& p, int ev, int j) {
  if (p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && j < kFTraceTiles)
    p.trace[ev * kFTraceTiles + j] = clock64();
}

// 2^x on the FMA pipe: split x = n + f (n integer, f in [0,1)), evaluate a
// cubic fitted to 2^f on [0,1) (max relative error 8.6e-5, far below bf16's
// 3.9e-3), and add n to the exponent. x = -inf (masked) gives 0.
__device__ __forceinline__ float exp2_fma(float x) {
  const float xc = fmaxf(x, -127.0f);
  const float n = floorf(xc);
  const float f = xc - n;
  const float pf = fmaf(fmaf(fmaf(0.07705903f, f, 0.22765373f), f, 0.69511485f), f, 1.0f);
  const float r = __int_as_float(__float_as_int(pf) + (static_cast<int>(n) << 23));
  return x == -INFINITY ? 0.0f : r;
}

template <bool EXT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    fa_prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmQe,
                      const __grid_constant__ CUtensorMap tmKe, const __grid_constant__ CUtensorMap tmK8,
                      const __grid_constant__ CUtensorMap tmV8, const __grid_constant__ CUtensorMap tmKe8,
                      const Params p) {
  pdl_trigger();
  pdl_wait();
  constexpr int QKB = qk_blocks(EXT);
  constexpr int STB = QKB + 2;     // blocks per KV stage
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                // QKB blocks of 64 dims
  uint8_t* sKV = smem + QKB * BLK;   // stage s: K blocks, V lo, V hi
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + KV_STAGES * STB * BLK);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;                 // [KV_STAGES]
  uint64_t* v_full = k_full + KV_STAGES;       // [KV_STAGES]
  // K stages are released once S of the tile is computed, V stages once its
  // PV is: the next K tiles load while the softmax still works on this one
  uint64_t* k_empty = v_full + KV_STAGES;      // [KV_STAGES]
  uint64_t* v_empty = k_empty + KV_STAGES;     // [KV_STAGES]
  uint64_t* s_full = v_empty + KV_STAGES;      // [2]
  uint64_t* p_full = s_full + 2;               // [2] by tile parity: the softmax may run a tile ahead of PV
  uint64_t* o_done = p_full + 2;               // [1]
  uint64_t* drain = o_done + 1;
  uint64_t* pair = drain + 1;                  // [4] per TMEM quadrant: the two softmax warps on it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pair + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(tmem_slot + 4);   // [2 tiles][2 halves][BQ] row maxima
  float* lsum = red + 4 * BQ;                               // [2 halves][BQ] row sums

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  const int seq = p.tiles[blockIdx.y * 2 + 0];
  const int qb = p.tiles[blockIdx.y * 2 + 1];
  const int kvh = h / (p.num_heads / p.num_kv_heads);
  const int qlen = p.q_len[seq];
  const int ctx = p.ctx_len[seq];
  const int row0 = p.q_start[seq] + qb * BQ;
  const int valid_rows = min(BQ, qlen - qb * BQ);
  const int pos0 = ctx - qlen + qb * BQ;           // position of row 0
  const int last_pos = pos0 + valid_rows - 1;
  const int n_kv = (last_pos + 1 + BKV - 1) / BKV;
  // this CTA's share of the key tiles: [j_lo, j_lo + nk)
  const int S = p.kv_splits > 1 ? p.kv_splits : 1;
  const int z = S > 1 ? blockIdx.z : 0;
  const int chunk = (n_kv + S - 1) / S;
  const int j_lo = z * chunk;
  const int nk = min(n_kv - j_lo, chunk);
  if (nk <= 0) {  // nothing in this share: mark it empty for the combine
    for (int r = threadIdx.x; r < valid_rows; r += blockDim.x)
      p.lse_part[(static_cast<size_t>(row0 + r) * p.num_heads + h) * S + z] = -INFINITY;
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(&p_full[0], 256);
    mbar_init(&p_full[1], 256);
    for (int i = 0; i < 4; ++i) mbar_init(&pair[i], 64);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    if (EXT) {
      tma_prefetch_desc(&tmQe);
      tma_prefetch_desc(&tmKe);
    }
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
    // lane 0 loads Q and the K tiles, lane 1 the V tiles, each at its own
    // pace (K stages free up after S, V stages after PV)
    if (lane < 2) {
      const bool is_k = lane == 0;
      const uint64_t pol = policy_evict_last();
      if (is_k) {
        mbar_expect_tx(q_full, QKB * BLK);
        tma_load_2d(sQ, &tmQ, q_full, h * p.q_hs, row0, pol);
        tma_load_2d(sQ + BLK, &tmQ, q_full, h * p.q_hs + 64, row0, pol);
        if (EXT) tma_load_2d(sQ + 2 * BLK, &tmQe, q_full, h * p.qe_hs, row0, pol);
      }
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      const int bt_row = p.bt_rows != nullptr ? p.bt_rows[seq] : seq;
      const int* bt = p.block_table + static_cast<size_t>(bt_row) * p.max_pages;
      const int n_pages = (ctx + PAGE - 1) / PAGE;
      long long issued = 0;
      int nxt[8];
      load_tile_pages(bt, j_lo, n_pages, nxt);
      for (int j = 0; j < nk; ++j) {
        const int st = j % KV_STAGES;
        const uint32_t ph = (j / KV_STAGES) & 1;
        int cur[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) cur[i] = nxt[i];
        if (j + 1 < nk) load_tile_pages(bt, j_lo + j + 1, n_pages, nxt);  // in flight while we wait
        if (!mbar_wait(&empty[st], ph ^ 1u, abort_flag, p.status, kStatusTimeoutEmpty)) break;
        uint8_t* base = sKV + st * STB * BLK;
        if (is_k) fstamp(p, FTR_TMA, j);
        // eight consecutive pages are one 128-row box per 64-dim block (the
        // same shared-memory image as eight page boxes: the 128-byte swizzle
        // repeats every 8 rows)
        bool run = true;
#pragma unroll
        for (int pg = 1; pg < BKV / PAGE; ++pg) run = run && cur[pg] == cur[0] + pg;
        if (is_k) {
          mbar_expect_tx(&full[st], QKB * BLK);
          if (run) {
            const int r = cur[0] * PAGE;
            tma_load_2d(base, &tmK8, &full[st], kvh * p.k_hs, r, pol);
            tma_load_2d(base + BLK, &tmK8, &full[st], kvh * p.k_hs + 64, r, pol);
            if (EXT) tma_load_2d(base + 2 * BLK, &tmKe8, &full[st], kvh * p.ke_hs, r, pol);
          } else {
#pragma unroll
            for (int pg = 0; pg < BKV / PAGE; ++pg) {
              const int r = cur[pg] * PAGE;
              tma_load_2d(base + pg * PAGE * 128, &tmK, &full[st], kvh * p.k_hs, r, pol);
              tma_load_2d(base + BLK + pg * PAGE * 128, &tmK, &full[st], kvh * p.k_hs + 64, r, pol);
              if (EXT) tma_load_2d(base + 2 * BLK + pg * PAGE * 128, &tmKe, &full[st], kvh * p.ke_hs, r, pol);
            }
          }
        } else {
          mbar_expect_tx(&full[st], 2 * BLK);
          if (run) {
            const int r = cur[0] * PAGE;
            tma_load_2d(base + QKB * BLK, &tmV8, &full[st], kvh * p.v_hs, r, pol);
            tma_load_2d(base + (QKB + 1) * BLK, &tmV8, &full[st], kvh * p.v_hs + 64, r, pol);
          } else {
#pragma unroll
            for (int pg = 0; pg < BKV / PAGE; ++pg) {
              const int r = cur[pg] * PAGE;
              tma_load_2d(base + QKB * BLK + pg * PAGE * 128, &tmV, &full[st], kvh * p.v_hs, r, pol);
              tma_load_2d(base + (QKB + 1) * BLK + pg * PAGE * 128, &tmV, &full[st], kvh * p.v_hs + 64, r,
                          pol);
            }
          }
        }
        ++issued;
      }
      // drain: every issued tile's bytes must have landed before exit
      if (is_k) mbar_wait(q_full, 0, nullptr, nullptr, 0, kWaitLimitNs / 4);
      long long first = issued > KV_STAGES ? issued - KV_STAGES : 0;
      for (long long i = first; i < issued; ++i)
        mbar_wait(&full[i % KV_STAGES], static_cast<uint32_t>((i / KV_STAGES) & 1), nullptr, nullptr, 0,
                  kWaitLimitNs / 4);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_qk = make_idesc_bf16(128, 128, false);
      const uint32_t idesc_pv = make_idesc_bf16(128, 128, true);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status, kStatusTimeoutFull);
      auto issue_pv = [&](int jj) -> bool {
        // O += P V_jj once softmax has written P for tile jj
        if (!mbar_wait(&p_full[jj & 1], static_cast<uint32_t>((jj >> 1) & 1), abort_flag, p.status,
                       kStatusTimeoutTmemEmpty))
          return false;
        const int st = jj % KV_STAGES;
        if (!mbar_wait(&v_full[st], static_cast<uint32_t>((jj / KV_STAGES) & 1), abort_flag, p.status,
                       kStatusTimeoutFull))
          return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sKV + st * STB * BLK + QKB * BLK);
        // P of tile jj sits in the first 32 columns of each 64-column half
        // of S(jj): keys 16s..16s+15 are 8 packed columns
        const uint32_t p_col = (jj & 1) ? S_COL1 : S_COL0;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint32_t a_tmem = tmem + p_col + (s >> 2) * 64 + (s & 3) * 8;
          // MN-major V: LBO = distance between the two 64-dim halves, SBO = 8 keys
          const uint64_t bd = make_sw128_desc(v_addr + s * 2048, BLK, 1024);
          umma_bf16_ts(tmem + O_COL, a_tmem, bd, idesc_pv, (jj > 0 || s > 0) ? 1u : 0u);
        }
        umma_commit(o_done);
        fstamp(p, FTR_PVISSUE, jj);
        umma_commit(&v_empty[st]);
        return true;
      };
      for (int j = 0; j < nk && ok; ++j) {
        const int st = j % KV_STAGES;
        if (!mbar_wait(&k_full[st], static_cast<uint32_t>((j / KV_STAGES) & 1), abort_flag, p.status,
                       kStatusTimeoutFull)) {
          ok = false;
          break;
        }
        fstamp(p, FTR_KFULL, j);
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sKV + st * STB * BLK);
        const uint32_t s_col = (j & 1) ? S_COL1 : S_COL0;
#pragma unroll
        for (int s = 0; s < 4 * QKB; ++s) {
          const uint32_t off = (s >> 2) * BLK + (s & 3) * 32;
          const uint64_t ad = make_sw128_desc(q_addr + off, 16, 1024);
          const uint64_t bd = make_sw128_desc(k_addr + off, 16, 1024);
          umma_bf16(tmem + s_col, ad, bd, idesc_qk, s > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[j & 1]);
        umma_commit(&k_empty[st]);   // K(j) is read once S(j) is done
        fstamp(p, FTR_SISSUE, j);
        if (j > 0 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && nk > 0) issue_pv(nk - 1);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, p.status, kStatusTimeoutFull);
    }
  } else {
    // softmax warps 2..9: two warpgroups per query tile. Warps w and w+4
    // share a TMEM lane quadrant (the same 32 rows); warpgroup `half` owns
    // keys [64*half, 64*half+64) of S and P and dims [64*half, +64) of O.
    const int q4 = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = q4 * 32 + lane;
    const int cb = half * 64;
    const int pos = pos0 + min(r, valid_rows - 1);
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    float m_run = -INFINITY;  // running max in log2 units (scaled)
    float l_run = 0.f;        // this half's share of the row sum
    bool ok = true;
    uint32_t pph = 0;         // phase of this quadrant's pair barrier
    auto pair_sync = [&]() {
      mbar_arrive(&pair[q4]);
      ok = mbar_wait_warp(&pair[q4], pph & 1u, abort_flag, p.status, kStatusTimeoutTmemFull) && ok;
      ++pph;
    };
    const bool tr0 = half == 0 && r == 0;  // one softmax thread stamps
    for (int j = 0; j < nk && ok; ++j) {
      if (!mbar_wait_warp(&s_full[j & 1], static_cast<uint32_t>((j >> 1) & 1), abort_flag, p.status,
                          kStatusTimeoutTmemFull)) {
        ok = false;
        break;
      }
      if (tr0) fstamp(p, FTR_SFULL, j);
      tc_fence_after();
      const uint32_t s_addr = lane_addr + ((j & 1) ? S_COL1 : S_COL0) + cb;
      const int kbase = (j_lo + j) * BKV;
      const int lim = pos - kbase - cb;  // local key c visible iff c <= lim
      // every row of the CTA sees the whole tile when it ends at or before the
      // position of row 0 (CTA-uniform): no per-element mask needed
      const bool full_tile = kbase + BKV - 1 <= pos0;
      uint32_t v[64];
      tmem_ld32(s_addr + 0, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      tmem_ld32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
      tmem_ld_wait();
      float mx = -INFINITY;
      if (full_tile) {
#pragma unroll
        for (int i = 0; i < 64; ++i) mx = fmaxf(mx, __uint_as_float(v[i]));
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          if (i > lim) v[i] = __float_as_uint(-INFINITY);
          mx = fmaxf(mx, __uint_as_float(v[i]));
        }
      }
      // combine the two halves' maxima of each row (double-buffered by tile)
      red[((j & 1) * 2 + half) * BQ + r] = mx;
      pair_sync();
      if (tr0) fstamp(p, FTR_PAIR, j);
      if (!ok) break;
      mx = fmaxf(red[((j & 1) * 2) * BQ + r], red[((j & 1) * 2 + 1) * BQ + r]) * p.scale_log2;
      const float m_new = fmaxf(m_run, mx);
      // Per-row choice (lazy rescale: keep a stale max unless the new one
      // exceeds it by 2^8). Both halves make the same choice for a row; the
      // TMEM rescale is warp-collective, so the warp rescales if ANY of its
      // rows needs it, with factor 1.0 for the others.
      const bool rescale = (j == 0) || (m_new > m_run + 8.0f);
      const float m_use = rescale ? m_new : m_run;
      // a row whose keys in this share are all masked so far keeps m = -inf
      // (only possible in a later share of a split row): no rescale, and
      // the exponentials below use 0 as reference so they give exact zeros
      const float alpha = (j == 0 || m_run == -INFINITY) ? 0.f : exp2f(m_run - m_use);
      const float m_ref = m_use == -INFINITY ? 0.f : m_use;
      const bool warp_rescale = __any_sync(0xffffffffu, rescale && j > 0);
      // O must not be rescaled while the previous tile's PV accumulates into
      // it: only a rescale waits for PV(j-1). P(j) goes to S(j)'s own
      // columns, which no MMA in flight reads or writes (S(j+2) reuses them
      // and is issued after PV(j); tcgen05.mma runs in issue order).
      if (j > 0 && warp_rescale) {
        if (!mbar_wait_warp(o_done, static_cast<uint32_t>((j - 1) & 1), abort_flag, p.status,
                            kStatusTimeoutTmemFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (warp_rescale) {
#pragma unroll 1
        for (int c0 = 0; c0 < 64; c0 += 16) {
          uint32_t o[16];
          tmem_ld16(lane_addr + O_COL + cb + c0, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st16(lane_addr + O_COL + cb + c0, o);
        }
        tmem_st_wait();
      }
      // P = 2^(s*scale - m): even columns on the MUFU unit, odd columns with
      // the FMA-pipe polynomial. Masked entries hold -inf and give exactly 0.
      float sum = 0.f;
      const float sl = p.scale_log2;
#pragma unroll
      for (int i = 0; i < 64; i += 2) {
        const float e0 = exp2f(fmaf(__uint_as_float(v[i]), sl, -m_ref));
        const float e1 = exp2_fma(fmaf(__uint_as_float(v[i + 1]), sl, -m_ref));
        __nv_bfloat162 bb = __floats2bfloat162_rn(e0, e1);
        sum += __low2float(bb) + __high2float(bb);
        v[i / 2] = *reinterpret_cast<uint32_t*>(&bb);   // packed pairs reuse the low half of v
      }
      // this half's S columns are already in registers: its packed P
      // overwrites the first 32 of them
      tmem_st32(s_addr, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      if (tr0) fstamp(p, FTR_SOFTMAX, j);
      l_run = l_run * alpha + sum;
      m_run = m_use;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
      if (tr0) fstamp(p, FTR_PARRIVE, j);
    }
    ok = __all_sync(0xffffffffu, ok);
    // row sums: add the two halves' shares
    lsum[half * BQ + r] = l_run;
    pair_sync();
    if (ok && nk > 0) {
      if (mbar_wait_warp(o_done, static_cast<uint32_t>((nk - 1) & 1), abort_flag, p.status,
                         kStatusTimeoutTmemFull)) {
        tc_fence_after();
        const float l = lsum[r] + lsum[BQ + r];
        const float inv = l > 0.f ? 1.0f / l : 0.f;
        const bool write = r < valid_rows;
        if (S > 1) {
          // this share's O / l and m + log2(l), merged by the combine kernel
          const size_t base = (static_cast<size_t>(row0 + r) * p.num_heads + h) * S + z;
          if (write && half == 0) p.lse_part[base] = l > 0.f ? m_run + __log2f(l) : -INFINITY;
          float* orow = p.o_part + base * D + cb;
#pragma unroll 1
          for (int c0 = 0; c0 < 64; c0 += 32) {
            uint32_t o[32];
            tmem_ld32(lane_addr + O_COL + cb + c0, o);
            tmem_ld_wait();
            if (write) {
#pragma unroll
              for (int i = 0; i < 32; i += 4)
                *reinterpret_cast<float4*>(orow + c0 + i) =
                    make_float4(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv,
                                __uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
            }
          }
        } else {
          __nv_bfloat16* orow = p.out + static_cast<size_t>(row0 + r) * p.ldo + h * D + cb;
#pragma unroll 1
          for (int c0 = 0; c0 < 64; c0 += 32) {
            uint32_t o[32];
            tmem_ld32(lane_addr + O_COL + cb + c0, o);
            tmem_ld_wait();
            if (write) {
#pragma unroll
              for (int i = 0; i < 32; i += 8) {
                uint4 w;
                w.x = pack_bf16(__uint_as_float(o[i + 0]) * inv, __uint_as_float(o[i + 1]) * inv);
                w.y = pack_bf16(__uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
                w.z = pack_bf16(__uint_as_float(o[i + 4]) * inv, __uint_as_float(o[i + 5]) * inv);
                w.w = pack_bf16(__uint_as_float(o[i + 6]) * inv, __uint_as_float(o[i + 7]) * inv);
                *reinterpret_cast<uint4*>(orow + c0 + i) = w;
              }
            }
          }
        }
      }
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
// Two query tiles per CTA (128-dim heads): 256 query rows of one head share
// every K / V tile, so each tile is read from shared memory by twice the
// math, and the tensor core alternates between the tiles while the other
// tile's softmax runs:
//   warp 0      TMA producer: Q0 / Q1 once, then K (lane 0) and V (lane 1)
//   warp 1      MMA issuer, per key tile j:
//                 PV0(j-1), S0(j), PV1(j-1), S1(j)
//               S_t(j) overwrites the columns that held P_t(j-1), so it is
//               issued after PV_t(j-1); tcgen05 MMAs run in issue order,
//               hence S_t(j) complete implies O_t holds every PV up to j-1.
//   warps 2..5  softmax of tile 0, one query row per thread (all 128 keys)
//   warps 6..9  softmax of tile 1
// TMEM: S_t / P_t at columns [128 t, 128 t + 128), O_t at [256 + 128 t, +128).
// A tile whose rows need fewer key tiles (the first tile of a causal pair)
// stops early; a pair whose second tile lies past the sequence runs tile 0
// alone.
constexpr int SMEM2 = 1024 + (4 + KV_STAGES * 4) * BLK + 1024;

// Packed fp32 pairs (Blackwell f32x2 FMA / add): two lanes of work per issue.
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x for two values on the FMA pipe, packed: x = n + f with n = round(x)
// (adding 1.5 * 2^23 leaves n in the low mantissa bits) and f in
// [-0.5, 0.5]; 2^f from a cubic fitted here to minimise the relative error
// on that interval (7.5e-5 at fp32, far below bf16's 3.9e-3); n joins the
// exponent by an integer add of n << 23 (the constant's own bits shift out).
// Inputs below -125 are clamped (the result stays a normal number).
__device__ __forceinline__ void exp2_poly2(float xa, float xb, float& ea, float& eb) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  const float a = fmaxf(xa, -125.0f), b = fmaxf(xb, -125.0f);
  const float ta = a + kRound, tb = b + kRound;
  const uint64_t n2 = fadd2(f2pack(ta, tb), f2pack(-kRound, -kRound));
  const uint64_t f2 = ffma2(n2, f2pack(-1.0f, -1.0f), f2pack(a, b));
  uint64_t p2 = ffma2(f2pack(0.05517098f, 0.05517098f), f2, f2pack(0.24260972f, 0.24260972f));
  p2 = ffma2(p2, f2, f2pack(0.69326097f, 0.69326097f));
  p2 = ffma2(p2, f2, f2pack(0.99992818f, 0.99992818f));
  float pa, pb;
  f2unpack(p2, pa, pb);
  ea = __uint_as_float((__float_as_uint(ta) << 23) + __float_as_uint(pa));
  eb = __uint_as_float((__float_as_uint(tb) << 23) + __float_as_uint(pb));
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <bool PACKED, int POLY>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    fa_prefill2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmK8,
                       const __grid_constant__ CUtensorMap tmV8, const Params p) {
  pdl_trigger();
  pdl_wait();
  constexpr int STB = 4;  // blocks per KV stage: K lo, K hi, V lo, V hi
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                // tile t: blocks 2t, 2t+1
  uint8_t* sKV = smem + 4 * BLK;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + KV_STAGES * STB * BLK);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;                 // [KV_STAGES]
  uint64_t* v_full = k_full + KV_STAGES;       // [KV_STAGES]
  uint64_t* k_empty = v_full + KV_STAGES;      // [KV_STAGES]
  uint64_t* v_empty = k_empty + KV_STAGES;     // [KV_STAGES]
  uint64_t* s_full = v_empty + KV_STAGES;      // [2] per query tile
  uint64_t* p_full = s_full + 2;               // [2] per query tile
  uint64_t* o_done = p_full + 2;               // [2] per query tile
  uint64_t* drain = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  const int seq = p.tiles[blockIdx.y * 2 + 0];
  const int qb = p.tiles[blockIdx.y * 2 + 1];   // first of the pair's two 128-row blocks
  const int kvh = h / (p.num_heads / p.num_kv_heads);
  const int qlen = p.q_len[seq];
  const int ctx = p.ctx_len[seq];
  int rows_t[2], pos0_t[2], nkv_t[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    rows_t[t] = min(BQ, qlen - (qb + t) * BQ);
    pos0_t[t] = ctx - qlen + (qb + t) * BQ;
    nkv_t[t] = rows_t[t] > 0 ? (pos0_t[t] + rows_t[t] + BKV - 1) / BKV : 0;
  }
  const int n_kv = max(nkv_t[0], nkv_t[1]);
  const int S = p.kv_splits > 1 ? p.kv_splits : 1;
  const int z = S > 1 ? blockIdx.z : 0;
  const int chunk = (n_kv + S - 1) / S;
  const int j_lo = z * chunk;
  const int nk = min(n_kv - j_lo, chunk);
  int nk_t[2];
#pragma unroll
  for (int t = 0; t < 2; ++t) nk_t[t] = max(0, min(nkv_t[t] - j_lo, chunk));
  const int row_base = p.q_start[seq] + qb * BQ;
  if (nk <= 0) {
    for (int r = threadIdx.x; r < 2 * BQ; r += blockDim.x)
      if (r < BQ ? r < rows_t[0] : r - BQ < rows_t[1])
        p.lse_part[(static_cast<size_t>(row_base + r) * p.num_heads + h) * S + z] = -INFINITY;
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 128);
      mbar_init(&o_done[t], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK8);
    tma_prefetch_desc(&tmV8);
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
    if (lane < 2) {
      const bool is_k = lane == 0;
      const uint64_t pol = policy_evict_last();
      if (is_k) {
        const int nq = rows_t[1] > 0 ? 2 : 1;
        mbar_expect_tx(q_full, nq * 2 * BLK);
        for (int t = 0; t < nq; ++t) {
          tma_load_2d(sQ + 2 * t * BLK, &tmQ, q_full, h * p.q_hs, row_base + t * BQ, pol);
          tma_load_2d(sQ + (2 * t + 1) * BLK, &tmQ, q_full, h * p.q_hs + 64, row_base + t * BQ, pol);
        }
      }
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      const int bt_row = p.bt_rows != nullptr ? p.bt_rows[seq] : seq;
      const int* bt = p.block_table + static_cast<size_t>(bt_row) * p.max_pages;
      const int n_pages = (ctx + PAGE - 1) / PAGE;
      const int hs = is_k ? p.k_hs : p.v_hs;
      const CUtensorMap* tm1 = is_k ? &tmK : &tmV;
      const CUtensorMap* tm8 = is_k ? &tmK8 : &tmV8;
      const int boff = is_k ? 0 : 2 * BLK;
      long long issued = 0;
      int nxt[8];
      load_tile_pages(bt, j_lo, n_pages, nxt);
      for (int j = 0; j < nk; ++j) {
        const int st = j % KV_STAGES;
        const uint32_t ph = (j / KV_STAGES) & 1;
        int cur[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) cur[i] = nxt[i];
        if (j + 1 < nk) load_tile_pages(bt, j_lo + j + 1, n_pages, nxt);
        if (!mbar_wait(&empty[st], ph ^ 1u, abort_flag, p.status, kStatusTimeoutEmpty)) break;
        uint8_t* base = sKV + st * STB * BLK + boff;
        if (is_k) fstamp(p, FTR_TMA, j);
        bool run = true;
#pragma unroll
        for (int pg = 1; pg < BKV / PAGE; ++pg) run = run && cur[pg] == cur[0] + pg;
        mbar_expect_tx(&full[st], 2 * BLK);
        if (run) {
          const int r = cur[0] * PAGE;
          tma_load_2d(base, tm8, &full[st], kvh * hs, r, pol);
          tma_load_2d(base + BLK, tm8, &full[st], kvh * hs + 64, r, pol);
        } else {
#pragma unroll
          for (int pg = 0; pg < BKV / PAGE; ++pg) {
            const int r = cur[pg] * PAGE;
            tma_load_2d(base + pg * PAGE * 128, tm1, &full[st], kvh * hs, r, pol);
            tma_load_2d(base + BLK + pg * PAGE * 128, tm1, &full[st], kvh * hs + 64, r, pol);
          }
        }
        ++issued;
      }
      if (is_k) mbar_wait(q_full, 0, nullptr, nullptr, 0, kWaitLimitNs / 4);
      long long first = issued > KV_STAGES ? issued - KV_STAGES : 0;
      for (long long i = first; i < issued; ++i)
        mbar_wait(&full[i % KV_STAGES], static_cast<uint32_t>((i / KV_STAGES) & 1), nullptr, nullptr, 0,
                  kWaitLimitNs / 4);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_qk = make_idesc_bf16(128, 128, false);
      const uint32_t idesc_pv = make_idesc_bf16(128, 128, true);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status, kStatusTimeoutFull);
      for (int j = 0; j <= nk && ok; ++j) {
        const int st = j % KV_STAGES;
        if (j < nk) {
          if (!mbar_wait(&k_full[st], static_cast<uint32_t>((j / KV_STAGES) & 1), abort_flag, p.status,
                         kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          fstamp(p, FTR_KFULL, j);
        }
        const int pst = (j + KV_STAGES - 1) % KV_STAGES;   // stage of key tile j-1
        bool v_ready = false;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int nkt = t ? nk_t[1] : nk_t[0];
          if (j >= 1 && j - 1 < nkt) {
            // O_t += P_t(j-1) V(j-1)
            if (!mbar_wait(&p_full[t], static_cast<uint32_t>((j - 1) & 1), abort_flag, p.status,
                           kStatusTimeoutTmemEmpty)) {
              ok = false;
              break;
            }
            if (!v_ready) {
              if (!mbar_wait(&v_full[pst], static_cast<uint32_t>(((j - 1) / KV_STAGES) & 1), abort_flag, p.status,
                             kStatusTimeoutFull)) {
                ok = false;
                break;
              }
              v_ready = true;
            }
            tc_fence_after();
            const uint32_t v_addr = smem_u32(sKV + pst * STB * BLK + 2 * BLK);
#pragma unroll
            for (int s = 0; s < 8; ++s) {
              // P_t packs keys 16s..16s+15 into columns 8s..8s+7 of S_t
              const uint64_t bd = make_sw128_desc(v_addr + s * 2048, BLK, 1024);
              umma_bf16_ts(tmem + O_COL + t * 128, tmem + t * 128 + s * 8, bd, idesc_pv,
                           (j > 1 || s > 0) ? 1u : 0u);
            }
            umma_commit(&o_done[t]);
            if (t == 0) fstamp(p, FTR_PVISSUE, j - 1);
          }
          if (j < nkt) {
            tc_fence_after();
            const uint32_t k_addr = smem_u32(sKV + st * STB * BLK);
            const uint32_t qa = q_addr + t * 2 * BLK;
#pragma unroll
            for (int s = 0; s < 8; ++s) {
              const uint32_t off = (s >> 2) * BLK + (s & 3) * 32;
              umma_bf16(tmem + t * 128, make_sw128_desc(qa + off, 16, 1024), make_sw128_desc(k_addr + off, 16, 1024),
                        idesc_qk, s > 0 ? 1u : 0u);
            }
            umma_commit(&s_full[t]);
            if (t == 0) fstamp(p, FTR_SISSUE, j);
          }
        }
        if (!ok) break;
        if (j < nk) umma_commit(&k_empty[st]);
        if (j >= 1) umma_commit(&v_empty[pst]);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, p.status, kStatusTimeoutFull);
    }
  } else {
    const int t = (warp - 2) >> 2;
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const int rows = t ? rows_t[1] : rows_t[0];   // selects: no dynamically indexed local arrays
    const int pos0 = t ? pos0_t[1] : pos0_t[0];
    const int nkt = t ? nk_t[1] : nk_t[0];
    const int pos = pos0 + min(r, max(rows, 1) - 1);
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const uint32_t s_addr = lane_addr + t * 128;
    const uint32_t o_addr = lane_addr + O_COL + t * 128;
    const float sl = p.scale_log2;
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    const bool tr0 = t == 0 && r == 0;
    for (int j = 0; j < nkt && ok; ++j) {
      if (!mbar_wait_warp(&s_full[t], static_cast<uint32_t>(j & 1), abort_flag, p.status, kStatusTimeoutTmemFull)) {
        ok = false;
        break;
      }
      if (tr0) fstamp(p, FTR_SFULL, j);
      tc_fence_after();
      const int kbase = (j_lo + j) * BKV;
      const int lim = pos - kbase;  // key c of the tile is visible iff c <= lim
      const bool full_tile = kbase + BKV - 1 <= pos0;
      // pass 1: the row maximum over all 128 keys
      float mx;
      {
        uint32_t v[128];
        tmem_ld32(s_addr + 0, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_ld32(s_addr + 64, *reinterpret_cast<uint32_t(*)[32]>(&v[64]));
        tmem_ld32(s_addr + 96, *reinterpret_cast<uint32_t(*)[32]>(&v[96]));
        tmem_ld_wait();
        if (!full_tile) {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i > lim) v[i] = __float_as_uint(-INFINITY);
        }
        float mx0 = __uint_as_float(v[0]), mx1 = __uint_as_float(v[1]);
#pragma unroll
        for (int i = 2; i < 128; i += 4) {
          mx0 = max3f(mx0, __uint_as_float(v[i]), __uint_as_float(v[i + 1]));
          mx1 = max3f(mx1, __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
        }
        mx = fmaxf(mx0, mx1) * sl;
      }
      const float m_new = fmaxf(m_run, mx);
      // lazy rescale: keep a stale max unless the new one exceeds it by 2^8
      const bool rescale = (j == 0) || (m_new > m_run + 8.0f);
      const float m_use = rescale ? m_new : m_run;
      const float alpha = (j == 0 || m_run == -INFINITY) ? 0.f : exp2f(m_run - m_use);
      const float m_ref = m_use == -INFINITY ? 0.f : m_use;
      // pass 2, per 64 keys: P = 2^(s*scale - m), half of the keys on the
      // MUFU unit and half with an FMA-pipe polynomial (masked keys give
      // exactly 0), packed bf16 pairs written over the S columns already read
      float sum0 = 0.f, sum1 = 0.f;
#pragma unroll 1
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t v[64];
        tmem_ld32(s_addr + hh * 64, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld32(s_addr + hh * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_ld_wait();
        if (!full_tile) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (hh * 64 + i > lim) v[i] = __float_as_uint(-INFINITY);
        }
        if constexpr (PACKED) {
          // scale and shift pairs with one f32x2 FMA; POLY of every 8 keys
          // through the packed polynomial on the FMA pipe, the rest on MUFU;
          // row sums as f32x2 adds of the unrounded values
          const uint64_t sl2 = f2pack(sl, sl), nm2 = f2pack(-m_ref, -m_ref);
          uint64_t s2a = f2pack(0.f, 0.f), s2b = s2a;
#pragma unroll
          for (int i = 0; i < 64; i += 8) {
            float x[8], e[8];
#pragma unroll
            for (int k = 0; k < 4; ++k)
              f2unpack(ffma2(f2pack(__uint_as_float(v[i + 2 * k]), __uint_as_float(v[i + 2 * k + 1])), sl2, nm2),
                       x[2 * k], x[2 * k + 1]);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const bool poly = (POLY == 4 && (k & 1)) || (POLY == 2 && (k & 3) == 3);
              if (!poly) e[k] = exp2f(x[k]);
            }
            if constexpr (POLY == 4) {
              exp2_poly2(x[1], x[3], e[1], e[3]);
              exp2_poly2(x[5], x[7], e[5], e[7]);
            } else if constexpr (POLY == 2) {
              exp2_poly2(x[3], x[7], e[3], e[7]);
            }
            if (POLY > 0 && !full_tile) {
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                const bool poly = (POLY == 4 && (k & 1)) || (POLY == 2 && (k & 3) == 3);
                if (poly && hh * 64 + i + k > lim) e[k] = 0.f;
              }
            }
            s2a = fadd2(s2a, f2pack(e[0], e[1]));
            s2b = fadd2(s2b, f2pack(e[2], e[3]));
            s2a = fadd2(s2a, f2pack(e[4], e[5]));
            s2b = fadd2(s2b, f2pack(e[6], e[7]));
#pragma unroll
            for (int k = 0; k < 4; ++k) v[i / 2 + k] = pack_bf16(e[2 * k], e[2 * k + 1]);
          }
          float a, b, c, d;
          f2unpack(s2a, a, b);
          f2unpack(s2b, c, d);
          sum0 += a + c;
          sum1 += b + d;
        } else {
#pragma unroll
          for (int i = 0; i < 64; i += 2) {
            const float e0 = exp2f(fmaf(__uint_as_float(v[i]), sl, -m_ref));
            const float e1 = exp2_fma(fmaf(__uint_as_float(v[i + 1]), sl, -m_ref));
            __nv_bfloat162 bb = __floats2bfloat162_rn(e0, e1);
            sum0 += __low2float(bb);
            sum1 += __high2float(bb);
            v[i / 2] = *reinterpret_cast<uint32_t*>(&bb);
          }
        }
        tmem_st32(s_addr + hh * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
      }
      // S_t(j) was issued after PV_t(j-1): O_t is complete up to j-1 and no
      // MMA touches it until P_t(j) is published (rescaled here, once the
      // scores are out of registers)
      if (__any_sync(0xffffffffu, rescale && j > 0)) {
#pragma unroll 1
        for (int c0 = 0; c0 < 128; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(o_addr + c0, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(o_addr + c0, o);
        }
      }
      if (tr0) fstamp(p, FTR_SOFTMAX, j);
      l_run = l_run * alpha + (sum0 + sum1);
      m_run = m_use;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
      if (tr0) fstamp(p, FTR_PARRIVE, j);
    }
    ok = __all_sync(0xffffffffu, ok);
    const bool write = r < rows;
    const size_t prow = static_cast<size_t>(row_base + t * BQ + r);
    if (nkt <= 0) {
      if (S > 1 && write) p.lse_part[(prow * p.num_heads + h) * S + z] = -INFINITY;
    } else if (ok && mbar_wait_warp(&o_done[t], static_cast<uint32_t>((nkt - 1) & 1), abort_flag, p.status,
                                    kStatusTimeoutTmemFull)) {
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.0f / l_run : 0.f;
      if (S > 1) {
        const size_t base = (prow * p.num_heads + h) * S + z;
        if (write) p.lse_part[base] = l_run > 0.f ? m_run + __log2f(l_run) : -INFINITY;
        float* orow = p.o_part + base * D;
#pragma unroll 1
        for (int c0 = 0; c0 < 128; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(o_addr + c0, o);
          tmem_ld_wait();
          if (write) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<float4*>(orow + c0 + i) =
                  make_float4(__uint_as_float(o[i]) * inv, __uint_as_float(o[i + 1]) * inv,
                              __uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
          }
        }
      } else {
        __nv_bfloat16* orow = p.out + prow * p.ldo + h * D;
#pragma unroll 1
        for (int c0 = 0; c0 < 128; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(o_addr + c0, o);
          tmem_ld_wait();
          if (write) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              uint4 w;
              w.x = pack_bf16(__uint_as_float(o[i + 0]) * inv, __uint_as_float(o[i + 1]) * inv);
              w.y = pack_bf16(__uint_as_float(o[i + 2]) * inv, __uint_as_float(o[i + 3]) * inv);
              w.z = pack_bf16(__uint_as_float(o[i + 4]) * inv, __uint_as_float(o[i + 5]) * inv);
              w.w = pack_bf16(__uint_as_float(o[i + 6]) * inv, __uint_as_float(o[i + 7]) * inv);
              *reinterpret_cast<uint4*>(orow + c0 + i) = w;
            }
          }
        }
      }
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

// Merge the key shares of split rows: out = sum_s 2^(lse_s - max) O_s / sum_s 2^(lse_s - max).
__global__ void fa_combine_kernel(const float* __restrict__ o_part, const float* __restrict__ lse_part, int S,
                                  int H, __nv_bfloat16* __restrict__ out, int ldo) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const size_t base = (static_cast<size_t>(row) * H + h) * S;
  float mx = -INFINITY;
  for (int s = 0; s < S; ++s) mx = fmaxf(mx, lse_part[base + s]);
  float num = 0.f, den = 0.f;
  if (mx != -INFINITY) {
    for (int s = 0; s < S; ++s) {
      const float lse = lse_part[base + s];
      if (lse == -INFINITY) continue;
      const float w = exp2f(lse - mx);
      den += w;
      num += o_part[(base + s) * D + d] * w;
    }
  }
  out[static_cast<size_t>(row) * ldo + h * D + d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
}

}  // namespace fa
}  // namespace ib200

using namespace ib200;

static long long* g_fa_trace = nullptr;

// Diagnostics: the next launches stamp CTA (0,0)'s pipeline events into
// trace[8 * 64] (clock64), or stop when trace is null.
extern "C" void ib_attn_prefill_set_trace(long long* trace) { g_fa_trace = trace; }

namespace {

struct FaOperand {
  const void* ptr;
  long long rows;  // rows addressable through the tensor map
  int ld;          // row stride (elements)
  int hs;          // column stride between heads (elements)
  int width;       // columns read per head (64 or 128)
  int heads;       // heads addressed (1 with hs == 0: shared)
};

bool fa_tmap(CUtensorMap* m, const FaOperand& o, int box_rows) {
  if (o.ptr == nullptr || (reinterpret_cast<uintptr_t>(o.ptr) & 15) != 0 || (o.ld % 8) != 0 || (o.hs % 8) != 0)
    return false;
  const long long cols = static_cast<long long>(o.heads - 1) * o.hs + o.width;
  if (cols > o.ld) return false;
  return cached_tmap_2d(m, o.ptr, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, o.rows, cols, o.ld, box_rows, 64);
}

// Softmax variant of the two-tile kernel: packed f32x2 arithmetic with 0
// (default), 2 or 4 of every 8 exponentials on the FMA-pipe polynomial
// (INFERA_FA_POLY), or scalar arithmetic (INFERA_FA_PACKED=0, for comparison).
// All on MUFU measured fastest: the softmax is bound by issue slots, and an
// exponential costs one MUFU issue against about six FMA-pipe issues (8192 x
// 8192 causal: 0.516 ms all on MUFU, 0.536 ms with 2 of 8 and 0.594 ms with
// 4 of 8 on the polynomial).
using Fa2Kernel = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
                           const CUtensorMap, const ib200::fa::Params);
Fa2Kernel fa2_variant() {
  using namespace ib200::fa;
  static const Fa2Kernel k = [] {
    const char* e = std::getenv("INFERA_FA_PACKED");
    if (e != nullptr && e[0] == '0') return static_cast<Fa2Kernel>(fa_prefill2_kernel<false, 4>);
    const char* pe = std::getenv("INFERA_FA_POLY");
    const int poly = pe != nullptr && *pe ? std::atoi(pe) : 0;
    if (poly == 0) return static_cast<Fa2Kernel>(fa_prefill2_kernel<true, 0>);
    if (poly == 2) return static_cast<Fa2Kernel>(fa_prefill2_kernel<true, 2>);
    return static_cast<Fa2Kernel>(fa_prefill2_kernel<true, 4>);
  }();
  return k;
}

template <bool EXT>
int fa_launch(const FaOperand& q, const FaOperand& k, const FaOperand& v, const FaOperand* qe, const FaOperand* ke,
              const int* tiles, int num_tiles, const int* q_start, const int* q_len, const int* ctx_len,
              const int* block_table, const int* bt_rows, int max_pages, int num_heads, int num_kv_heads,
              float scale, void* out, int ldo, int* status, int kv_splits, float* o_part, float* lse_part,
              int tile_rows, cudaStream_t stream) {
  using namespace ib200::fa;
  if (num_tiles <= 0 || q.rows <= 0) return 0;
  if (tile_rows != 128 && (EXT || tile_rows != 256)) return -1;
  if ((ldo % 8) != 0 || num_kv_heads <= 0 || num_heads % num_kv_heads != 0) return -1;
  if (kv_splits > 1 && (o_part == nullptr || lse_part == nullptr || (reinterpret_cast<uintptr_t>(o_part) & 15)))
    return -1;
  CUtensorMap tq, tk, tv, tqe, tke, tk8, tv8, tke8;
  if (!fa_tmap(&tq, q, 128) || !fa_tmap(&tk, k, 16) || !fa_tmap(&tv, v, 16)) return -2;
  if (!fa_tmap(&tk8, k, 128) || !fa_tmap(&tv8, v, 128)) return -2;
  if (EXT) {
    if (!fa_tmap(&tqe, *qe, 128) || !fa_tmap(&tke, *ke, 16) || !fa_tmap(&tke8, *ke, 128)) return -2;
  } else {
    tqe = tq;
    tke = tk;
    tke8 = tk8;
  }
  Params p;
  p.tiles = tiles;
  p.q_start = q_start;
  p.q_len = q_len;
  p.ctx_len = ctx_len;
  p.block_table = block_table;
  p.bt_rows = bt_rows;
  p.max_pages = max_pages;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.q_hs = q.hs;
  p.k_hs = k.hs;
  p.v_hs = v.hs;
  p.qe_hs = EXT ? qe->hs : 0;
  p.ke_hs = EXT ? ke->hs : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.status = status;
  p.trace = g_fa_trace;
  p.kv_splits = kv_splits > 1 ? kv_splits : 1;
  p.o_part = o_part;
  p.lse_part = lse_part;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(fa_prefill_kernel<EXT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes(EXT));
    if (!EXT) {
      cudaFuncSetAttribute(fa_prefill2_kernel<true, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2);
      cudaFuncSetAttribute(fa_prefill2_kernel<true, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2);
      cudaFuncSetAttribute(fa_prefill2_kernel<true, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2);
      cudaFuncSetAttribute(fa_prefill2_kernel<false, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2);
    }
    attr_set[dev] = true;
  }
  dim3 grid(num_heads, num_tiles, p.kv_splits);
  if (tile_rows == 256)
    launch_pdl(fa2_variant(), grid, NUM_THREADS, SMEM2, stream, tq, tk, tv, tk8, tv8, p);
  else
    launch_pdl(fa_prefill_kernel<EXT>, grid, NUM_THREADS, smem_bytes(EXT), stream, tq, tk, tv, tqe, tke, tk8, tv8, tke8, p);
  if (p.kv_splits > 1)
    fa_combine_kernel<<<dim3(static_cast<unsigned>(q.rows), num_heads), D, 0, stream>>>(
        o_part, lse_part, p.kv_splits, num_heads, static_cast<__nv_bfloat16*>(out), ldo);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

}  // namespace

// q: [T, ldq] bf16 with head h at columns [h*128, h*128+128).
// k_cache / v_cache: [num_slots, num_kv_heads*128] bf16.
// tiles: device int32 [num_tiles, 2] (seq, q_block of 128 rows), longest
// first; tile_rows 256: each entry covers blocks q_block and q_block + 1
// (two query tiles per CTA), 128: one block.
// kv_splits > 1: each tile's key tiles are shared out over that many CTAs
// whose partials (o_part fp32 [T*num_heads*kv_splits*128], lse_part
// [T*num_heads*kv_splits]) a combine kernel merges into out.
extern "C" int ib_attn_prefill(const void* q, int T, int ldq, const void* k_cache, const void* v_cache,
                               long long num_slots, const int* tiles, int num_tiles, const int* q_start,
                               const int* q_len, const int* ctx_len, const int* block_table, const int* bt_rows,
                               int max_pages,
                               int num_heads, int num_kv_heads, float scale, void* out, int ldo, int* status,
                               int kv_splits, float* o_part, float* lse_part, int tile_rows, cudaStream_t stream) {
  using namespace ib200::fa;
  if (T <= 0) return 0;
  const int kvw = num_kv_heads * D;
  const FaOperand fq{q, T, ldq, D, D, num_heads};
  const FaOperand fk{k_cache, num_slots, kvw, D, D, num_kv_heads};
  const FaOperand fv{v_cache, num_slots, kvw, D, D, num_kv_heads};
  return fa_launch<false>(fq, fk, fv, nullptr, nullptr, tiles, num_tiles, q_start, q_len, ctx_len, block_table,
                          bt_rows, max_pages, num_heads, num_kv_heads, scale, out, ldo, status, kv_splits, o_part,
                          lse_part, tile_rows, stream);
}

// Attention over 128 + 64 score dims (MLA prefill, not absorbed):
//   q  [T, ldq]:   head h's 128 nope dims at column h*q_hs
//   qe [T, ldqe]:  head h's 64 rope dims at column h*qe_hs
//   k  [rows, ldk]: key head g's 128 nope dims at column g*k_hs
//   ke [rows, ldke]: key head g's 64 rope dims at column g*ke_hs (0: shared)
//   v  [rows, ldv]: value head g's 128 dims at column g*v_hs
// k / ke / v rows are addressed through the block table like cache slots
// (page of 16 rows); out [T, ldo] gets head h at columns h*128.
extern "C" int ib_attn_prefill_ext(const void* q, int T, int ldq, int q_hs, const void* qe, int ldqe, int qe_hs,
                                   const void* k, int ldk, int k_hs, const void* ke, int ldke, int ke_hs,
                                   const void* v, int ldv, int v_hs, long long num_rows, const int* tiles,
                                   int num_tiles, const int* q_start, const int* q_len, const int* ctx_len,
                                   const int* block_table, const int* bt_rows, int max_pages, int num_heads,
                                   int num_kv_heads, float scale, void* out, int ldo, int* status,
                                   int kv_splits, float* o_part, float* lse_part, cudaStream_t stream) {
  using namespace ib200::fa;
  if (T <= 0) return 0;
  const FaOperand fq{q, T, ldq, q_hs, D, num_heads};
  const FaOperand fqe{qe, T, ldqe, qe_hs, 64, qe_hs == 0 ? 1 : num_heads};
  const FaOperand fk{k, num_rows, ldk, k_hs, D, num_kv_heads};
  const FaOperand fke{ke, num_rows, ldke, ke_hs, 64, ke_hs == 0 ? 1 : num_kv_heads};
  const FaOperand fv{v, num_rows, ldv, v_hs, D, num_kv_heads};
  return fa_launch<true>(fq, fk, fv, &fqe, &fke, tiles, num_tiles, q_start, q_len, ctx_len, block_table, bt_rows,
                         max_pages, num_heads, num_kv_heads, scale, out, ldo, status, kv_splits, o_part, lse_part,
                         128, stream);
}
