// Paged decode attention (one query token per sequence, GQA) on tcgen05.
//
// One CTA handles (sequence, KV head, KV split) and walks its share of the
// sequence in tiles of 128 keys (8 pages):
//   warp 0      TMA producer: K and V tiles page by page (16 rows x 64 dims
//               boxes) into a 3-stage ring
//   warp 1      MMA issuer:
//                 S^T[128 keys, 16]   = K_tile . Q^T        (A = K, K-major)
//                 O^T[128 dims, 16]   = V_tile^T . P        (A = V, MN-major)
//               the 16 columns are query-head slots (G <= 8 real heads of
//               the KV group, the rest zero)
//   warps 2..5  thread <-> key row for the softmax (max over keys through a
//               bounded mbarrier-based group barrier, one exp2 per head per key),
//               P into one of two shared-memory buffers; they also stage Q.
// O^T accumulates in TMEM across the tiles. The softmax keeps a running max
// per head and rescales O only when a tile's max exceeds it by more than
// 2^8 (lazy rescale: the thread <-> dim row multiplies its O^T row in
// TMEM), so a tile's softmax never waits for the previous tile's PV; the
// double-buffered P is only reused after the PV two tiles back.
// Split partials (output normalised by its own sum, LSE in log2 units) are
// merged by a combine kernel when a sequence is split.
//
// The kernel moves every K/V byte once with TMA and does almost no ALU work
// per byte, so it runs at HBM bandwidth. KV layout per layer:
// [num_slots, Hkv * 128] bf16, slot = page * 16 + offset.
//
// Reference parity: decode attention runs inside the reference's engines
// (vLLM / SGLang / AITER); there is no source in its tree to mirror.
#include "sm100.cuh"
#include "tma_host.h"

namespace ib200 {
namespace dtc {

constexpr int D = 128;
constexpr int BKV = 128;
constexpr int PAGE = 16;
constexpr int STAGES = 3;
constexpr int BLK = 128 * 128;      // 128 rows x 128 B: one 64-dim half of a 128-key tile
constexpr int NQ = 16;              // UMMA N (query-head slots)
constexpr int QBLK = NQ * 128;      // 16 rows x 128 B
constexpr int MAXG = 8;
constexpr int NUM_THREADS = 192;
constexpr int SMEM_BYTES = 1024 + STAGES * 4 * BLK + 6 * QBLK + 1024;
constexpr uint32_t TMEM_COLS = 64;  // S0 [0,16) S1 [16,32) O [32,48)
constexpr uint32_t O_COL = 32;
constexpr float kRescaleLog2 = 8.0f;  // lazy rescale threshold (log2 units)

struct Params {
  const __nv_bfloat16* q;
  int ldq;
  const int* block_table;
  const int* bt_rows;
  const int* seq_lens;
  int max_pages;
  int hq, hkv, G;
  int splits;
  float scale_log2;
  float* o_part;   // [B, hq, splits, D]
  float* lse_part; // [B, hq, splits]
  __nv_bfloat16* out;
  int ldo;
  int* status;
  // > 0: every split covers this many 128-key tiles starting at split *
  // tiles_per_split (the same absolute key range in every sequence, so the
  // CTAs that read a prefix shared by several sequences run together and
  // its pages are served from L2); 0: each sequence's tiles are divided
  // evenly over the splits
  int tiles_per_split;
  int l2_policy;   // K/V loads: 0 evict_first, 1 evict_normal, 2 evict_last
};

__device__ __forceinline__ uint32_t s_col(int j) { return (j & 1) ? 16u : 0u; }

// byte offset of element (row, k) of a 16-row K-major block pair
// [lo: k < 64 | hi: k >= 64] in the 128-byte-swizzled layout
__device__ __forceinline__ uint32_t qp_offset(int row, int k) {
  const int half = k >> 6, kk = k & 63;
  return static_cast<uint32_t>(half * QBLK + row * 128 + ((((kk >> 3) ^ (row & 7))) << 4) + (kk & 7) * 2);
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    decode_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                     const __grid_constant__ CUtensorMap tmK8, const __grid_constant__ CUtensorMap tmV8,
                     const Params p) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int G = p.G;
  const int len = p.seq_lens[b];
  const int n_tiles = (len + BKV - 1) / BKV;
  const int tps = p.tiles_per_split > 0 ? p.tiles_per_split : (n_tiles + p.splits - 1) / p.splits;
  const int t0 = split * tps;
  const int t1 = min(n_tiles, t0 + tps);
  if (t0 >= t1) {  // nothing in this split: mark it empty for the combine
    if (p.splits > 1) {
      if (threadIdx.x < G)
        p.lse_part[(static_cast<size_t>(b) * p.hq + kvh * G + threadIdx.x) * p.splits + split] = -INFINITY;
    } else {
      for (int i = threadIdx.x; i < G * D; i += blockDim.x)
        p.out[static_cast<size_t>(b) * p.ldo + kvh * G * D + i] = __float2bfloat16(0.f);
    }
    return;
  }
  const int nt = t1 - t0;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sKV = smem;                        // stage s: K lo, K hi, V lo, V hi
  uint8_t* sQ = smem + STAGES * 4 * BLK;      // Q lo, Q hi
  uint8_t* sP = sQ + 2 * QBLK;                // [2 buffers] P lo, P hi (rows = head slots, cols = keys)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 4 * QBLK);
  uint64_t* k_full = bars;
  uint64_t* v_full = k_full + STAGES;
  uint64_t* kv_empty = v_full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;       // [2]
  uint64_t* p_full = s_full + 2;              // [2] one per P buffer
  uint64_t* pv_done = p_full + 2;             // [2] PV of tile j commits to pv_done[j & 1]
  uint64_t* q_ready = pv_done + 2;
  uint64_t* grp = q_ready + 1;                // bounded barrier of the 128 softmax threads
  uint64_t* drain = grp + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(tmem_slot + 4);    // [2][4][MAXG]
  float* lred = red + 2 * 4 * MAXG;                         // [4][MAXG]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(&p_full[0], 128);
    mbar_init(&p_full[1], 128);
    mbar_init(&pv_done[0], 1);
    mbar_init(&pv_done[1], 1);
    mbar_init(q_ready, 128);
    mbar_init(grp, 128);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmK8);
    tma_prefetch_desc(&tmV8);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = p.l2_policy == 1 ? policy_evict_normal()
                                            : (p.l2_policy == 2 ? policy_evict_last() : policy_evict_first());
      const int bt_row = p.bt_rows != nullptr ? p.bt_rows[b] : b;
      const int* bt = p.block_table + static_cast<size_t>(bt_row) * p.max_pages;
      const int n_pages = (len + PAGE - 1) / PAGE;
      long long issued = 0;
      int nxt[8];
      load_tile_pages(bt, t0, n_pages, nxt);
      for (int j = 0; j < nt; ++j) {
        const int st = j % STAGES;
        int cur[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) cur[i] = nxt[i];
        if (j + 1 < nt) load_tile_pages(bt, t0 + j + 1, n_pages, nxt);  // in flight while we wait
        if (!mbar_wait(&kv_empty[st], static_cast<uint32_t>(((j / STAGES) & 1) ^ 1), abort_flag, p.status,
                       kStatusTimeoutEmpty))
          break;
        uint8_t* base = sKV + st * 4 * BLK;
        // eight consecutive pages are one 128-row box per half (the 128-byte
        // swizzle repeats every 8 rows, so the shared-memory image is the
        // same as eight page boxes)
        bool run = true;
#pragma unroll
        for (int pg = 1; pg < BKV / PAGE; ++pg) run = run && cur[pg] == cur[0] + pg;
        mbar_expect_tx(&k_full[st], 2 * BLK);
        if (run) {
          tma_load_2d(base, &tmK8, &k_full[st], kvh * D, cur[0] * PAGE, pol);
          tma_load_2d(base + BLK, &tmK8, &k_full[st], kvh * D + 64, cur[0] * PAGE, pol);
        } else {
#pragma unroll
          for (int pg = 0; pg < BKV / PAGE; ++pg) {
            const int row = cur[pg] * PAGE;
            tma_load_2d(base + pg * PAGE * 128, &tmK, &k_full[st], kvh * D, row, pol);
            tma_load_2d(base + BLK + pg * PAGE * 128, &tmK, &k_full[st], kvh * D + 64, row, pol);
          }
        }
        mbar_expect_tx(&v_full[st], 2 * BLK);
        if (run) {
          tma_load_2d(base + 2 * BLK, &tmV8, &v_full[st], kvh * D, cur[0] * PAGE, pol);
          tma_load_2d(base + 3 * BLK, &tmV8, &v_full[st], kvh * D + 64, cur[0] * PAGE, pol);
        } else {
#pragma unroll
          for (int pg = 0; pg < BKV / PAGE; ++pg) {
            const int row = cur[pg] * PAGE;
            tma_load_2d(base + 2 * BLK + pg * PAGE * 128, &tmV, &v_full[st], kvh * D, row, pol);
            tma_load_2d(base + 3 * BLK + pg * PAGE * 128, &tmV, &v_full[st], kvh * D + 64, row, pol);
          }
        }
        ++issued;
      }
      long long first = issued > STAGES ? issued - STAGES : 0;
      for (long long i = first; i < issued; ++i) {
        mbar_wait(&k_full[i % STAGES], static_cast<uint32_t>((i / STAGES) & 1), nullptr, nullptr, 0,
                  kWaitLimitNs / 4);
        mbar_wait(&v_full[i % STAGES], static_cast<uint32_t>((i / STAGES) & 1), nullptr, nullptr, 0,
                  kWaitLimitNs / 4);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc_bf16(128, NQ);
      const uint32_t idesc_o = make_idesc_bf16(128, NQ, false, true);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t p_addr = smem_u32(sP);
      bool ok = mbar_wait(q_ready, 0, abort_flag, p.status, kStatusTimeoutFull);
      tc_fence_after();
      auto issue_pv = [&](int jj) -> bool {
        const int st = jj % STAGES;
        if (!mbar_wait(&p_full[jj & 1], static_cast<uint32_t>((jj >> 1) & 1), abort_flag, p.status,
                       kStatusTimeoutTmemEmpty))
          return false;
        if (!mbar_wait(&v_full[st], static_cast<uint32_t>((jj / STAGES) & 1), abort_flag, p.status,
                       kStatusTimeoutFull))
          return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sKV + st * 4 * BLK + 2 * BLK);
        const uint32_t pb = p_addr + static_cast<uint32_t>((jj & 1) * 2 * QBLK);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          // A = V^T, MN-major: LBO = distance to the dims 64..127 block, SBO = 8 keys
          const uint64_t ad = make_sw128_desc(v_addr + s * 2048, BLK, 1024);
          const uint64_t bd = make_sw128_desc(pb + (s < 4 ? s * 32 : QBLK + (s - 4) * 32), 16, 1024);
          umma_bf16(tmem + O_COL, ad, bd, idesc_o, (jj > 0 || s > 0) ? 1u : 0u);
        }
        umma_commit(&pv_done[jj & 1]);
        umma_commit(&kv_empty[st]);
        return true;
      };
      for (int j = 0; j < nt && ok; ++j) {
        const int st = j % STAGES;
        if (!mbar_wait(&k_full[st], static_cast<uint32_t>((j / STAGES) & 1), abort_flag, p.status,
                       kStatusTimeoutFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sKV + st * 4 * BLK);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint64_t ad = make_sw128_desc(k_addr + (s < 4 ? s * 32 : BLK + (s - 4) * 32), 16, 1024);
          const uint64_t bd = make_sw128_desc(q_addr + (s < 4 ? s * 32 : QBLK + (s - 4) * 32), 16, 1024);
          umma_bf16(tmem + s_col(j), ad, bd, idesc_s, s > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[j & 1]);
        if (j > 0 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) issue_pv(nt - 1);
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, p.status, kStatusTimeoutFull);
    }
  } else {
    const int t = threadIdx.x - 64;   // 0..127
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;     // key row of S, dim row of O
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    // Barrier of the four softmax warps built on an mbarrier so that every
    // wait stays bounded (a warp that gave up cannot strand the others).
    uint32_t gph = 0;
    bool ok = true;
    auto group_sync = [&]() {
      mbar_arrive(grp);
      ok = mbar_wait_warp(grp, gph & 1u, abort_flag, p.status, kStatusTimeoutTmemFull) && ok;
      ++gph;
    };
    // stage Q (head slots >= G and both P buffers start at zero)
    for (int i = t; i < 6 * QBLK / 16; i += 128) reinterpret_cast<uint4*>(sQ)[i] = make_uint4(0, 0, 0, 0);
    group_sync();
    for (int idx = t; idx < G * 64; idx += 128) {
      const int h = idx >> 6, d = (idx & 63) * 2;
      const uint32_t v =
          *reinterpret_cast<const uint32_t*>(p.q + static_cast<size_t>(b) * p.ldq + (kvh * G + h) * D + d);
      *reinterpret_cast<uint32_t*>(sQ + qp_offset(h, d)) = v;
    }
    fence_proxy_async_smem();
    mbar_arrive(q_ready);

    float m_run[MAXG], l_part[MAXG], acc[MAXG];
#pragma unroll
    for (int h = 0; h < MAXG; ++h) {
      m_run[h] = -INFINITY;
      l_part[h] = 0.f;
      acc[h] = 0.f;
    }
    // wait until the PV of tile jj has completed (its commit is the
    // ((jj >> 1) + 1)-th completion of pv_done[jj & 1]; no later PV on that
    // barrier can have been issued yet when this is called)
    auto wait_pv = [&](int jj) -> bool {
      if (!mbar_wait_warp(&pv_done[jj & 1], static_cast<uint32_t>((jj >> 1) & 1), abort_flag, p.status,
                          kStatusTimeoutTmemFull))
        return false;
      tc_fence_after();
      return true;
    };
    for (int j = 0; j < nt && ok; ++j) {
      if (!mbar_wait_warp(&s_full[j & 1], static_cast<uint32_t>((j >> 1) & 1), abort_flag, p.status,
                          kStatusTimeoutTmemFull)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[16];
      tmem_ld16(lane_addr + s_col(j), sv);
      tmem_ld_wait();
      const bool valid = (t0 + j) * BKV + r < len;
      float s[MAXG];
#pragma unroll
      for (int h = 0; h < MAXG; ++h) {
        s[h] = (valid && h < G) ? __uint_as_float(sv[h]) * p.scale_log2 : -INFINITY;
        float mx = s[h];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red[((j & 1) * 4 + q4) * MAXG + h] = mx;
      }
      group_sync();
      if (!ok) break;
      // new running maxima; every thread derives the same values from red,
      // so the rescale decision below is uniform over the CTA
      float alpha[MAXG];
      bool any_rescale = false;
#pragma unroll
      for (int h = 0; h < MAXG; ++h) {
        const float* rr = red + (j & 1) * 4 * MAXG;
        const float tmax = fmaxf(fmaxf(rr[h], rr[MAXG + h]), fmaxf(rr[2 * MAXG + h], rr[3 * MAXG + h]));
        alpha[h] = 1.f;
        if (m_run[h] == -INFINITY) {
          m_run[h] = tmax;                       // first keys of this head: nothing accumulated yet
        } else if (tmax > m_run[h] + kRescaleLog2) {
          alpha[h] = exp2f(m_run[h] - tmax);
          m_run[h] = tmax;
          any_rescale = true;
        }
      }
      if (any_rescale) {
        // O^T holds every earlier tile: once the last PV landed, scale each
        // rescaled head's column (this thread owns dim row r)
        if (!wait_pv(j - 1)) {
          ok = false;
          break;
        }
        uint32_t ov[16];
        tmem_ld16(lane_addr + O_COL, ov);
        tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < MAXG; ++h) ov[h] = __float_as_uint(__uint_as_float(ov[h]) * alpha[h]);
        tmem_st16(lane_addr + O_COL, ov);
        tmem_st_wait();
      }
      float pj[MAXG];
#pragma unroll
      for (int h = 0; h < MAXG; ++h) {
        pj[h] = (s[h] == -INFINITY || m_run[h] == -INFINITY) ? 0.f : exp2f(s[h] - m_run[h]);
        l_part[h] = l_part[h] * alpha[h] + pj[h];
      }
      // P buffer j & 1 was last read by the PV of tile j - 2
      if (j >= 2 && !wait_pv(j - 2)) {
        ok = false;
        break;
      }
      uint8_t* pbuf = sP + (j & 1) * 2 * QBLK;
#pragma unroll
      for (int h = 0; h < MAXG; ++h)
        if (h < G) *reinterpret_cast<__nv_bfloat16*>(pbuf + qp_offset(h, r)) = __float2bfloat16(pj[h]);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[j & 1]);
    }
    ok = __all_sync(0xffffffffu, ok);
    if (ok && wait_pv(nt - 1)) {
      uint32_t ov[16];
      tmem_ld16(lane_addr + O_COL, ov);
      tmem_ld_wait();
#pragma unroll
      for (int h = 0; h < MAXG; ++h) acc[h] = __uint_as_float(ov[h]);
    }
    // softmax denominators: sum of the per-key partials over the 128 rows
#pragma unroll
    for (int h = 0; h < MAXG; ++h) {
      float v = l_part[h];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) lred[q4 * MAXG + h] = v;
    }
    group_sync();
#pragma unroll
    for (int h = 0; h < MAXG; ++h) {
      if (h >= G || !ok) break;
      const float l = lred[h] + lred[MAXG + h] + lred[2 * MAXG + h] + lred[3 * MAXG + h];
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int head = kvh * G + h;
      if (p.splits == 1) {
        p.out[static_cast<size_t>(b) * p.ldo + head * D + r] = __float2bfloat16(acc[h] * inv);
      } else {
        const size_t slot = (static_cast<size_t>(b) * p.hq + head) * p.splits + split;
        p.o_part[slot * D + r] = acc[h] * inv;
        if (r == 0) p.lse_part[slot] = l > 0.f ? m_run[h] + log2f(l) : -INFINITY;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// o = sum_s 2^(lse_s - M) o_s / sum_s 2^(lse_s - M)
__global__ void combine_kernel(const Params p) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const size_t base = (static_cast<size_t>(b) * p.hq + h) * p.splits;
  float mx = -INFINITY;
  for (int s = 0; s < p.splits; ++s) mx = fmaxf(mx, p.lse_part[base + s]);
  float num = 0.f, den = 0.f;
  if (mx != -INFINITY) {
    for (int s = 0; s < p.splits; ++s) {
      const float lse = p.lse_part[base + s];
      if (lse == -INFINITY) continue;
      const float w = exp2f(lse - mx);
      den += w;
      num += p.o_part[(base + s) * D + d] * w;
    }
  }
  p.out[static_cast<size_t>(b) * p.ldo + h * D + d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
}

}  // namespace dtc
}  // namespace ib200

using namespace ib200;

// q [B, ldq] bf16 (head h at columns h*128); caches [num_slots, hkv*128];
// block_table [rows, max_pages] with bt_rows[b] (null: row b);
// o_part / lse_part: fp32 scratch of B*hq*splits*128 / B*hq*splits (only
// touched when splits > 1).
// tiles_per_split > 0: split s covers tiles [s * tiles_per_split, +tiles_per_split)
// of every sequence (splits * tiles_per_split * 128 must cover the longest
// sequence); l2_policy: 0 evict_first, 1 evict_normal, 2 evict_last for K/V.
extern "C" int ib_attn_decode_tc_ex(const void* q, int ldq, const void* k_cache, const void* v_cache,
                                    long long num_slots, const int* block_table, const int* bt_rows,
                                    const int* seq_lens, int max_pages, int B, int hq, int hkv, int splits,
                                    float scale, float* o_part, float* lse_part, void* out, int ldo, int* status,
                                    int tiles_per_split, int l2_policy, cudaStream_t stream) {
  using namespace ib200::dtc;
  if (B <= 0) return 0;
  if (hkv <= 0 || hq % hkv != 0 || hq / hkv > MAXG || splits < 1 || (ldq % 2) != 0) return -1;
  if (splits > 1 && (o_part == nullptr || lse_part == nullptr)) return -1;
  const int kvw = hkv * D;
  CUtensorMap tk, tv, tk8, tv8;
  if (!cached_tmap_2d(&tk, k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, num_slots, kvw, kvw, 16, 64)) return -2;
  if (!cached_tmap_2d(&tv, v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, num_slots, kvw, kvw, 16, 64)) return -2;
  if (!cached_tmap_2d(&tk8, k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, num_slots, kvw, kvw, 128, 64)) return -2;
  if (!cached_tmap_2d(&tv8, v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, num_slots, kvw, kvw, 128, 64)) return -2;
  Params p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.ldq = ldq;
  p.block_table = block_table;
  p.bt_rows = bt_rows;
  p.seq_lens = seq_lens;
  p.max_pages = max_pages;
  p.hq = hq;
  p.hkv = hkv;
  p.G = hq / hkv;
  p.splits = splits;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o_part = o_part;
  p.lse_part = lse_part;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.status = status;
  p.tiles_per_split = tiles_per_split;
  p.l2_policy = l2_policy;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(decode_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    attr_set[dev] = true;
  }
  dim3 grid(B, hkv, splits);
  launch_pdl(decode_tc_kernel, grid, NUM_THREADS, SMEM_BYTES, stream, tk, tv, tk8, tv8, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return static_cast<int>(e);
  if (splits > 1) {
    launch_pdl(combine_kernel, dim3(B, hq), D, 0, stream, p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return 0;
}

extern "C" int ib_attn_decode_tc(const void* q, int ldq, const void* k_cache, const void* v_cache, long long num_slots,
                                 const int* block_table, const int* bt_rows, const int* seq_lens, int max_pages, int B,
                                 int hq, int hkv, int splits, float scale, float* o_part, float* lse_part, void* out,
                                 int ldo, int* status, cudaStream_t stream) {
  return ib_attn_decode_tc_ex(q, ldq, k_cache, v_cache, num_slots, block_table, bt_rows, seq_lens, max_pages, B, hq,
                              hkv, splits, scale, o_part, lse_part, out, ldo, status, 0, 0, stream);
}
