// bf16 GEMM on the 5th-generation tensor cores (tcgen05 / TMEM / TMA).
//
//   C[M, N] = A[M, K] . W[N, K]^T        (nn.Linear layout, both K-major)
//
// Persistent, warp-specialised kernel, one CTA per SM:
//   warp 0      TMA producer (one elected lane) -> 4-deep (fp8: 5-deep) smem ring
//   warp 1      TMEM allocator + MMA issuer (one elected lane)
//   warps 2..5  epilogue: tcgen05.ld -> registers -> global
// Two TMEM accumulators (2 x 256 fp32 columns) let the epilogue of tile i
// overlap the main loop of tile i+1.
//
// Two operand orders:
//   normal  : UMMA M = 128 tokens,       UMMA N = 256 output features
//   swap-AB : UMMA M = 128 out features, UMMA N = tokens rounded up to 16
// Swap-AB is the decode shape (few tokens): the weight streams through the
// 128-row side and every SM keeps HBM busy. Small tile counts are split along
// K; split partials are reduced with fp32 vector atomics into a zeroed
// workspace and a finalize kernel converts (and re-zeroes the workspace).
//
// Epilogues: plain bf16 store, or SwiGLU on row-interleaved (gate, up)
// weights (row 2j = gate_j, row 2j+1 = up_j) writing silu(g)*u.
//
// fp8 (W8A8, e4m3) instantiation: the same pipeline with one 128-byte
// stage = 128 K elements, issued as kind::mxf8f6f4.block_scale MMAs. Weights
// carry one UE8M0 scale per 128x128 block and activations one per token and
// 128-wide K group; the tensor core applies them per 32-wide K chunk, so no
// promotion pass is needed. Four extra warps (6..9, one per TMEM lane
// quadrant) stage each pipeline stage's scale factors into TMEM with
// tcgen05.st: the weight block's byte in 4 columns, the tile's token scales
// in 8 columns (token r at lane r % 32, column r / 32, replicated in every
// lane quadrant). fp8 always runs swap-AB (UMMA M = 128 output features,
// UMMA N = up to 192 tokens, a multiple of 32); TMEM holds two 192-column
// accumulators and four 16-column scale slots.
//
// Reference parity: the reference delegates all GEMMs to its engines
// (vLLM/hipBLASLt); there is no GEMM source in it to mirror.
#include <cstdlib>

#include "sm100.cuh"
#include "tma_host.h"

namespace ib200 {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // one 128-byte swizzle atom of bf16
constexpr int STAGES = 4;
constexpr int MAX_BN = 256;
constexpr int P_STAGE = BM * BK * 2;      // 16 KiB
constexpr int Q_STAGE = MAX_BN * BK * 2;  // 32 KiB
constexpr int NUM_THREADS = 192;
constexpr int TMEM_COLS = 512;
constexpr int STAGES_FP8 = 5;                  // shorter MMA time per byte: a deeper ring
constexpr int Q_STAGE_FP8 = 192 * 128;         // 192 token rows x 128 e4m3
constexpr int SMEM_BF16 = STAGES * (P_STAGE + Q_STAGE);
constexpr int SMEM_FP8 = STAGES_FP8 * (P_STAGE + Q_STAGE_FP8);
constexpr int SMEM_BYTES = 1024 + (SMEM_BF16 > SMEM_FP8 ? SMEM_BF16 : SMEM_FP8) + 256;
constexpr int NUM_THREADS_FP8 = 320;
constexpr int MAX_BN_FP8 = 192;
constexpr int BK_FP8 = 128;           // one 128-byte swizzle atom of e4m3
constexpr int SF_COL0 = 2 * MAX_BN_FP8;  // scale slots after the accumulators
constexpr int SF_SLOT = 16;              // per stage: A scales at +0 (4), B at +8 (8)
// Small token tiles (bn <= 64, decode-size GEMMs that stream the weights):
// Q slots of 64 rows let the same shared memory hold an 8-deep ring, which
// keeps more weight bytes in flight per SM. fp8 scale slots then end at
// TMEM column SF_COL0 + 8 * SF_SLOT = 512.
constexpr int DEEP_BN = 64;
constexpr int STAGES_DEEP = 8;
constexpr int Q_STAGE_DEEP = DEEP_BN * 128;   // 64 rows x 128 bytes (bf16 or e4m3 K atom)
static_assert(STAGES_DEEP * (P_STAGE + Q_STAGE_DEEP) <= (SMEM_BF16 > SMEM_FP8 ? SMEM_BF16 : SMEM_FP8),
              "the deep ring fits the shared memory the kernel is launched with");
static_assert(SF_COL0 + STAGES_DEEP * SF_SLOT <= TMEM_COLS, "fp8 scale slots of the deep ring fit in TMEM");

enum Epi : int { EPI_BF16 = 0, EPI_SWIGLU = 1, EPI_ATOMIC_F32 = 2 };
constexpr int kMaxPeers = 8;

struct Params {
  int M, N, K;      // logical problem: tokens, features (pre-activation), reduction
  int bn;           // UMMA N
  int p_tiles, q_tiles, splits, kbps, nkb;
  int swap;         // 1: P = W (features), Q = A (tokens)
  int epi;
  void* out;        // bf16 [M, ldc] or fp32 [M, N] workspace
  int ldc;
  int* status;
  // push mode (world >= 2, EPI_BF16 only): every output tile is stored to
  // world destinations (this rank's receive slot on every rank, peers over
  // NVLink), then the last CTA bumps one arrival counter on every rank
  int push;
  int world;
  void* peer_out[kMaxPeers];
  unsigned int* peer_flag[kMaxPeers];
  unsigned int* done_ctr;   // local, zero between launches
  int push_owner;           // 1: a tile of token rows goes only to rank (row block % world) (reduce-scatter)
  long long* trace;         // optional: clock64 stamps of CTA 0's pipeline events (TRG_*)
  // grouped mode (MoE experts, swap-AB only): tile t = gtab[t] = {expert,
  // feature tile, first token row, end token row of the expert}; *gnum tiles
  int grouped;
  const int4* gtab;
  const int* gnum;
  int n_per_expert;         // weight rows per expert (the grouped GEMM's N)
  // grouped push (expert-parallel return fused into the epilogue): output
  // row m goes to rank row_map[m] >> 27, row row_map[m] & (2^27 - 1) of
  // peer_out[rank]; then every rank's peer_flag is bumped once (push = 1)
  const int* row_map;
  // fp8: UE8M0 scale bytes. sf_w [ceil(rows of W / 128), sf_w_ld] (one per
  // 128x128 weight block); sf_a [K / 128, sf_a_ld] (K-group-major, one per
  // token and 128-wide K group)
  const uint8_t* sf_w;
  const uint8_t* sf_a;
  int sf_w_ld, sf_a_ld;
  // optional: the A rows (and fp8 scales) are being stored into this rank's
  // memory by other GPUs (expert-parallel dispatch); their readers wait,
  // bounded, until *wait_flag >= wait_target before the first read
  const unsigned int* wait_flag;
  unsigned int wait_target;
  uint64_t wait_limit_ns;   // bound of that wait (0: kWaitLimitNs)
  int wait_per_expert;      // grouped: wait_flag[e] per local expert, waited before each of e's tiles
  int streamk;              // each CTA takes an equal share of the (tile, k-block) steps of tiles
                            // [dp_tiles, total) (fp32 atomic epilogue), after whole tiles blockIdx.x,
                            // +gridDim.x below dp_tiles written directly (epi_dp into out_dp)
  int dp_tiles;
  int epi_dp;
  void* out_dp;
  // optional: per-tile counters of k-blocks accumulated into the workspace
  // (zero between launches); the CTA whose share completes a tile reads the
  // tile back, stores it (epi_dp into out_dp) and re-zeroes it, so no
  // finalize kernel runs
  unsigned int* tile_ctr;
};

// Bounded wait for the dispatch's arrival counter (release-incremented by
// each sender after its stores). On success the generic-proxy view is
// ordered before this thread's later TMA (async-proxy) reads; on timeout the
// status is recorded and the CTA's other roles are released through
// abort_flag.
__device__ __forceinline__ bool wait_arrivals(const Params& p, volatile int* abort_flag, int expert = 0) {
  if (p.wait_flag == nullptr) return true;
  const unsigned int* flag = p.wait_flag + (p.wait_per_expert ? expert : 0);
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v >= p.wait_target) break;
    if (((++spins) & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > (p.wait_limit_ns ? p.wait_limit_ns : kWaitLimitNs)) {
        record_status(p.status, kStatusTimeoutPeer);
        *abort_flag = 1;
        return false;
      }
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// pipeline event stamps of CTA 0 (trace[event * kTraceSteps + k-step]) for diagnosis
enum : int { TRG_TMA = 0, TRG_FULL, TRG_SFFULL, TRG_ISSUED, TRG_SFARRIVE, kTraceEventsG };
constexpr int kTraceSteps = 128;

__device__ __forceinline__ void gstamp(const Params& p, int ev, long long i) {
  if (p.trace != nullptr && blockIdx.x == 0 && i < kTraceSteps) p.trace[ev * kTraceSteps + i] = clock64();
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ void tile_coords(const Params& p, int t, int& pt, int& qt, int& sp) {
  if (p.grouped) {
    pt = t;
    qt = 0;
    sp = 0;
    return;
  }
  sp = t % p.splits;
  int rest = t / p.splits;
  if (p.swap) {  // the token tiles of one weight tile run back to back (the weight tile read once)
    qt = rest % p.q_tiles;
    pt = rest / p.q_tiles;
  } else {       // the row blocks of one weight block run back to back
    pt = rest % p.p_tiles;
    qt = rest / p.p_tiles;
  }
}

// The (tile, k-block range) segments one CTA works through, in order: tiles
// blockIdx.x, +gridDim.x with their split-K share, or (stream-K) one equal
// contiguous share of all tiles x k-blocks, cut at tile boundaries. Every
// role walks the same sequence.
struct SegIter {
  long long k, hi;
  int t;
};

__device__ __forceinline__ void seg_begin(const Params& p, int total, SegIter& it) {
  it.t = blockIdx.x;
  if (p.streamk) {
    const long long all = static_cast<long long>(total - p.dp_tiles) * p.nkb;
    it.k = all * blockIdx.x / gridDim.x;
    it.hi = all * (blockIdx.x + 1) / gridDim.x;
  }
}

__device__ __forceinline__ bool seg_next(const Params& p, int total, SegIter& it, int& t, int& kb0, int& kb1) {
  if (p.streamk) {
    if (it.t < p.dp_tiles) {  // whole tiles first (full waves), written directly
      t = it.t;
      it.t += gridDim.x;
      kb0 = 0;
      kb1 = p.nkb;
      return true;
    }
    if (it.k >= it.hi) return false;
    t = p.dp_tiles + static_cast<int>(it.k / p.nkb);
    kb0 = static_cast<int>(it.k % p.nkb);
    kb1 = static_cast<int>(min(static_cast<long long>(p.nkb), kb0 + (it.hi - it.k)));
    it.k += kb1 - kb0;
    return true;
  }
  if (it.t >= total) return false;
  t = it.t;
  it.t += gridDim.x;
  int pt, qt, sp;
  tile_coords(p, t, pt, qt, sp);
  kb0 = sp * p.kbps;
  kb1 = min(kb0 + p.kbps, p.nkb);
  return true;
}

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// Epilogue for a chunk of `ncols` accumulator columns starting at `c0`.
// `r` holds this thread's row of the chunk (row = TMEM lane).
template <int NC>
__device__ __forceinline__ void store_chunk(const Params& p, int pt, int qt, int row, int c0,
                                            const uint32_t (&r)[NC], bool dp) {
  // dp: a whole tile of a stream-K run, stored directly
  const int epi = dp ? p.epi_dp : p.epi;
  void* const out = dp ? p.out_dp : p.out;
  if (!p.swap) {
    const int m = pt * BM + row;
    const int n0 = qt * p.bn + c0;
    if (epi == EPI_BF16) {
      if (m >= p.M) return;
      const int nout = p.push ? p.world : 1;
      for (int d = 0; d < nout; ++d) {
        if (p.push && p.push_owner && d != pt % p.world) continue;
        void* base = p.push ? p.peer_out[d] : out;
        __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(base) + static_cast<size_t>(m) * p.ldc + n0;
        if (n0 + NC <= p.N && (p.ldc & 7) == 0) {
#pragma unroll
          for (int j = 0; j < NC; j += 8) {
            uint4 v;
            v.x = pack_bf16(__uint_as_float(r[j + 0]), __uint_as_float(r[j + 1]));
            v.y = pack_bf16(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
            v.z = pack_bf16(__uint_as_float(r[j + 4]), __uint_as_float(r[j + 5]));
            v.w = pack_bf16(__uint_as_float(r[j + 6]), __uint_as_float(r[j + 7]));
            *reinterpret_cast<uint4*>(C + j) = v;
          }
        } else {
#pragma unroll
          for (int j = 0; j < NC; ++j)
            if (n0 + j < p.N) C[j] = __float2bfloat16(__uint_as_float(r[j]));
        }
      }
    } else if (epi == EPI_SWIGLU) {
      if (m >= p.M) return;
      __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(out) + static_cast<size_t>(m) * p.ldc + n0 / 2;
      if (n0 + NC <= p.N && (p.ldc & 7) == 0) {
#pragma unroll
        for (int j = 0; j < NC; j += 16) {
          float o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            o[i] = silu(__uint_as_float(r[j + 2 * i])) * __uint_as_float(r[j + 2 * i + 1]);
          uint4 v;
          v.x = pack_bf16(o[0], o[1]);
          v.y = pack_bf16(o[2], o[3]);
          v.z = pack_bf16(o[4], o[5]);
          v.w = pack_bf16(o[6], o[7]);
          *reinterpret_cast<uint4*>(C + j / 2) = v;
        }
      } else {
#pragma unroll
        for (int j = 0; j < NC; j += 2)
          if (n0 + j + 1 < p.N)
            C[j / 2] = __float2bfloat16(silu(__uint_as_float(r[j])) * __uint_as_float(r[j + 1]));
      }
    } else {
      if (m >= p.M) return;
      float* W = reinterpret_cast<float*>(out) + static_cast<size_t>(m) * p.N + n0;
      if (n0 + NC <= p.N && (p.N & 3) == 0) {
#pragma unroll
        for (int j = 0; j < NC; j += 4)
          red_add_v4(W + j, __uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                     __uint_as_float(r[j + 3]));
      } else {
#pragma unroll
        for (int j = 0; j < NC; ++j)
          if (n0 + j < p.N) atomicAdd(W + j, __uint_as_float(r[j]));
      }
    }
  } else {
    // swap-AB: row = output feature, columns = tokens
    const int n = pt * BM + row;
    const int m0 = qt * p.bn + c0;
    if (epi == EPI_BF16) {
      if (n >= p.N) return;
      const int nout = p.push ? p.world : 1;
      for (int d = 0; d < nout; ++d) {
        __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(p.push ? p.peer_out[d] : out) + n;
#pragma unroll
        for (int j = 0; j < NC; ++j)
          if (m0 + j < p.M && !(p.push && p.push_owner && d != ((m0 + j) >> 7) % p.world))
            C[static_cast<size_t>(m0 + j) * p.ldc] = __float2bfloat16(__uint_as_float(r[j]));
      }
    } else if (epi == EPI_SWIGLU) {
      // lanes 2j / 2j+1 hold gate_j / up_j for the same tokens
      const bool even = (threadIdx.x & 1) == 0;
      __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(out) + n / 2;
#pragma unroll
      for (int j = 0; j < NC; ++j) {
        float mine = __uint_as_float(r[j]);
        float other = __shfl_xor_sync(0xffffffffu, mine, 1);
        if (even && n + 1 < p.N && m0 + j < p.M)
          C[static_cast<size_t>(m0 + j) * p.ldc] = __float2bfloat16(silu(mine) * other);
      }
    } else {
      if (n >= p.N) return;
      float* W = reinterpret_cast<float*>(out) + n;
#pragma unroll
      for (int j = 0; j < NC; ++j)
        if (m0 + j < p.M) atomicAdd(W + static_cast<size_t>(m0 + j) * p.N, __uint_as_float(r[j]));
    }
  }
}

// The tile's reduced fp32 sums, read back from the workspace by the CTA
// that completed it (and zeroed there), stored like a whole tile.
template <int NC>
__device__ __forceinline__ void finish_chunk(const Params& p, int pt, int qt, int row, int c0) {
  float* ws = reinterpret_cast<float*>(p.out);
  uint32_t r[NC];
  if (p.swap) {
    const int n = pt * BM + row;
    const int m0 = qt * p.bn + c0;
#pragma unroll
    for (int j = 0; j < NC; ++j) {
      float v = 0.f;
      if (n < p.N && m0 + j < p.M) {
        float* a = ws + static_cast<size_t>(m0 + j) * p.N + n;
        v = __ldcg(a);
        __stcg(a, 0.f);
      }
      r[j] = __float_as_uint(v);
    }
  } else {
    const int m = pt * BM + row;
    const int n0 = qt * p.bn + c0;
#pragma unroll
    for (int j = 0; j < NC; ++j) {
      float v = 0.f;
      if (m < p.M && n0 + j < p.N) {
        float* a = ws + static_cast<size_t>(m) * p.N + n0 + j;
        v = __ldcg(a);
        __stcg(a, 0.f);
      }
      r[j] = __float_as_uint(v);
    }
  }
  store_chunk<NC>(p, pt, qt, row, c0, r, true);
}

// Grouped-mode epilogue (swap-AB): TMEM lane = feature of the expert,
// columns = that expert's token rows [m0, mend).
template <int NC>
__device__ __forceinline__ void store_chunk_grouped(const Params& p, int t, int row, int c0, const uint32_t (&r)[NC]) {
  const int4 g = p.gtab[t];
  const int n = g.y * BM + row;
  const int m0 = g.z + c0;
  if (p.epi == EPI_SWIGLU) {
    const bool even = (threadIdx.x & 1) == 0;
    __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(p.out) + n / 2;
#pragma unroll
    for (int j = 0; j < NC; ++j) {
      const float mine = __uint_as_float(r[j]);
      const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
      if (even && n + 1 < p.n_per_expert && m0 + j < g.w)
        C[static_cast<size_t>(m0 + j) * p.ldc] = __float2bfloat16(silu(mine) * other);
    }
  } else if (p.row_map != nullptr) {
    if (n >= p.n_per_expert) return;
#pragma unroll
    for (int j = 0; j < NC; ++j) {
      if (m0 + j < g.w) {
        const int code = __ldg(p.row_map + m0 + j);
        __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(p.peer_out[code >> 27]);
        C[static_cast<size_t>(code & 0x7FFFFFF) * p.ldc + n] = __float2bfloat16(__uint_as_float(r[j]));
      }
    }
  } else {
    if (n >= p.n_per_expert) return;
    __nv_bfloat16* C = reinterpret_cast<__nv_bfloat16*>(p.out) + n;
#pragma unroll
    for (int j = 0; j < NC; ++j)
      if (m0 + j < g.w) C[static_cast<size_t>(m0 + j) * p.ldc] = __float2bfloat16(__uint_as_float(r[j]));
  }
}

__device__ __forceinline__ int tile_prow(const Params& p, int t, int pt) {
  if (p.grouped) {
    const int4 g = p.gtab[t];
    return g.x * p.n_per_expert + g.y * BM;
  }
  return pt * BM;
}

__device__ __forceinline__ int tile_qrow(const Params& p, int t, int qt) {
  return p.grouped ? p.gtab[t].z : qt * p.bn;
}

// DEEP: the 8-deep ring with 64-row Q slots (launched only when p.bn <= DEEP_BN)
template <bool FP8, bool DEEP>
__global__ void __launch_bounds__(FP8 ? NUM_THREADS_FP8 : NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmQ,
                const Params p) {
  constexpr int kBK = FP8 ? BK_FP8 : BK;          // K elements per stage (128 bytes per row)
  constexpr int kAccCols = FP8 ? MAX_BN_FP8 : MAX_BN;
  constexpr int kStages = DEEP ? STAGES_DEEP : (FP8 ? STAGES_FP8 : STAGES);
  constexpr int kQStage = DEEP ? Q_STAGE_DEEP : (FP8 ? Q_STAGE_FP8 : Q_STAGE);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sP = smem;
  uint8_t* sQ = smem + kStages * P_STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sQ + kStages * kQStage);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* tfull = bars + 2 * kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* sf_full = drain + 1;  // fp8: scale factors of a stage are in TMEM
  uint64_t* ebar = sf_full + kStages;    // the 4 epilogue warps (in-kernel split reduction)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ebar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* s_last = abort_flag + 1;  // epilogue: this CTA completed the tile

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // PDL: let the next kernel be scheduled once every CTA got here. A
  // grouped run reads device data of earlier kernels from the start (tile
  // table, tile count) and waits for them at once; a dense run lets its
  // producer put the first stages' weight tiles (static data) in flight
  // before it waits (every other thread waits right after the setup).
  pdl_trigger();
  const bool early_weights = !p.grouped;
  if (!early_weights) pdl_wait();
  const int total = p.grouped ? *p.gnum : p.p_tiles * p.q_tiles * p.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    mbar_init(ebar, 128);
    if (FP8)
      for (int s = 0; s < kStages; ++s) mbar_init(&sf_full[s], 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmP);
    tma_prefetch_desc(&tmQ);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (early_weights && !(warp == 0 && lane == 0)) pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_act = policy_evict_last();
      const uint64_t pol_w = policy_evict_first();
      const uint64_t polP = p.swap ? pol_w : pol_act;
      const uint64_t polQ = p.swap ? pol_act : pol_w;
      const uint32_t tx = static_cast<uint32_t>((BM + p.bn) * 128);
      uint32_t stage = 0, phase = 0;
      long long issued = 0;
      // weight tiles of this CTA's first stages, issued before the previous
      // kernel has finished (their stages are fresh: no empty wait); each
      // stage's activation tile follows after pdl_wait()
      int pre = 0;
      if (early_weights) {
        SegIter it0;
        seg_begin(p, total, it0);
        int t0, a0, a1;
        while (pre < kStages && seg_next(p, total, it0, t0, a0, a1)) {
          int pt0, qt0, sp0;
          tile_coords(p, t0, pt0, qt0, sp0);
          for (int kb = a0; kb < a1 && pre < kStages; ++kb, ++pre) {
            mbar_expect_tx(&full[pre], tx);
            if (p.swap)
              tma_load_2d(sP + pre * P_STAGE, &tmP, &full[pre], kb * kBK, tile_prow(p, t0, pt0), polP);
            else
              tma_load_2d(sQ + pre * kQStage, &tmQ, &full[pre], kb * kBK, tile_qrow(p, t0, qt0), polQ);
          }
        }
        pdl_wait();
      }
      // one wait for the whole round, or per tile on the tile's expert
      bool ok = p.wait_per_expert ? true : wait_arrivals(p, abort_flag);
      SegIter it;
      seg_begin(p, total, it);
      int t, kb0, kb1;
      while (ok && seg_next(p, total, it, t, kb0, kb1)) {
        int pt, qt, sp;
        tile_coords(p, t, pt, qt, sp);
        if (p.wait_per_expert && !wait_arrivals(p, abort_flag, p.gtab[t].x)) {
          ok = false;
          break;
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (issued < pre) {  // its weight tile is already in flight
            if (p.swap)
              tma_load_2d(sQ + stage * kQStage, &tmQ, &full[stage], kb * kBK, tile_qrow(p, t, qt), polQ);
            else
              tma_load_2d(sP + stage * P_STAGE, &tmP, &full[stage], kb * kBK, tile_prow(p, t, pt), polP);
            gstamp(p, TRG_TMA, issued);
            ++issued;
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status, kStatusTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[stage], tx);
          tma_load_2d(sP + stage * P_STAGE, &tmP, &full[stage], kb * kBK, tile_prow(p, t, pt), polP);
          tma_load_2d(sQ + stage * kQStage, &tmQ, &full[stage], kb * kBK, tile_qrow(p, t, qt), polQ);
          gstamp(p, TRG_TMA, issued);
          ++issued;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Let every copy already issued land before the CTA can exit.
        long long first = issued > kStages ? issued - kStages : 0;
        for (long long i = first; i < issued; ++i)
          mbar_wait(&full[i % kStages], static_cast<uint32_t>((i / kStages) & 1), nullptr, nullptr, 0,
                    kWaitLimitNs / 4);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = FP8 ? make_idesc_mxf8(BM, p.bn) : make_idesc_bf16(BM, p.bn);
      uint32_t stage = 0, phase = 0;
      int local = 0;
      bool ok = true;
      long long steps = 0;
      SegIter it;
      seg_begin(p, total, it);
      int t, kb0, kb1;
      for (; ok && seg_next(p, total, it, t, kb0, kb1); ++local) {
        const uint32_t acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, abort_flag, p.status, kStatusTimeoutTmemEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kAccCols;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status, kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          gstamp(p, TRG_FULL, steps);
          if (FP8 && !mbar_wait(&sf_full[stage], phase, abort_flag, p.status, kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          gstamp(p, TRG_SFFULL, steps);
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sP + stage * P_STAGE);
          const uint32_t b_addr = smem_u32(sQ + stage * kQStage);
          // four UMMAs per 128-byte stage: K = 16 (bf16) or 32 (e4m3) each,
          // 32 bytes further into the swizzle atom
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t ad = make_sw128_desc(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = make_sw128_desc(b_addr + kk * 32, 16, 1024);
            if (FP8) {
              const uint32_t sfa = tmem_base + SF_COL0 + stage * SF_SLOT;
              umma_mxf8(d_tmem, ad, bd, idesc, sfa, sfa + 8, (kb > kb0 || kk > 0) ? 1u : 0u);
            } else {
              umma_bf16(d_tmem, ad, bd, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
            }
          }
          umma_commit(&empty[stage]);
          gstamp(p, TRG_ISSUED, steps);
          ++steps;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) umma_commit(&tfull[acc]);
      }
      // Every MMA this thread issued must be finished before TMEM is freed.
      umma_commit(drain);
      mbar_wait(drain, 0, nullptr, p.status, kStatusTimeoutFull);
    }
  } else if (FP8 && warp >= 6) {
    // scale-factor stagers: one warp per TMEM lane quadrant writes the same
    // values into its own quadrant. The scale bytes of stage i+4 are loaded
    // while stage i is stored, so a global-load latency is not paid once
    // per stage.
    const int q = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    // fetch cursor over the (tile, k-block) sequence this CTA walks
    int ft = blockIdx.x, fkb = 0, fkb1 = 0, fwrow = 0, ftok0 = 0;
    bool fresh = true;
    auto fetch = [&](uint32_t& wb, uint32_t (&r)[8]) -> bool {
      while (true) {
        if (ft >= total) return false;
        if (fresh) {
          int pt, qt, sp;
          tile_coords(p, ft, pt, qt, sp);
          if (p.wait_per_expert) {  // this tile's scales arrive with its expert's rows
            int ok = 1;
            if (lane == 0) ok = wait_arrivals(p, abort_flag, p.gtab[ft].x) ? 1 : 0;
            if (__shfl_sync(0xffffffffu, ok, 0) == 0) return false;
          }
          fkb = sp * p.kbps;
          fkb1 = min(fkb + p.kbps, p.nkb);
          fwrow = tile_prow(p, ft, pt) / BM;
          ftok0 = tile_qrow(p, ft, qt);
          fresh = false;
        }
        if (fkb < fkb1) break;
        ft += gridDim.x;
        fresh = true;
      }
      wb = __ldg(p.sf_w + static_cast<size_t>(fwrow) * p.sf_w_ld + fkb);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int tok = ftok0 + c * 32 + lane;
        r[c] = (c * 32 < p.bn && tok < p.M) ? __ldg(p.sf_a + static_cast<size_t>(fkb) * p.sf_a_ld + tok) : 127u;
      }
      ++fkb;
      return true;
    };
    uint32_t stage = 0, phase = 0;
    long long sf_steps = 0;
    auto store = [&](uint32_t wb, const uint32_t (&r)[8]) -> bool {
      if (!mbar_wait_warp(&empty[stage], phase ^ 1u, abort_flag, p.status, kStatusTimeoutEmpty)) return false;
      tc_fence_after();  // the MMAs that read this slot before have completed
      uint32_t rr[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) rr[c] = r[c] * 0x01010101u;
      const uint32_t w4 = wb * 0x01010101u;
      const uint32_t slot = tmem_base + lane_base + SF_COL0 + stage * SF_SLOT;
      tmem_st4(slot, w4, w4, w4, w4);
      tmem_st8(slot + 8, rr);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sf_full[stage]);
      if (lane == 0 && warp == 6) gstamp(p, TRG_SFARRIVE, sf_steps);
      ++sf_steps;
      if (++stage == kStages) {
        stage = 0;
        phase ^= 1u;
      }
      return true;
    };
    // four register sets in flight: the loads of stage i+4 are issued when
    // stage i is stored (compile-time indices keep them in registers)
    constexpr int kAhead = 4;
    uint32_t wv[kAhead], rv[kAhead][8];
    bool has[kAhead];
    bool arrived = true;
    if (p.wait_flag != nullptr && !p.wait_per_expert) {   // the activation scales arrive with the dispatched rows
      if (lane == 0) arrived = wait_arrivals(p, abort_flag);
      arrived = __shfl_sync(0xffffffffu, arrived ? 1 : 0, 0) != 0;
    }
#pragma unroll
    for (int k = 0; k < kAhead; ++k) has[k] = arrived && fetch(wv[k], rv[k]);
    bool go = arrived;
    while (go) {
#pragma unroll
      for (int k = 0; k < kAhead; ++k) {
        if (go && has[k]) {
          if (!store(wv[k], rv[k])) {
            go = false;
          } else {
            has[k] = fetch(wv[k], rv[k]);
          }
        } else {
          go = false;
        }
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = q * 32 + lane;
    int local = 0;
    uint32_t eph = 0;        // phase of the epilogue warps' mbarrier
    SegIter it;
    seg_begin(p, total, it);
    int t, kb0, kb1;
    for (; seg_next(p, total, it, t, kb0, kb1); ++local) {
      int pt, qt, sp;
      tile_coords(p, t, pt, qt, sp);
      const uint32_t acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait_warp(&tfull[acc], acc_phase, abort_flag, p.status, kStatusTimeoutTmemFull)) break;
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * kAccCols;
      const bool dp = p.streamk && t < p.dp_tiles;
      int c0 = 0;
      for (; c0 + 32 <= p.bn; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(t_row + c0, r);
        tmem_ld_wait();
        if (p.grouped) store_chunk_grouped<32>(p, t, row, c0, r);
        else store_chunk<32>(p, pt, qt, row, c0, r, dp);
      }
      if (c0 < p.bn) {
        uint32_t r[16];
        tmem_ld16(t_row + c0, r);
        tmem_ld_wait();
        if (p.grouped) store_chunk_grouped<16>(p, t, row, c0, r);
        else store_chunk<16>(p, pt, qt, row, c0, r, dp);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (p.tile_ctr != nullptr && !p.grouped && !dp && p.epi == EPI_ATOMIC_F32) {
        // this share's partial sums are in the workspace: count its
        // k-blocks; the share that completes the tile stores it. The
        // epilogue warps meet on a bounded mbarrier (never an unbounded
        // bar.sync: a warp that gave up on a wait must not strand the rest).
        __threadfence();
        mbar_arrive(ebar);
        if (!mbar_wait_warp(ebar, eph & 1u, abort_flag, p.status, kStatusTimeoutTmemFull)) break;
        ++eph;
        if (threadIdx.x == 64) {
          const unsigned add = static_cast<unsigned>(kb1 - kb0);
          const unsigned old = atomicAdd(&p.tile_ctr[t / p.splits], add);
          *s_last = (old + add == static_cast<unsigned>(p.nkb)) ? 1 : 0;
        }
        mbar_arrive(ebar);
        if (!mbar_wait_warp(ebar, eph & 1u, abort_flag, p.status, kStatusTimeoutTmemFull)) break;
        ++eph;
        if (*s_last) {
          __threadfence();
          int c1 = 0;
          for (; c1 + 32 <= p.bn; c1 += 32) finish_chunk<32>(p, pt, qt, row, c1);
          if (c1 < p.bn) finish_chunk<16>(p, pt, qt, row, c1);
          if (threadIdx.x == 64) p.tile_ctr[t / p.splits] = 0;
        }
      }
    }
  }

  // push mode: make this thread's peer stores visible system-wide before
  // the CTA reports completion
  if (p.push && warp >= 2 && warp < 6) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if (p.push && threadIdx.x == 0) {
    // the last CTA to finish signals every rank once for the whole GEMM
    if (atomicAdd(p.done_ctr, 1u) == gridDim.x - 1) {
      *p.done_ctr = 0;
      __threadfence_system();
      for (int d = 0; d < p.world; ++d) atomicAdd_system(p.peer_flag[d], 1u);
    }
  }
}

// Reduce the fp32 split-K workspace into the bf16 output (optionally
// applying SwiGLU) and zero the workspace for its next use.
struct PushDst {
  void* out[kMaxPeers];
  unsigned int* flag[kMaxPeers];
};

// Split-K finalize for push mode: fp32 workspace -> bf16 rows stored to
// every rank's receive slot (zeroing the workspace), then the last CTA
// signals every rank once.
__global__ void splitk_finalize_push_kernel(float* __restrict__ ws, int M, int N, int ldc, int world,
                                            const PushDst dst, unsigned int* done_ctr, int owner) {
  const int m = blockIdx.y;
  // owner mode (reduce-scatter): row m goes only to rank (m / 128) % world
  const int d0 = owner ? (m / BM) % world : 0;
  const int d1 = owner ? d0 + 1 : world;
  if (m < M) {
    float* row = ws + static_cast<size_t>(m) * N;
    for (int n = (blockIdx.x * blockDim.x + threadIdx.x) * 4; n < N; n += gridDim.x * blockDim.x * 4) {
      if (n + 4 <= N) {
        float4 v = *reinterpret_cast<float4*>(row + n);
        *reinterpret_cast<float4*>(row + n) = make_float4(0.f, 0.f, 0.f, 0.f);
        uint2 o;
        o.x = pack_bf16(v.x, v.y);
        o.y = pack_bf16(v.z, v.w);
        for (int d = d0; d < d1; ++d)
          *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(dst.out[d]) + static_cast<size_t>(m) * ldc + n) = o;
      } else {
        for (int j = n; j < N; ++j) {
          const __nv_bfloat16 b = __float2bfloat16(row[j]);
          row[j] = 0.f;
          for (int d = d0; d < d1; ++d) static_cast<__nv_bfloat16*>(dst.out[d])[static_cast<size_t>(m) * ldc + j] = b;
        }
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(done_ctr, 1u) == gridDim.x * gridDim.y - 1) {
      *done_ctr = 0;
      __threadfence_system();
      for (int d = 0; d < world; ++d) atomicAdd_system(dst.flag[d], 1u);
    }
  }
}

__global__ void splitk_finalize_kernel(float* __restrict__ ws, __nv_bfloat16* __restrict__ out, int M, int N,
                                       int ldc, int swiglu, int n_begin) {
  pdl_trigger();
  pdl_wait();
  const int m = blockIdx.y;
  if (m >= M) return;
  float* row = ws + static_cast<size_t>(m) * N;
  __nv_bfloat16* orow = out + static_cast<size_t>(m) * ldc;
  if (!swiglu) {
    for (int n = n_begin + (blockIdx.x * blockDim.x + threadIdx.x) * 4; n < N; n += gridDim.x * blockDim.x * 4) {
      if (n + 4 <= N) {
        float4 v = *reinterpret_cast<float4*>(row + n);
        *reinterpret_cast<float4*>(row + n) = make_float4(0.f, 0.f, 0.f, 0.f);
        uint2 o;
        o.x = pack_bf16(v.x, v.y);
        o.y = pack_bf16(v.z, v.w);
        *reinterpret_cast<uint2*>(orow + n) = o;
      } else {
        for (int j = n; j < N; ++j) {
          orow[j] = __float2bfloat16(row[j]);
          row[j] = 0.f;
        }
      }
    }
  } else {
    for (int n = n_begin + (blockIdx.x * blockDim.x + threadIdx.x) * 4; n < N; n += gridDim.x * blockDim.x * 4) {
      float4 v = *reinterpret_cast<float4*>(row + n);
      *reinterpret_cast<float4*>(row + n) = make_float4(0.f, 0.f, 0.f, 0.f);
      uint32_t o = pack_bf16(silu(v.x) * v.y, silu(v.z) * v.w);
      *reinterpret_cast<uint32_t*>(orow + n / 2) = o;
    }
  }
}

struct Plan {
  Params p;
  int grid;
};

static long long* g_gemm_trace = nullptr;

template <bool FP8, bool DEEP>
inline int launch_gemm_variant(const CUtensorMap& tmP, const CUtensorMap& tmQ, const Params& p, int grid,
                               cudaStream_t stream) {
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaFuncSetAttribute(gemm_kernel<FP8, DEEP>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    attr_set[dev] = true;
  }
  launch_pdl_g(gemm_kernel<FP8, DEEP>, grid, FP8 ? NUM_THREADS_FP8 : NUM_THREADS, SMEM_BYTES, stream, tmP, tmQ, p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

template <bool FP8>
inline int launch_gemm(const CUtensorMap& tmP, const CUtensorMap& tmQ, const Params& p_in, int grid,
                       cudaStream_t stream) {
  Params p = p_in;
  p.trace = g_gemm_trace;
  // INFERA_GEMM_DEEP=0 keeps small tiles on the shallow ring (for comparison)
  static const bool deep = [] {
    const char* v = getenv("INFERA_GEMM_DEEP");
    return v == nullptr || v[0] != '0';
  }();
  if (deep && p.bn <= DEEP_BN) return launch_gemm_variant<FP8, true>(tmP, tmQ, p, grid, stream);
  return launch_gemm_variant<FP8, false>(tmP, tmQ, p, grid, stream);
}

// Split-K factor for a plan whose tiles are set: minimise waves/split (time
// in units of one full tile), with a 3% penalty per extra split for the
// atomics and the finalize pass. (Splitting above one wave of tiles - 224
// decode tiles on 148 SMs - measured slower: 58.8 vs 54.5 us for
// 64 x 28672 x 4096.)
inline void choose_splits(Plan& pl, int num_sms, int force_split) {
  Params& p = pl.p;
  const int tiles = p.p_tiles * p.q_tiles;
  int best = 1;
  if (force_split > 0) {
    best = force_split;
  } else if (tiles < num_sms) {
    double best_cost = 1e30;
    for (int s = 1; s <= 16; ++s) {
      if (p.nkb / s < 4 && s > 1) break;
      double waves = static_cast<double>((tiles * s + num_sms - 1) / num_sms);
      double cost = waves / s * (1.0 + 0.03 * (s - 1));
      if (cost < best_cost - 1e-9) {
        best_cost = cost;
        best = s;
      }
    }
  }
  if ((p.N % 4) != 0) best = 1;
  p.kbps = (p.nkb + best - 1) / best;
  p.splits = (p.nkb + p.kbps - 1) / p.kbps;
  const int units = tiles * p.splits;
  pl.grid = units < num_sms ? units : num_sms;
}

// fp8 plan: always swap-AB; token tiles of up to 192 (multiples of 32)
// balanced over the token count.
inline Plan make_plan_fp8(int M, int N, int K, int num_sms, int force_split) {
  Plan pl{};
  Params& p = pl.p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.nkb = K / BK_FP8;
  p.swap = 1;
  const int qt = M > 0 ? (M + MAX_BN_FP8 - 1) / MAX_BN_FP8 : 1;
  const int per = (M + qt - 1) / qt;
  p.bn = ((per + 31) / 32) * 32;
  p.p_tiles = (N + BM - 1) / BM;
  p.q_tiles = qt;
  choose_splits(pl, num_sms, force_split);
  return pl;
}

// Choose operand order, tile width and split-K factor for one problem.
// Largest token count that runs swap-AB (weights on the 128-row MMA side,
// tokens as N in up to two tiles of <= 256): every weight tile is read by
// the CTAs of its token tiles back to back, instead of once per 128-token
// row block. Above 128 tokens this pays only for wide weights (N >= 16384:
// 288 tokens x 28672 x 4096 runs 0.134 ms swapped against 0.157 ms; 288 x
// 4096 x 14336 runs 0.061 ms swapped against 0.052 ms).
// INFERA_GEMM_SWAP_MAX overrides (128: swap only for one token tile of <= 128).
inline int swap_max_tokens() {
  static const int v = [] {
    const char* e = std::getenv("INFERA_GEMM_SWAP_MAX");
    return e != nullptr && *e ? std::atoi(e) : 512;
  }();
  return v;
}

inline Plan make_plan(int M, int N, int K, int num_sms, int force_split, int swap_max = -1) {
  Plan pl{};
  Params& p = pl.p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.nkb = (K + BK - 1) / BK;
  if (swap_max < 0) swap_max = swap_max_tokens();
  p.swap = (M <= 128 || (M <= swap_max && N >= 16384)) ? 1 : 0;
  if (p.swap) {
    p.q_tiles = M > 0 ? (M + MAX_BN - 1) / MAX_BN : 1;
    const int per = (M + p.q_tiles - 1) / p.q_tiles;
    p.bn = ((per + 15) / 16) * 16;
    p.p_tiles = (N + BM - 1) / BM;
  } else {
    p.bn = MAX_BN;
    p.p_tiles = (M + BM - 1) / BM;
    p.q_tiles = (N + MAX_BN - 1) / MAX_BN;
  }
  choose_splits(pl, num_sms, force_split);
  // Stream-K when whole tiles would leave most of the last wave idle (e.g.
  // 224 weight tiles of a 64-token decode GEMM on 148 SMs: 2 waves for 1.51
  // waves of work): every CTA takes 1/num_sms of all k-steps, partial tiles
  // meet in the fp32 workspace.
  const int tiles = p.p_tiles * p.q_tiles;
  if (force_split == 0 && p.splits == 1 && tiles >= num_sms && tiles < 4 * num_sms && p.nkb >= 8 &&
      (p.N % 4) == 0) {
    const int waves = (tiles + num_sms - 1) / num_sms;
    if (static_cast<double>(tiles) / (waves * num_sms) < 0.85) {
      p.streamk = 1;
      pl.grid = num_sms;
      // whole tiles for the full waves, stream-K only over the partial wave
      // (plus one full wave when the partial one is under half the SMs, so
      // no share is a sliver): most tiles skip the workspace. The whole
      // tiles end on a weight-row block (swap-AB) / token-column tile
      // boundary, so the workspace columns are one contiguous range.
      const int rem = tiles % num_sms;
      int sk = rem >= num_sms / 2 ? rem : rem + num_sms;
      if (sk > tiles) sk = tiles;
      const int unit = p.swap ? p.q_tiles : p.p_tiles;
      p.dp_tiles = ((tiles - sk) / unit) * unit;
    }
  }
  return pl;
}

}  // namespace gemm
}  // namespace ib200

using namespace ib200;

namespace ib200 {
namespace gemm {

// Operand element type of one launch: bf16, or e4m3 with UE8M0 block scales.
struct Operands {
  bool fp8;
  const uint8_t* sf_a;  // [K/128, sf_a_ld]
  int sf_a_ld;
  const uint8_t* sf_w;  // [weight rows / 128, K/128]
};

inline bool operands_ok(const Operands& o, int K, int lda, int ldw) {
  if (!o.fp8) return (K % 8) == 0 && (lda % 8) == 0 && (ldw % 8) == 0;
  return (K % BK_FP8) == 0 && (lda % 16) == 0 && (ldw % 16) == 0 && o.sf_a != nullptr && o.sf_w != nullptr;
}

inline void set_scales(Params& p, const Operands& o) {
  p.sf_a = o.sf_a;
  p.sf_a_ld = o.sf_a_ld;
  p.sf_w = o.sf_w;
  p.sf_w_ld = p.K / BK_FP8;
}

inline bool encode_pq(const Operands& o, const Params& p, const void* A, const void* W, long long w_rows, int lda,
                      int ldw, CUtensorMap* tmP, CUtensorMap* tmQ) {
  const void* Pbase = p.swap ? W : A;
  const void* Qbase = p.swap ? A : W;
  const long long Prows = p.swap ? w_rows : p.M;
  const long long Qrows = p.swap ? p.M : w_rows;
  const int Pld = p.swap ? ldw : lda;
  const int Qld = p.swap ? lda : ldw;
  if (o.fp8)
    return cached_tmap_2d(tmP, Pbase, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, Prows, p.K, Pld, BM, BK_FP8) &&
           cached_tmap_2d(tmQ, Qbase, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, Qrows, p.K, Qld, p.bn, BK_FP8);
  return cached_tmap_2d(tmP, Pbase, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Prows, p.K, Pld, BM, BK) &&
         cached_tmap_2d(tmQ, Qbase, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, Qrows, p.K, Qld, p.bn, BK);
}

inline int launch(const Operands& o, const CUtensorMap& tmP, const CUtensorMap& tmQ, const Params& p, int grid,
                  cudaStream_t stream) {
  return o.fp8 ? launch_gemm<true>(tmP, tmQ, p, grid, stream) : launch_gemm<false>(tmP, tmQ, p, grid, stream);
}

// Per-device tile counters for the in-kernel split reduction (registered by
// the host scratch owner; absent: the finalize kernel reduces).
struct TileCounters {
  unsigned int* ptr = nullptr;
  int n = 0;
};
inline TileCounters& tile_counters() {
  static TileCounters t[64];
  int dev = 0;
  cudaGetDevice(&dev);
  return t[dev >= 0 && dev < 64 ? dev : 0];
}

// defer: a split result stays in the fp32 workspace (every tile through it,
// no finalize); *in_ws (optional) reports whether it did.
inline int run_dense(const Operands& o, const void* A, const void* W, void* out, int M, int N, int K, int lda,
                     int ldw, int ldc, int epi, float* ws, int force_split, int* status, cudaStream_t stream,
                     bool defer = false, int* in_ws = nullptr) {
  if (in_ws != nullptr) *in_ws = 0;
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if (!operands_ok(o, K, lda, ldw)) return -1;
  if (epi == EPI_SWIGLU && (N % 2) != 0) return -1;
  const int num_sms = num_sms_for_current_device();
  const int fs = ws == nullptr ? 1 : force_split;
  Plan pl = o.fp8 ? make_plan_fp8(M, N, K, num_sms, fs) : make_plan(M, N, K, num_sms, fs);
  Params& p = pl.p;
  p.status = status;
  p.ldc = ldc;
  p.push = 0;
  p.world = 1;
  p.done_ctr = nullptr;
  p.grouped = 0;
  set_scales(p, o);
  if (ws == nullptr) p.streamk = 0;
  const bool split = p.splits > 1 || p.streamk;
  p.epi = split ? EPI_ATOMIC_F32 : epi;
  p.out = split ? static_cast<void*>(ws) : out;
  p.epi_dp = epi;
  p.out_dp = out;
  if (!p.streamk || defer) p.dp_tiles = 0;
  const TileCounters& tc = tile_counters();
  p.tile_ctr = split && !defer && tc.ptr != nullptr && p.p_tiles * p.q_tiles <= tc.n ? tc.ptr : nullptr;
  CUtensorMap tmP, tmQ;
  if (!encode_pq(o, p, A, W, N, lda, ldw, &tmP, &tmQ)) return -2;
  int rc = launch(o, tmP, tmQ, p, pl.grid, stream);
  if (rc != 0) return rc;
  if (split && defer) {
    if (in_ws != nullptr) *in_ws = 1;
    return 0;
  }
  if (split && p.tile_ctr == nullptr) {
    // stream-K: only the columns of the tiles past dp_tiles went through
    // the workspace (swap-AB: weight-row blocks, else token-column tiles)
    const int n_begin = p.streamk ? (p.swap ? (p.dp_tiles / p.q_tiles) * BM : (p.dp_tiles / p.p_tiles) * p.bn) : 0;
    dim3 g((N - n_begin + 1023) / 1024, M);
    launch_pdl(splitk_finalize_kernel, g, 256, 0, stream, ws, static_cast<__nv_bfloat16*>(out), M, N, ldc,
                                                  epi == EPI_SWIGLU ? 1 : 0, n_begin);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return 0;
}

inline int run_push(const Operands& o, const void* A, const void* W, int M, int N, int K, int lda, int ldw, int ldc,
                    int world, void* const* peer_out, unsigned int* const* peer_flag, unsigned int* done_ctr,
                    float* ws, int* status, cudaStream_t stream, int owner = 0) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if (!operands_ok(o, K, lda, ldw)) return -1;
  if (world < 1 || world > kMaxPeers) return -1;
  const int num_sms = num_sms_for_current_device();
  // split K like the plain GEMM does (small M leaves most SMs idle
  // otherwise); the split path pushes from its finalize kernel
  const int fs = ws == nullptr ? 1 : 0;
  Plan pl = o.fp8 ? make_plan_fp8(M, N, K, num_sms, fs) : make_plan(M, N, K, num_sms, fs, 128);
  Params& p = pl.p;
  p.streamk = 0;  // peer-store epilogues write whole tiles
  const bool split = p.splits > 1;
  p.status = status;
  p.ldc = split ? N : ldc;
  p.epi = split ? EPI_ATOMIC_F32 : EPI_BF16;
  p.out = split ? static_cast<void*>(ws) : peer_out[0];
  p.push = split ? 0 : 1;
  p.world = world;
  for (int d = 0; d < kMaxPeers; ++d) {
    p.peer_out[d] = d < world ? peer_out[d] : nullptr;
    p.peer_flag[d] = d < world ? peer_flag[d] : nullptr;
  }
  p.done_ctr = done_ctr;
  p.grouped = 0;
  p.push_owner = owner;  // reduce-scatter: token row m goes to rank (m / 128) % world
  set_scales(p, o);
  CUtensorMap tmP, tmQ;
  if (!encode_pq(o, p, A, W, N, lda, ldw, &tmP, &tmQ)) return -2;
  int rc = launch(o, tmP, tmQ, p, pl.grid, stream);
  if (rc != 0) return rc;
  if (split) {
    PushDst dst;
    for (int d = 0; d < kMaxPeers; ++d) {
      dst.out[d] = p.peer_out[d];
      dst.flag[d] = p.peer_flag[d];
    }
    dim3 g((N + 1023) / 1024, M);
    splitk_finalize_push_kernel<<<g, 256, 0, stream>>>(ws, M, N, ldc, world, dst, done_ctr, owner);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return 0;
}

inline int run_grouped(const Operands& o, const void* A, const void* W, void* out, int R, int N, int K, int E,
                       int lda, int ldw, int ldc, int epi, const int* gtab, const int* gnum, int bn, int grid_tiles,
                       int* status, cudaStream_t stream, const int* row_map = nullptr, int world = 1,
                       void* const* peer_out = nullptr, unsigned int* const* peer_flag = nullptr,
                       unsigned int* done_ctr = nullptr, const unsigned int* wait_flag = nullptr,
                       unsigned int wait_target = 0, uint64_t wait_limit_ns = 0, int wait_per_expert = 0) {
  if (R <= 0 || N <= 0 || K <= 0 || E <= 0) return 0;
  if (!operands_ok(o, K, lda, ldw) || (N % BM) != 0) return -1;
  if (o.fp8 ? (bn < 32 || bn > MAX_BN_FP8 || (bn % 32) != 0) : (bn < 16 || bn > MAX_BN || (bn % 16) != 0))
    return -1;
  if (epi == EPI_SWIGLU && (N % 2) != 0) return -1;
  Params p{};
  p.M = R;
  p.N = N;
  p.K = K;
  p.bn = bn;
  p.swap = 1;
  p.splits = 1;
  p.nkb = o.fp8 ? K / BK_FP8 : (K + BK - 1) / BK;
  p.kbps = p.nkb;
  p.p_tiles = 1;
  p.q_tiles = 1;
  p.epi = epi;
  p.out = out;
  p.ldc = ldc;
  p.status = status;
  p.grouped = 1;
  p.gtab = reinterpret_cast<const int4*>(gtab);
  p.gnum = gnum;
  p.n_per_expert = N;
  p.row_map = row_map;
  p.wait_flag = wait_flag;
  p.wait_target = wait_target;
  p.wait_limit_ns = wait_limit_ns;
  p.wait_per_expert = wait_flag != nullptr && wait_per_expert ? 1 : 0;
  if (row_map != nullptr) {
    if (epi != EPI_BF16 || world < 1 || world > kMaxPeers || done_ctr == nullptr) return -1;
    p.push = 1;
    p.world = world;
    for (int d = 0; d < kMaxPeers; ++d) {
      p.peer_out[d] = d < world ? peer_out[d] : nullptr;
      p.peer_flag[d] = d < world ? peer_flag[d] : nullptr;
    }
    p.done_ctr = done_ctr;
  }
  set_scales(p, o);
  CUtensorMap tmP, tmQ;
  if (!encode_pq(o, p, A, W, static_cast<long long>(E) * N, lda, ldw, &tmP, &tmQ)) return -2;
  const int num_sms = num_sms_for_current_device();
  const int grid = grid_tiles < num_sms ? (grid_tiles > 0 ? grid_tiles : 1) : num_sms;
  return launch(o, tmP, tmQ, p, grid, stream);
}

}  // namespace gemm
}  // namespace ib200

// C ABI. Returns 0 on success, a negative code on bad arguments / encode
// failure, or a CUDA error code from the launch.
//   epi: 0 = bf16 store, 1 = SwiGLU (out has N/2 columns)
//   ws : fp32 workspace of >= M*N floats, all zero on entry (left zero), only
//        touched when the plan splits K; may be null if split_k == 1 forced.
extern "C" int ib_gemm_bf16(const void* A, const void* W, void* out, int M, int N, int K, int lda, int ldw,
                            int ldc, int epi, float* ws, int force_split, int* status, cudaStream_t stream) {
  const gemm::Operands o{false, nullptr, 0, nullptr};
  return gemm::run_dense(o, A, W, out, M, N, K, lda, ldw, ldc, epi, ws, force_split, status, stream);
}

// As ib_gemm_bf16 (plain epilogue), but a split-K / stream-K result is left
// in ws ([M, N] fp32, row stride N) for its consumer to read and zero;
// *in_ws = 1 then, 0 when the GEMM wrote out directly.
extern "C" int ib_gemm_bf16_deferred(const void* A, const void* W, void* out, int M, int N, int K, int lda, int ldw,
                                     int ldc, float* ws, int* status, int* in_ws, cudaStream_t stream) {
  const gemm::Operands o{false, nullptr, 0, nullptr};
  return gemm::run_dense(o, A, W, out, M, N, K, lda, ldw, ldc, gemm::EPI_BF16, ws, 0, status, stream, true, in_ws);
}

// W8A8 e4m3 GEMM with UE8M0 block scales: A [M, K] e4m3 (row pitch lda
// bytes), sf_a [K/128, sf_a_ld] (token-group scales, K-group-major), W
// [N, K] e4m3, sf_w [ceil(N/128), K/128] (128x128 block scales); out bf16.
extern "C" int ib_gemm_fp8(const void* A, const uint8_t* sf_a, int sf_a_ld, const void* W, const uint8_t* sf_w,
                           void* out, int M, int N, int K, int lda, int ldw, int ldc, int epi, float* ws,
                           int force_split, int* status, cudaStream_t stream) {
  const gemm::Operands o{true, sf_a, sf_a_ld, sf_w};
  return gemm::run_dense(o, A, W, out, M, N, K, lda, ldw, ldc, epi, ws, force_split, status, stream);
}

// Fused GEMM + one-shot all-reduce push (row-parallel tensor-parallel
// layers): out = A @ W^T computed locally, each tile stored to
// peer_out[d] (this rank's receive slot on rank d, bf16 [M, ldc]) for every
// rank d, then peer_flag[d] (rank d's arrival counter for this rank) is
// incremented once. done_ctr: a local zero-initialised counter.
extern "C" int ib_gemm_bf16_push(const void* A, const void* W, int M, int N, int K, int lda, int ldw, int ldc,
                                 int world, void* const* peer_out, unsigned int* const* peer_flag,
                                 unsigned int* done_ctr, float* ws, int* status, cudaStream_t stream) {
  const gemm::Operands o{false, nullptr, 0, nullptr};
  return gemm::run_push(o, A, W, M, N, K, lda, ldw, ldc, world, peer_out, peer_flag, done_ctr, ws, status, stream);
}

// Reduce-scatter variant (two-shot all-reduce, first half): each 128-row
// block of the output goes only to rank (block % world).
extern "C" int ib_gemm_bf16_push_rs(const void* A, const void* W, int M, int N, int K, int lda, int ldw, int ldc,
                                    int world, void* const* peer_out, unsigned int* const* peer_flag,
                                    unsigned int* done_ctr, float* ws, int* status, cudaStream_t stream) {
  const gemm::Operands o{false, nullptr, 0, nullptr};
  return gemm::run_push(o, A, W, M, N, K, lda, ldw, ldc, world, peer_out, peer_flag, done_ctr, ws, status, stream,
                        1);
}

extern "C" int ib_gemm_fp8_push_rs(const void* A, const uint8_t* sf_a, int sf_a_ld, const void* W,
                                   const uint8_t* sf_w, int M, int N, int K, int lda, int ldw, int ldc, int world,
                                   void* const* peer_out, unsigned int* const* peer_flag, unsigned int* done_ctr,
                                   float* ws, int* status, cudaStream_t stream) {
  const gemm::Operands o{true, sf_a, sf_a_ld, sf_w};
  return gemm::run_push(o, A, W, M, N, K, lda, ldw, ldc, world, peer_out, peer_flag, done_ctr, ws, status, stream,
                        1);
}

extern "C" int ib_gemm_fp8_push(const void* A, const uint8_t* sf_a, int sf_a_ld, const void* W, const uint8_t* sf_w,
                                int M, int N, int K, int lda, int ldw, int ldc, int world, void* const* peer_out,
                                unsigned int* const* peer_flag, unsigned int* done_ctr, float* ws, int* status,
                                cudaStream_t stream) {
  const gemm::Operands o{true, sf_a, sf_a_ld, sf_w};
  return gemm::run_push(o, A, W, M, N, K, lda, ldw, ldc, world, peer_out, peer_flag, done_ctr, ws, status, stream);
}

// Grouped GEMM over experts (swap-AB): for every tile {e, n_tile, m0, mend}
// of gtab[0 .. *gnum), out[m, :] (rows m0 .. mend-1) = A[m, :] @ W[e]^T
// restricted to features [n_tile*128, +128). A: [R, K] tokens sorted by
// expert; W: [E, N, K] stacked; out: [R, ldc] (N/2 columns with SwiGLU).
// bn: token columns per tile (16 / 32 / 64 / 128 / 256); grid_tiles: the
// most tiles gtab can hold (sizes the persistent grid).
extern "C" int ib_gemm_grouped(const void* A, const void* W, void* out, int R, int N, int K, int E, int lda, int ldw,
                               int ldc, int epi, const int* gtab, const int* gnum, int bn, int grid_tiles, int* status,
                               cudaStream_t stream) {
  const gemm::Operands o{false, nullptr, 0, nullptr};
  return gemm::run_grouped(o, A, W, out, R, N, K, E, lda, ldw, ldc, epi, gtab, gnum, bn, grid_tiles, status, stream);
}

// Grouped GEMM (bf16, or fp8 when sf_w is not null) over rows that other
// GPUs are still storing into A (and sf_a): the TMA producer and the scale
// stagers first wait, bounded, until *wait_flag >= wait_target (the
// expert-parallel dispatch's arrival counter), so the dispatch's wait is
// fused into the up projection instead of being its own launch.
extern "C" int ib_gemm_grouped_wait(const void* A, const uint8_t* sf_a, int sf_a_ld, const void* W,
                                    const uint8_t* sf_w, void* out, int R, int N, int K, int E, int lda, int ldw,
                                    int ldc, int epi, const int* gtab, const int* gnum, int bn, int grid_tiles,
                                    const unsigned int* wait_flag, unsigned int wait_target, int* status,
                                    cudaStream_t stream) {
  const gemm::Operands o{sf_w != nullptr, sf_a, sf_a_ld, sf_w};
  return gemm::run_grouped(o, A, W, out, R, N, K, E, lda, ldw, ldc, epi, gtab, gnum, bn, grid_tiles, status, stream,
                           nullptr, 1, nullptr, nullptr, nullptr, wait_flag, wait_target);
}

// As ib_gemm_grouped_wait with one arrival counter per local expert:
// wait_flag[e] >= wait_target is waited (bounded) before each tile of
// expert e, by the TMA producer and (fp8) the scale stagers, so an
// expert's tiles start as soon as its rows from every source are in.
extern "C" int ib_gemm_grouped_wait_ex(const void* A, const uint8_t* sf_a, int sf_a_ld, const void* W,
                                       const uint8_t* sf_w, void* out, int R, int N, int K, int E, int lda, int ldw,
                                       int ldc, int epi, const int* gtab, const int* gnum, int bn, int grid_tiles,
                                       const unsigned int* wait_flag, unsigned int wait_target, int per_expert,
                                       unsigned long long wait_limit_ns, int* status, cudaStream_t stream) {
  const gemm::Operands o{sf_w != nullptr, sf_a, sf_a_ld, sf_w};
  return gemm::run_grouped(o, A, W, out, R, N, K, E, lda, ldw, ldc, epi, gtab, gnum, bn, grid_tiles, status, stream,
                           nullptr, 1, nullptr, nullptr, nullptr, wait_flag, wait_target, wait_limit_ns, per_expert);
}

// As ib_gemm_grouped_wait with the arrival wait bounded by wait_limit_ns
// instead of the default 2 s. On expiry the status word gets
// kStatusTimeoutPeer (5), every role of the CTA stops, drains what it
// issued, frees its TMEM and returns, so the context stays usable.
extern "C" int ib_gemm_grouped_wait_for(const void* A, const uint8_t* sf_a, int sf_a_ld, const void* W,
                                        const uint8_t* sf_w, void* out, int R, int N, int K, int E, int lda, int ldw,
                                        int ldc, int epi, const int* gtab, const int* gnum, int bn, int grid_tiles,
                                        const unsigned int* wait_flag, unsigned int wait_target,
                                        unsigned long long wait_limit_ns, int* status, cudaStream_t stream) {
  const gemm::Operands o{sf_w != nullptr, sf_a, sf_a_ld, sf_w};
  return gemm::run_grouped(o, A, W, out, R, N, K, E, lda, ldw, ldc, epi, gtab, gnum, bn, grid_tiles, status, stream,
                           nullptr, 1, nullptr, nullptr, nullptr, wait_flag, wait_target, wait_limit_ns);
}

// fp8 grouped GEMM: as above with e4m3 operands; sf_a [K/128, sf_a_ld] over
// the sorted rows, sf_w [E*N/128, K/128]; bn a multiple of 32 up to 192.
extern "C" int ib_gemm_fp8_grouped(const void* A, const uint8_t* sf_a, int sf_a_ld, const void* W,
                                   const uint8_t* sf_w, void* out, int R, int N, int K, int E, int lda, int ldw,
                                   int ldc, int epi, const int* gtab, const int* gnum, int bn, int grid_tiles,
                                   int* status, cudaStream_t stream) {
  const gemm::Operands o{true, sf_a, sf_a_ld, sf_w};
  return gemm::run_grouped(o, A, W, out, R, N, K, E, lda, ldw, ldc, epi, gtab, gnum, bn, grid_tiles, status, stream);
}

// Grouped GEMM whose epilogue stores every output row m straight into a
// peer's buffer: row_map[m] = (rank << 27) | row, peer_out[rank] bf16 with
// row pitch ldc; after the whole GEMM, peer_flag[d] += 1 on every rank d
// (done_ctr: a local zero-initialised counter). The expert-parallel return
// of the MoE layer, fused into its down projection. fp8: sf_a / sf_w as in
// ib_gemm_fp8_grouped (null for bf16).
extern "C" int ib_gemm_grouped_push(const void* A, const uint8_t* sf_a, int sf_a_ld, const void* W,
                                    const uint8_t* sf_w, int R, int N, int K, int E, int lda, int ldw, int ldc,
                                    const int* gtab, const int* gnum, int bn, int grid_tiles, const int* row_map,
                                    int world, void* const* peer_out, unsigned int* const* peer_flag,
                                    unsigned int* done_ctr, int* status, cudaStream_t stream) {
  const gemm::Operands o{sf_w != nullptr, sf_a, sf_a_ld, sf_w};
  return gemm::run_grouped(o, A, W, nullptr, R, N, K, E, lda, ldw, ldc, gemm::EPI_BF16, gtab, gnum, bn, grid_tiles,
                           status, stream, row_map, world, peer_out, peer_flag, done_ctr);
}

// Plan introspection for tests and benchmarks: writes
// [swap, bn, p_tiles, q_tiles, splits, kbps, grid].
extern "C" void ib_gemm_bf16_plan(int M, int N, int K, int num_sms, int force_split, int* out7) {
  using namespace ib200::gemm;
  Plan pl = make_plan(M, N, K, num_sms, force_split);
  out7[0] = pl.p.swap;
  out7[1] = pl.p.bn;
  out7[2] = pl.p.p_tiles;
  out7[3] = pl.p.q_tiles;
  // a stream-K plan needs the split-K workspace and finalize pass too: it
  // reports splits = -1
  out7[4] = pl.p.streamk ? -1 : pl.p.splits;
  out7[5] = pl.p.kbps;
  out7[6] = pl.grid;
}

extern "C" void ib_gemm_fp8_plan(int M, int N, int K, int num_sms, int force_split, int* out7) {
  using namespace ib200::gemm;
  Plan pl = make_plan_fp8(M, N, K, num_sms, force_split);
  out7[0] = pl.p.swap;
  out7[1] = pl.p.bn;
  out7[2] = pl.p.p_tiles;
  out7[3] = pl.p.q_tiles;
  out7[4] = pl.p.splits;
  out7[5] = pl.p.kbps;
  out7[6] = pl.grid;
}

// Diagnostics: the next GEMM launches stamp CTA 0's pipeline events into
// trace[5 * 128] (clock64), or stop when trace is null.
// Register n zero-initialised uint32 tile counters on the current device
// (null: none): split-K and stream-K GEMMs then reduce inside the kernel.
extern "C" void ib_gemm_set_tile_counters(void* ptr, int n) {
  auto& t = ib200::gemm::tile_counters();
  t.ptr = static_cast<unsigned int*>(ptr);
  t.n = ptr != nullptr ? n : 0;
}

// Whether dense GEMMs on the current device reduce split partials in-kernel.
extern "C" int ib_gemm_fused_reduce() { return ib200::gemm::tile_counters().ptr != nullptr ? 1 : 0; }

extern "C" void ib_gemm_set_trace(long long* trace) { ib200::gemm::g_gemm_trace = trace; }
