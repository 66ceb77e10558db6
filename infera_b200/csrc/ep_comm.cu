// Expert-parallel dispatch and return over NVLink peer memory (no
// all-to-all library call on the data path).
//
// Every rank holds, in a CUDA-IPC region mapped by all ranks, a receive
// buffer laid out [local expert][source rank][rows] and a return buffer
// laid out like its own expert-sorted rows. With the all-gathered counts
// C[src][expert] (int32 [W, E], every rank has the same copy):
//
//   ib_ep_offsets   per rank: where each of its sorted rows lands on its
//                   destination (dst_off[E]), its local experts' row ranges
//                   (loc_off[El+1]) and every source's sorted offsets
//                   (src_off[W, E]);
//   ib_ep_dispatch  copies each sorted row x[r] (expert e) to
//                   recv[dest(e)][dst_off[e] + r - offsets[e]] with 16-byte
//                   peer stores, then the last CTA adds 1 to an arrival
//                   counter on every rank;
//   ib_ep_dispatch_q the same for e4m3 rows plus their UE8M0 scale columns
//                   (the sender quantised them; half the bytes of bf16);
//   ib_ep_dispatch_ex / ib_ep_dispatch_q_ex: the same, plus per-expert
//                   arrival counters: when the last row of (this source,
//                   expert e) has been stored, its destination's counter of
//                   local expert e grows by 1 (experts this source sends no
//                   rows to are signalled at once), so the destination's up
//                   projection starts an expert's tiles as soon as that
//                   expert's rows from every source are in;
//   ib_ep_wait      waits (bounded, 2 s) until all W arrivals of a round are in
//                   (the up projection can instead wait inside its own
//                   producer: ib_gemm_grouped_wait);
//   ib_ep_return    copies each expert-output row p < loc_off[El] (local
//                   expert e, source s) back to ret[s][src_off[s][e] + (p -
//                   start of (e, s))], then signals like the dispatch.
//
// Waits are bounded by %globaltimer; on timeout a status word is set and
// the kernel returns, so a dead rank turns into an error, not a hang.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ib200 {
namespace ep {

constexpr int kMaxRanks = 8;
constexpr int kStatusTimeoutEp = 0x4201;
constexpr unsigned long long kWaitNs = 2000000000ull;

struct Peers {
  void* buf[kMaxRanks];            // recv (dispatch) or ret (return) base on each rank
  unsigned int* flag[kMaxRanks];   // arrival counter on each rank for this phase
  unsigned int* eflag[kMaxRanks];  // per-local-expert arrival counters on each rank (null: not used)
};

// Per-expert arrival signalling of one dispatched row (every thread of the
// CTA calls it after its stores of the row): the row's stores are made
// visible system-wide, counted in local_done[e], and the CTA that stores
// the last row of expert e bumps the destination's counter of e.
__device__ __forceinline__ void row_landed(const Peers& pr, unsigned int* local_done, const int* offsets, int e,
                                           int El) {
  if (pr.eflag[0] == nullptr) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int n_e = static_cast<unsigned int>(offsets[e + 1] - offsets[e]);
    if (atomicAdd(&local_done[e], 1u) == n_e - 1) {
      local_done[e] = 0;  // no other increment of e this round
      __threadfence_system();
      const int d = e / El;
      atomicAdd_system(pr.eflag[d] + (e - d * El), 1u);
    }
  }
}

// experts this source sends nothing to are complete from the start
__device__ __forceinline__ void signal_empty_experts(const Peers& pr, const int* offsets, int E, int El) {
  if (pr.eflag[0] == nullptr || blockIdx.x != 0) return;
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    if (offsets[e + 1] == offsets[e]) {
      const int d = e / El;
      atomicAdd_system(pr.eflag[d] + (e - d * El), 1u);
    }
}

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// single block; W * E <= blockDim-friendly sizes (E <= 1024, W <= 8)
__global__ void offsets_kernel(const int* __restrict__ C, int W, int E, int rank, int* __restrict__ dst_off,
                               int* __restrict__ loc_off, int* __restrict__ src_off) {
  const int El = E / W;
  // src_off[s, e] = sum_{e' < e} C[s][e']
  for (int s = threadIdx.x; s < W; s += blockDim.x) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      src_off[s * E + e] = acc;
      acc += C[s * E + e];
    }
  }
  // dst_off[e] for this rank as the source: the block of expert e on its
  // destination starts after the destination's earlier local experts (all
  // sources) and after the lower-ranked sources of expert e
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int d = e / El;
    int acc = 0;
    for (int e2 = d * El; e2 < e; ++e2)
      for (int s = 0; s < W; ++s) acc += C[s * E + e2];
    for (int s = 0; s < rank; ++s) acc += C[s * E + e];
    dst_off[e] = acc;
  }
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int el = 0; el < El; ++el) {
      loc_off[el] = acc;
      for (int s = 0; s < W; ++s) acc += C[s * E + rank * El + el];
    }
    loc_off[El] = acc;
  }
}

__device__ __forceinline__ int find_bin(const int* __restrict__ off, int n, int r) {
  // largest e with off[e] <= r (off[0] = 0, non-decreasing, n + 1 entries)
  int lo = 0, hi = n;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (off[mid] <= r) lo = mid;
    else hi = mid;
  }
  return lo;
}

__device__ __forceinline__ void signal_all(unsigned int* done_ctr, const Peers& pr, int world) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(done_ctr, 1u) == gridDim.x - 1) {
      *done_ctr = 0;
      __threadfence_system();
      for (int d = 0; d < world; ++d) atomicAdd_system(pr.flag[d], 1u);
    }
  }
}

// one CTA per group of rows; rows are H bf16 (H * 2 % 16 == 0)
__global__ void __launch_bounds__(256) dispatch_kernel(const uint4* __restrict__ x, int rows, int vec_per_row,
                                                       const int* __restrict__ offsets, int E, int El,
                                                       const int* __restrict__ dst_off, Peers pr, int world,
                                                       unsigned int* done_ctr, unsigned int* local_done) {
  signal_empty_experts(pr, offsets, E, El);
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int e = find_bin(offsets, E, r);
    const int d = e / El;
    const long long pos = static_cast<long long>(dst_off[e]) + (r - offsets[e]);
    uint4* dst = static_cast<uint4*>(pr.buf[d]) + pos * vec_per_row;
    const uint4* src = x + static_cast<long long>(r) * vec_per_row;
    for (int i = threadIdx.x; i < vec_per_row; i += blockDim.x) dst[i] = __ldg(src + i);
    row_landed(pr, local_done, offsets, e, El);
  }
  signal_all(done_ctr, pr, world);
}

// fp8 dispatch: the sender quantised its sorted rows (e4m3 rows of
// vec_per_row 16-byte vectors, UE8M0 scales sf [n_groups, sf_ld], one
// column per row); each row and its n_groups scale bytes go to the same
// place on the destination (recv rows, recv_sf [n_groups, recv_sf_ld]), so
// the receiver's fp8 grouped GEMM reads them without a quantisation pass.
__global__ void __launch_bounds__(256) dispatch_q_kernel(const uint4* __restrict__ x, int rows, int vec_per_row,
                                                         const uint8_t* __restrict__ sf, int sf_ld, int n_groups,
                                                         const int* __restrict__ offsets, int E, int El,
                                                         const int* __restrict__ dst_off, Peers pr, Peers psf,
                                                         int recv_sf_ld, int world, unsigned int* done_ctr,
                                                         unsigned int* local_done) {
  signal_empty_experts(pr, offsets, E, El);
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const int e = find_bin(offsets, E, r);
    const int d = e / El;
    const long long pos = static_cast<long long>(dst_off[e]) + (r - offsets[e]);
    uint4* dst = static_cast<uint4*>(pr.buf[d]) + pos * vec_per_row;
    const uint4* src = x + static_cast<long long>(r) * vec_per_row;
    for (int i = threadIdx.x; i < vec_per_row; i += blockDim.x) dst[i] = __ldg(src + i);
    uint8_t* dsf = static_cast<uint8_t*>(psf.buf[d]);
    for (int g = threadIdx.x; g < n_groups; g += blockDim.x)
      dsf[static_cast<long long>(g) * recv_sf_ld + pos] = __ldg(sf + static_cast<long long>(g) * sf_ld + r);
    row_landed(pr, local_done, offsets, e, El);
  }
  signal_all(done_ctr, pr, world);
}

__global__ void __launch_bounds__(256) return_kernel(const uint4* __restrict__ y, int rows, int vec_per_row,
                                                     const int* __restrict__ C, int W, int E, int El, int rank,
                                                     const int* __restrict__ loc_off,
                                                     const int* __restrict__ src_off, Peers pr,
                                                     unsigned int* done_ctr) {
  const int nrows = min(rows, loc_off[El]);  // rows actually received this round
  for (int p = blockIdx.x; p < nrows; p += gridDim.x) {
    const int el = find_bin(loc_off, El, p);
    const int e = rank * El + el;
    int rel = p - loc_off[el];
    int s = 0;
    while (s < W - 1 && rel >= C[s * E + e]) {
      rel -= C[s * E + e];
      ++s;
    }
    const long long src_row = static_cast<long long>(src_off[s * E + e]) + rel;
    uint4* dst = static_cast<uint4*>(pr.buf[s]) + src_row * vec_per_row;
    const uint4* src = y + static_cast<long long>(p) * vec_per_row;
    for (int i = threadIdx.x; i < vec_per_row; i += blockDim.x) dst[i] = __ldg(src + i);
  }
  signal_all(done_ctr, pr, W);
}

// row_map[p] = (source rank << 27) | (row in the source's sorted rows) for
// every received row p < loc_off[El] (the return_kernel's mapping, for a
// GEMM epilogue that stores its outputs straight to the sources)
__global__ void row_map_kernel(int rows, const int* __restrict__ C, int W, int E, int El, int rank,
                               const int* __restrict__ loc_off, const int* __restrict__ src_off,
                               int* __restrict__ row_map) {
  const int nrows = min(rows, loc_off[El]);
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < nrows; p += gridDim.x * blockDim.x) {
    const int el = find_bin(loc_off, El, p);
    const int e = rank * El + el;
    int rel = p - loc_off[el];
    int s = 0;
    while (s < W - 1 && rel >= C[s * E + e]) {
      rel -= C[s * E + e];
      ++s;
    }
    row_map[p] = (s << 27) | (src_off[s * E + e] + rel);
  }
}

__global__ void wait_kernel(const unsigned int* flag, unsigned int target, int* status, unsigned long long limit_ns) {
  if (threadIdx.x != 0) return;
  const unsigned long long t0 = gtimer();
  while (ld_acquire_sys(flag) < target) {
    if (gtimer() - t0 > limit_ns) {
      atomicCAS(status, 0, kStatusTimeoutEp);
      return;
    }
  }
}

}  // namespace ep
}  // namespace ib200

using namespace ib200::ep;

extern "C" int ib_ep_offsets(const int* C, int W, int E, int rank, int* dst_off, int* loc_off, int* src_off,
                             cudaStream_t stream) {
  if (W < 1 || W > kMaxRanks || E % W) return -1;
  offsets_kernel<<<1, 256, 0, stream>>>(C, W, E, rank, dst_off, loc_off, src_off);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

// peer_buf / peer_flag: host arrays of `world` device pointers
// peer_eflag (null: no per-expert counters): each rank's per-local-expert
// counters; local_done: E zeroed counters of this rank (reset by the kernel)
extern "C" int ib_ep_dispatch_ex(const void* x, int rows, int H, const int* offsets, int E, int world,
                                 const int* dst_off, void* const* peer_buf, unsigned int* const* peer_flag,
                                 unsigned int* const* peer_eflag, unsigned int* local_done, unsigned int* done_ctr,
                                 cudaStream_t stream) {
  if (world < 1 || world > kMaxRanks || (H * 2) % 16) return -1;
  if (peer_eflag != nullptr && local_done == nullptr) return -1;
  Peers pr{};
  for (int d = 0; d < world; ++d) {
    pr.buf[d] = peer_buf[d];
    pr.flag[d] = peer_flag[d];
    pr.eflag[d] = peer_eflag != nullptr ? peer_eflag[d] : nullptr;
  }
  const int grid = rows < 1 ? 1 : (rows < 2048 ? rows : 2048);
  dispatch_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint4*>(x), rows, H * 2 / 16, offsets, E, E / world,
                                            dst_off, pr, world, done_ctr, local_done);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

extern "C" int ib_ep_dispatch(const void* x, int rows, int H, const int* offsets, int E, int world,
                              const int* dst_off, void* const* peer_buf, unsigned int* const* peer_flag,
                              unsigned int* done_ctr, cudaStream_t stream) {
  return ib_ep_dispatch_ex(x, rows, H, offsets, E, world, dst_off, peer_buf, peer_flag, nullptr, nullptr, done_ctr,
                           stream);
}

// fp8 rows (row_bytes % 16 == 0) with their scale columns; peer_sf: each
// rank's recv_sf base ([n_groups, recv_sf_ld] bytes)
extern "C" int ib_ep_dispatch_q_ex(const void* x, int rows, int row_bytes, const uint8_t* sf, int sf_ld,
                                   int n_groups, const int* offsets, int E, int world, const int* dst_off,
                                   void* const* peer_buf, void* const* peer_sf, int recv_sf_ld,
                                   unsigned int* const* peer_flag, unsigned int* const* peer_eflag,
                                   unsigned int* local_done, unsigned int* done_ctr, cudaStream_t stream) {
  if (world < 1 || world > kMaxRanks || row_bytes % 16 || n_groups < 0) return -1;
  if (peer_eflag != nullptr && local_done == nullptr) return -1;
  Peers pr{}, psf{};
  for (int d = 0; d < world; ++d) {
    pr.buf[d] = peer_buf[d];
    pr.flag[d] = peer_flag[d];
    pr.eflag[d] = peer_eflag != nullptr ? peer_eflag[d] : nullptr;
    psf.buf[d] = peer_sf[d];
  }
  const int grid = rows < 1 ? 1 : (rows < 2048 ? rows : 2048);
  dispatch_q_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint4*>(x), rows, row_bytes / 16, sf, sf_ld, n_groups,
                                              offsets, E, E / world, dst_off, pr, psf, recv_sf_ld, world, done_ctr,
                                              local_done);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

extern "C" int ib_ep_dispatch_q(const void* x, int rows, int row_bytes, const uint8_t* sf, int sf_ld, int n_groups,
                                const int* offsets, int E, int world, const int* dst_off, void* const* peer_buf,
                                void* const* peer_sf, int recv_sf_ld, unsigned int* const* peer_flag,
                                unsigned int* done_ctr, cudaStream_t stream) {
  return ib_ep_dispatch_q_ex(x, rows, row_bytes, sf, sf_ld, n_groups, offsets, E, world, dst_off, peer_buf, peer_sf,
                             recv_sf_ld, peer_flag, nullptr, nullptr, done_ctr, stream);
}

extern "C" int ib_ep_return(const void* y, int rows, int H, const int* C, int world, int E, int rank,
                            const int* loc_off, const int* src_off, void* const* peer_buf,
                            unsigned int* const* peer_flag, unsigned int* done_ctr, cudaStream_t stream) {
  if (world < 1 || world > kMaxRanks || (H * 2) % 16) return -1;
  Peers pr{};
  for (int d = 0; d < world; ++d) {
    pr.buf[d] = peer_buf[d];
    pr.flag[d] = peer_flag[d];
  }
  const int grid = rows < 1 ? 1 : (rows < 2048 ? rows : 2048);
  return_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint4*>(y), rows, H * 2 / 16, C, world, E, E / world,
                                          rank, loc_off, src_off, pr, done_ctr);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

extern "C" int ib_ep_wait(const unsigned int* flag, unsigned int target, int* status, cudaStream_t stream) {
  wait_kernel<<<1, 32, 0, stream>>>(flag, target, status, kWaitNs);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

// As ib_ep_wait with the wait bounded by limit_ns; on expiry *status gets
// 0x4201 (if it was 0) and the kernel returns.
extern "C" int ib_ep_wait_for(const unsigned int* flag, unsigned int target, int* status, unsigned long long limit_ns,
                              cudaStream_t stream) {
  wait_kernel<<<1, 32, 0, stream>>>(flag, target, status, limit_ns);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

extern "C" int ib_ep_row_map(const int* C, int W, int E, int rank, const int* loc_off, const int* src_off,
                             int rows, int* row_map, cudaStream_t stream) {
  if (W < 1 || W > kMaxRanks || E % W || rows <= 0) return rows <= 0 ? 0 : -1;
  const int grid = (rows + 255) / 256 < 1024 ? (rows + 255) / 256 : 1024;
  row_map_kernel<<<grid, 256, 0, stream>>>(rows, C, W, E, E / W, rank, loc_off, src_off, row_map);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}
