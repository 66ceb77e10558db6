// Tensor-parallel communication over NVLink peer memory.
//
// One-shot all-reduce fused into the row-parallel GEMM (ib_gemm_bf16_push in
// gemm_bf16.cu) and into the following residual-add + RMSNorm:
//
//   producer (every rank): out tile -> its receive slot on EVERY rank
//                          (peer stores over NVLink), then one arrival
//                          increment on every rank once the whole GEMM is
//                          stored (last-CTA pattern, system-scope fences)
//   consumer (every rank): wait until every rank's arrival counter has
//                          passed this round, then h += sum of the world
//                          partials (fp32), x = RMSNorm(h) * w
//
// Receive buffers and counters are double-buffered by "parity" (the two
// all-reduces of a layer alternate), which makes a reuse safe without a
// reverse handshake: a peer can only push round k+2 into this rank's parity
// buffer after it consumed round k+1, which needs this rank's push of
// round k+1, which this rank issues only after consuming round k.
//
// Every wait is bounded (2 s by %globaltimer); on timeout the kernel records
// a status code, skips its math and still completes its bookkeeping, so a
// rank that died leaves the others with an error status, not a hang.
//
// Symmetric memory: each rank cudaMalloc's its region and exports it with
// cudaIpcGetMemHandle; peers map it with cudaIpcOpenMemHandle (plain peer
// loads/stores, no multicast objects).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ib200 {
namespace tp {

constexpr int kStatusTimeoutArrive = 0x4101;
constexpr unsigned long long kWaitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float bf2f(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

constexpr int kMaxRanks = 8;

struct ArParams {
  const __nv_bfloat16* recv;  // this parity's receive region: [world][rows][ld]
  long long src_stride;       // elements between source slots
  int ld;
  const unsigned int* flags;  // [world] arrival counters (this parity)
  unsigned int* consumed;     // rounds consumed so far (this parity)
  unsigned int* fin_ctr;      // CTAs finished in this launch (zero between launches)
  int world, M, H;
  __nv_bfloat16* h;           // residual [M, H], updated in place
  const __nv_bfloat16* w;     // RMSNorm weight [H]
  float eps;
  __nv_bfloat16* x;           // normalized output [M, H]
  int* status;
  // two-shot (reduce-scatter) mode: this rank handles only its row blocks
  // ((row / 128) % world == rank), stores each normalised row into every
  // rank's x buffer and, once all its rows are out, bumps every rank's x
  // arrival counter
  int owner, rank;
  __nv_bfloat16* x_peer[kMaxRanks];
  unsigned int* x_flag[kMaxRanks];
};

template <int VPT>
__global__ void __launch_bounds__(256) ar_add_rmsnorm_kernel(const ArParams p) {
  __shared__ int s_ok;
  __shared__ float s_red[8];
  __shared__ unsigned int s_target;
  const int tid = threadIdx.x;
  if (tid == 0) {
    const unsigned int target = *reinterpret_cast<volatile unsigned int*>(p.consumed) + 1u;
    s_target = target;
    int ok = 1;
    const unsigned long long t0 = globaltimer();
    for (int src = 0; src < p.world && ok; ++src) {
      while (ld_acquire_sys(p.flags + src) < target) {
        if (globaltimer() - t0 > kWaitNs) {
          atomicCAS(p.status, 0, kStatusTimeoutArrive);
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  const int row = blockIdx.x;
  const bool mine = !p.owner || ((row >> 7) % p.world) == p.rank;
  if (s_ok && row < p.M && mine) {
    const int nvec = p.H / 8;
    float acc[VPT][8];
    float ss = 0.f;
    __nv_bfloat16* hrow = p.h + static_cast<size_t>(row) * p.H;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = tid + k * 256;
      if (v < nvec) {
        const uint4 hv = *reinterpret_cast<const uint4*>(hrow + v * 8);
        const uint16_t* hb = reinterpret_cast<const uint16_t*>(&hv);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[k][i] = 0.f;
        for (int src = 0; src < p.world; ++src) {
          const __nv_bfloat16* r = p.recv + src * p.src_stride + static_cast<size_t>(row) * p.ld + v * 8;
          const uint4 rv = *reinterpret_cast<const uint4*>(r);
          const uint16_t* rb = reinterpret_cast<const uint16_t*>(&rv);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[k][i] += bf2f(rb[i]);
        }
        uint4 out;
        uint32_t* o32 = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          // the residual is kept in bf16: round exactly as the stored value
          const __nv_bfloat162 s = __floats2bfloat162_rn(bf2f(hb[i]) + acc[k][i], bf2f(hb[i + 1]) + acc[k][i + 1]);
          o32[i / 2] = *reinterpret_cast<const uint32_t*>(&s);
          acc[k][i] = __low2float(s);
          acc[k][i + 1] = __high2float(s);
          ss += acc[k][i] * acc[k][i] + acc[k][i + 1] * acc[k][i + 1];
        }
        *reinterpret_cast<uint4*>(hrow + v * 8) = out;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) s_red[tid >> 5] = ss;
    __syncthreads();
    if (tid < 32) {
      float t = tid < 8 ? s_red[tid] : 0.f;
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
      if (tid == 0) s_red[0] = t;
    }
    __syncthreads();
    const float rstd = rsqrtf(s_red[0] / static_cast<float>(p.H) + p.eps);
    __nv_bfloat16* xrow = p.x + static_cast<size_t>(row) * p.H;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = tid + k * 256;
      if (v < nvec) {
        const uint4 wv = *reinterpret_cast<const uint4*>(p.w + v * 8);
        const uint16_t* wb = reinterpret_cast<const uint16_t*>(&wv);
        uint4 out;
        uint32_t* o32 = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
        for (int i = 0; i < 8; i += 2)
          o32[i / 2] = pack2(acc[k][i] * rstd * bf2f(wb[i]), acc[k][i + 1] * rstd * bf2f(wb[i + 1]));
        if (p.owner) {
          for (int d = 0; d < p.world; ++d)
            *reinterpret_cast<uint4*>(p.x_peer[d] + static_cast<size_t>(row) * p.H + v * 8) = out;
        } else {
          *reinterpret_cast<uint4*>(xrow + v * 8) = out;
        }
      }
    }
  }
  if (p.owner) __threadfence_system();  // the broadcast rows before the arrival signal
  // bookkeeping: the last CTA marks this round consumed
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(p.fin_ctr, 1u) == gridDim.x - 1) {
      *p.fin_ctr = 0;
      *reinterpret_cast<volatile unsigned int*>(p.consumed) = s_target;
      __threadfence_system();
      if (p.owner)
        for (int d = 0; d < p.world; ++d) atomicAdd_system(p.x_flag[d], 1u);
    }
  }
}

// Bounded wait until *flag >= target (the x rows of every owner arrived).
__global__ void tp_wait_kernel(const unsigned int* flag, unsigned int target, int* status,
                               unsigned long long limit_ns) {
  if (threadIdx.x != 0) return;
  const unsigned long long t0 = globaltimer();
  while (ld_acquire_sys(flag) < target) {
    if (globaltimer() - t0 > limit_ns) {
      atomicCAS(status, 0, kStatusTimeoutArrive);
      return;
    }
  }
}

// Bounded wait until *flag >= *consumed + inc, then *consumed advances by
// inc. The target lives in device memory, so a CUDA graph that replays this
// launch waits for each replay's own arrivals (a host-side target would be
// frozen into the graph).
__global__ void tp_wait_next_kernel(const unsigned int* flag, unsigned int* consumed, unsigned int inc, int* status,
                                    unsigned long long limit_ns) {
  if (threadIdx.x != 0) return;
  const unsigned int target = *reinterpret_cast<volatile unsigned int*>(consumed) + inc;
  const unsigned long long t0 = globaltimer();
  while (ld_acquire_sys(flag) < target) {
    if (globaltimer() - t0 > limit_ns) {
      atomicCAS(status, 0, kStatusTimeoutArrive);
      break;
    }
  }
  *reinterpret_cast<volatile unsigned int*>(consumed) = target;
}

}  // namespace tp
}  // namespace ib200

using namespace ib200::tp;

extern "C" int ib_ar_add_rmsnorm(const void* recv, long long src_stride, int ld, const unsigned int* flags,
                                 unsigned int* consumed, unsigned int* fin_ctr, int world, int M, int H, void* h,
                                 const void* w, float eps, void* x, int* status, cudaStream_t stream) {
  if (M <= 0) return 0;
  if ((H % 8) != 0 || (ld % 8) != 0 || H > 8 * 256 * 8 || world < 1) return -1;
  ArParams p;
  p.recv = static_cast<const __nv_bfloat16*>(recv);
  p.src_stride = src_stride;
  p.ld = ld;
  p.flags = flags;
  p.consumed = consumed;
  p.fin_ctr = fin_ctr;
  p.world = world;
  p.M = M;
  p.H = H;
  p.h = static_cast<__nv_bfloat16*>(h);
  p.w = static_cast<const __nv_bfloat16*>(w);
  p.eps = eps;
  p.x = static_cast<__nv_bfloat16*>(x);
  p.status = status;
  p.owner = 0;
  p.rank = 0;
  const int vpt = (H / 8 + 255) / 256;
  if (vpt <= 2) ar_add_rmsnorm_kernel<2><<<M, 256, 0, stream>>>(p);
  else if (vpt <= 4) ar_add_rmsnorm_kernel<4><<<M, 256, 0, stream>>>(p);
  else ar_add_rmsnorm_kernel<8><<<M, 256, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

// ---------------------------------------------------------------------------
// symmetric memory via CUDA IPC

extern "C" int ib_sym_alloc(size_t bytes, void** out) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return static_cast<int>(e);
  }
  *out = p;
  return 0;
}

extern "C" int ib_sym_free(void* p) { return static_cast<int>(cudaFree(p)); }

extern "C" int ib_ipc_handle(void* p, void* out64) {
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) return static_cast<int>(e);
  static_assert(sizeof(h) == 64, "CUDA IPC handle is 64 bytes");
  memcpy(out64, &h, sizeof(h));
  return 0;
}

extern "C" int ib_ipc_open(const void* h64, void** out) {
  cudaIpcMemHandle_t h;
  memcpy(&h, h64, sizeof(h));
  return static_cast<int>(cudaIpcOpenMemHandle(out, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int ib_ipc_close(void* p) { return static_cast<int>(cudaIpcCloseMemHandle(p)); }

extern "C" int ib_can_access_peer(int dev, int peer) {
  int ok = 0;
  cudaDeviceCanAccessPeer(&ok, dev, peer);
  return ok;
}

// Let kernels on the current device access `peer`'s memory directly (one
// process driving two GPUs). Already-enabled counts as success.
extern "C" int ib_enable_peer_access(int peer) {
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return 0;
  }
  return static_cast<int>(e);
}

// Two-shot consumer: like ib_ar_add_rmsnorm for this rank's row blocks only
// (h holds valid rows only there); the normalised rows go to x_peer[d] on
// every rank d, then every rank's x_flag[d] is incremented once.
extern "C" int ib_ar_add_rmsnorm_rs(const void* recv, long long src_stride, int ld, const unsigned int* flags,
                                    unsigned int* consumed, unsigned int* fin_ctr, int world, int rank, int M, int H,
                                    void* h, const void* w, float eps, void* const* x_peer,
                                    unsigned int* const* x_flag, int* status, cudaStream_t stream) {
  if (M <= 0) return 0;
  if ((H % 8) != 0 || (ld % 8) != 0 || H > 8 * 256 * 8 || world < 1 || world > kMaxRanks) return -1;
  ArParams p;
  p.recv = static_cast<const __nv_bfloat16*>(recv);
  p.src_stride = src_stride;
  p.ld = ld;
  p.flags = flags;
  p.consumed = consumed;
  p.fin_ctr = fin_ctr;
  p.world = world;
  p.M = M;
  p.H = H;
  p.h = static_cast<__nv_bfloat16*>(h);
  p.w = static_cast<const __nv_bfloat16*>(w);
  p.eps = eps;
  p.x = nullptr;
  p.status = status;
  p.owner = 1;
  p.rank = rank;
  for (int d = 0; d < kMaxRanks; ++d) {
    p.x_peer[d] = d < world ? static_cast<__nv_bfloat16*>(x_peer[d]) : nullptr;
    p.x_flag[d] = d < world ? x_flag[d] : nullptr;
  }
  const int vpt = (H / 8 + 255) / 256;
  if (vpt <= 2) ar_add_rmsnorm_kernel<2><<<M, 256, 0, stream>>>(p);
  else if (vpt <= 4) ar_add_rmsnorm_kernel<4><<<M, 256, 0, stream>>>(p);
  else ar_add_rmsnorm_kernel<8><<<M, 256, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

extern "C" int ib_tp_wait(const unsigned int* flag, unsigned int target, int* status, cudaStream_t stream) {
  tp_wait_kernel<<<1, 32, 0, stream>>>(flag, target, status, ib200::tp::kWaitNs);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

// Graph-safe form (see tp_wait_next_kernel): waits for `inc` more arrivals
// than the previous call on the same `consumed` counter had.
extern "C" int ib_tp_wait_next(const unsigned int* flag, unsigned int* consumed, unsigned int inc, int* status,
                               cudaStream_t stream) {
  ib200::tp::tp_wait_next_kernel<<<1, 32, 0, stream>>>(flag, consumed, inc, status, ib200::tp::kWaitNs);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

// As ib_tp_wait with the wait bounded by limit_ns; on expiry *status gets
// 0x4101 (if it was 0) and the kernel returns.
extern "C" int ib_tp_wait_for(const unsigned int* flag, unsigned int target, int* status,
                              unsigned long long limit_ns, cudaStream_t stream) {
  tp_wait_kernel<<<1, 32, 0, stream>>>(flag, target, status, limit_ns);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}
