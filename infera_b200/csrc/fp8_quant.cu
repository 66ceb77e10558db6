// Activation quantisation for the W8A8 GEMMs: bf16 rows -> e4m3 with one
// UE8M0 (power-of-two) scale per token and 128-wide K group.
//
//   e   = smallest integer with amax / 2^e <= 448 (e4m3's largest finite
//         value), clamped to [-126, 126]; 0 for an all-zero group
//   q   = e4m3(x * 2^-e)  (round to nearest even, saturating)
//   sf  = e + 127         (stored K-group-major: sf[g * ld_sf + m])
//
// One warp per (token, group): 32 lanes x 4 elements. The K-group-major
// scale layout lets the GEMM's scale-staging warps read 32 consecutive
// tokens of one group with one coalesced load.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ib200 {
namespace q8 {

__device__ __forceinline__ int ue8m0_exp(float amax) {
  if (!(amax > 0.f)) return 0;
  const float r = amax / 448.0f;
  const uint32_t b = __float_as_uint(r);
  int e = static_cast<int>((b >> 23) & 0xffu) - 127;  // floor(log2 r) for normal r
  if (b & 0x7fffffu) e += 1;                          // round up unless r is a power of two
  return max(-126, min(126, e));
}

__device__ __forceinline__ float exp2_int(int e) { return __uint_as_float(static_cast<uint32_t>(127 + e) << 23); }

__global__ void __launch_bounds__(256) quant_act_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int M, int KG,
                                                        uint8_t* __restrict__ q, int ldq, uint8_t* __restrict__ sf,
                                                        int ldsf) {
  const int gw = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= M * KG) return;
  const int m = gw / KG;
  const int g = gw - m * KG;
  const uint2 v = *reinterpret_cast<const uint2*>(x + static_cast<size_t>(m) * ldx + g * 128 + lane * 4);
  float f[4] = {__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u), __uint_as_float(v.y << 16),
                __uint_as_float(v.y & 0xffff0000u)};
  float a = fmaxf(fmaxf(fabsf(f[0]), fabsf(f[1])), fmaxf(fabsf(f[2]), fabsf(f[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  const int e = ue8m0_exp(a);
  const float inv = exp2_int(-e);
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(f[0] * inv, f[1] * inv), __NV_SATFINITE,
                                                           __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(f[2] * inv, f[3] * inv), __NV_SATFINITE,
                                                           __NV_E4M3);
  *reinterpret_cast<uint32_t*>(q + static_cast<size_t>(m) * ldq + g * 128 + lane * 4) =
      static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  if (lane == 0) sf[static_cast<size_t>(g) * ldsf + m] = static_cast<uint8_t>(e + 127);
}

}  // namespace q8
}  // namespace ib200

// x bf16 [M, K] (row pitch ldx elements, a multiple of 4), K % 128 == 0;
// q e4m3 [M, ldq]; sf uint8 [K/128, ldsf] with ldsf >= M.
extern "C" int ib_quant_fp8_act(const void* x, int ldx, int M, int K, void* q, int ldq, void* sf, int ldsf,
                                cudaStream_t stream) {
  if (M <= 0) return 0;
  if ((K % 128) != 0 || (ldx % 4) != 0 || (ldq % 4) != 0 || ldsf < M) return -1;
  const int KG = K / 128;
  const long long warps = static_cast<long long>(M) * KG;
  const int grid = static_cast<int>((warps + 7) / 8);
  ib200::q8::quant_act_kernel<<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), ldx, M, KG,
                                                        static_cast<uint8_t*>(q), ldq, static_cast<uint8_t*>(sf),
                                                        ldsf);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}
