// Allocation-free variant of the paged decode-attention entry point.
//
// This entry point has no counterpart in the reference project; it exists for
// callers of this library that cannot allocate device memory themselves.
//
// Who needs it: code that runs where cudaMalloc is off limits or harmful -
// plugins hosted by an inference server or framework that owns every byte of
// device memory through its own pool and caps (a raw cudaMalloc there escapes
// that accounting and can fail under the cap), latency-critical paths where
// cudaMalloc/cudaFree would synchronise the device, and host code that simply
// has no allocator to hand the split-KV partial buffers to. Such a caller
// passes only its inputs and its output; the partial results of the split-KV
// reduction live in a fixed-size array inside this library.
//
// Contract:
//  * Scratch: one file-scope device array of IB_DECODE_NOALLOC_MAX_ROWS rows
//    of 128 floats plus one float per row (a little over 8 MiB). Every GPU
//    on which the library is used holds it until the process exits.
//  * Limit: B * num_q_heads * splits must not exceed
//    IB_DECODE_NOALLOC_MAX_ROWS; larger calls return IB_DECODE_NOALLOC_TOO_BIG
//    and launch nothing. splits == 1 needs no scratch and has no limit.
//  * First call on a device: the call looks up the device address of the
//    scratch array (cudaGetSymbolAddress, with that device current) and
//    caches it. Make that first call outside any stream capture.
//  * Sharing: every call on a device uses the same scratch array, which keeps
//    the last call's partials. Calls whose kernels overlap on the GPU (for
//    example on two streams without ordering between them) race on it;
//    serialise them. Nothing in the scratch needs to start at zero: every
//    split writes its own slot before the combine reads it.
//  * The call allocates nothing: no cudaMalloc, cudaFree or allocating
//    library routine.
//
// Arguments match ib_attn_decode minus its two scratch pointers. Returns 0 on
// success, a negative code for bad arguments, or a CUDA error code.
#pragma once

#include <cuda_runtime.h>

#define IB_DECODE_NOALLOC_MAX_ROWS 16384
#define IB_DECODE_NOALLOC_TOO_BIG (-3)
#define IB_DECODE_NOALLOC_SETUP_FAILED (-4)

#ifdef __cplusplus
extern "C" {
#endif

int ib_attn_decode_noalloc(const void* q, int ldq, const void* k_cache, const void* v_cache,
                           const int* block_table, const int* bt_rows, const int* seq_lens, int max_pages, int B,
                           int hq, int hkv, int splits, float scale, void* out, int ldo, cudaStream_t stream);

// The row limit above, for callers that size their batches at run time.
int ib_attn_decode_noalloc_max_rows(void);

#ifdef __cplusplus
}
#endif
