// Allocation-free C entry point for absorbed-MLA sparse decode attention.
//
// This entry point has no counterpart in the reference; it exists for callers that cannot allocate device memory
// on their own — for example a serving runtime that hands kernels only pre-registered buffers, code running while a
// memory pool is frozen, or a plain-C host without access to PyTorch's caching allocator.  Such callers pass inputs
// and outputs only; the split-K partial results this kernel needs live in a fixed 32 MiB array that the library
// reserves statically on every GPU that loads it, for the lifetime of the process.
//
// Contract:
//   * q   [T, H, 576] bf16, kv [S, 576] bf16 (the latent cache), idx [T, K] int32 slots (-1 = no key),
//     out [T, H, 512] bf16; all device pointers, contiguous; H <= 128.
//   * The key list is split across CTAs exactly as the allocating entry point does (the same split count, so both
//     produce bitwise-identical outputs); the scratch must hold T * splits * H * 514 floats, after a 256-byte status
//     word.  Larger problems are rejected with cudaErrorInvalidValue before any launch, and
//     cb_noalloc_last_error() says why.
//   * A return value of 0 means the kernels were launched.  The kernel's own waits are bounded; if one runs out the
//     kernel stops early, leaves `out` undefined and records an error code in the status word, which every call
//     resets to 0 on its stream.  cb_noalloc_status() copies that word back (it synchronises the stream): 0 means
//     the last call on this device completed normally.
//   * No cudaMalloc, cudaFree or allocating library routine is called.
//   * The first call on a device resolves the device address of the scratch array (cudaGetSymbolAddress) with that
//     device current; make that first call before any stream capture on that device.
//   * Every call shares the one scratch array and leaves the last call's partial sums in it.  Calls that can
//     overlap on the GPU (different streams without ordering between them) race on the scratch; order them.
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Returns a cudaError_t value (0 = success).
int cb_sparse_mla_noalloc(const void* q, int T, int H, const void* kv, int S, const int* idx, int K, float scale,
                          void* out, cudaStream_t stream);

// Status word of the last call on the current device (0 = ok; otherwise the kernel's bounded-wait error code).
// Synchronises `stream`.  Returns a cudaError_t value.
int cb_noalloc_status(cudaStream_t stream, int* kernel_status);

// Bytes of the static scratch array, and the message of the last rejected or failed call on this thread.
size_t cb_noalloc_scratch_bytes(void);
const char* cb_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
