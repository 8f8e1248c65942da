// Allocation-free C entry point of the rl_b200 native library.
//
// This entry point has no counterpart in the reference framework; it exists for
// callers of this library that cannot allocate device memory themselves:
//   * code embedded in a host runtime that owns all device memory (for example
//     a serving process that reserves the whole HBM at start-up, so any further
//     cudaMalloc fails or competes with its own pool), and
//   * latency-critical paths that must not risk the implicit device-wide
//     synchronisation that cudaMalloc / cudaFree can cause.
// Such callers pass only their inputs and outputs; the scratch the kernel needs
// lives in a fixed, statically sized device array inside this library.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Maximum sizes served by the static scratch array (4 MiB of fp32 per device).
#define RLB_NOALLOC_MAX_HIDDEN 8192
#define RLB_NOALLOC_MAX_CTAS 128

// RMSNorm backward for bf16 rows, without any device allocation.
//
//   dy, x : [rows, hidden] bf16, contiguous      (x is the forward input)
//   w     : [hidden] bf16                        (norm weight)
//   rstd  : [rows] fp32                          (1/rms saved by the forward)
//   dx    : [rows, hidden] bf16 output
//   dw    : [hidden] fp32 output (weight gradient, overwritten, not accumulated)
//   stream: CUDA stream to launch on (0 = legacy default stream)
//
// Returns 0 on success; a non-zero code otherwise, with a message available from
// rlb_noalloc_last_error().  Sizes beyond RLB_NOALLOC_MAX_HIDDEN are rejected.
//
// Scratch: per-CTA partial sums of dw live in one static __device__ array of
// RLB_NOALLOC_MAX_CTAS x RLB_NOALLOC_MAX_HIDDEN floats, which every GPU that
// loads this library holds until the process exits.  All calls share it, and
// every call fully overwrites the part it uses, so nothing needs clearing
// between calls - but calls whose executions overlap on the GPU (on different
// streams, or from different host threads without ordering) race on it.
//
// Set-up: the first call on each device looks up the device address of the
// scratch array (cudaGetSymbolAddress, with the caller's current device) and
// caches it; make that first call before any stream capture.  The caller must
// have the device that owns the pointers current.
//
// When the array is placed on a device: with CUDA's lazy module loading (the
// default since CUDA 12.2) the library's device code, and with it this 4 MiB
// array, is loaded onto a device at its first use there - the first call of
// this function on that device, not the load of the library.  A host runtime
// that reserves all free device memory for its own pool should therefore make
// one call (any valid size) on each device BEFORE reserving that pool;
// otherwise the first call can fail with an out-of-memory error.  Later calls
// on the same device allocate nothing.
int rlb_rmsnorm_bwd_noalloc(const void* dy, const void* x, const void* w, const float* rstd, void* dx, float* dw,
                            int rows, int hidden, cudaStream_t stream);

const char* rlb_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
