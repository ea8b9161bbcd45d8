// LayerNorm backward that allocates nothing.
//
// This entry point has no counterpart in the reference; it exists for callers of
// this library that are not allowed to allocate device memory while they run, for
// example code that executes inside a host callback or a framework hook that holds
// an allocator lock, a runtime that pre-plans all of its memory up front, or a C
// program that links the library without any allocator of its own. The regular
// path (mdl::layernorm_bwd) needs a caller-provided `partials` buffer for the
// per-CTA partial sums of the gamma/beta gradients; this variant keeps those
// partial sums in a fixed device array that lives inside the library instead.
//
// Contract:
//   * Inputs and outputs are the caller's, exactly as for mdl::layernorm_bwd:
//     dy (or dy_bcast * bcast_scale), a, b, mean, rstd, gamma -> dx, dx2, and
//     dgamma / dbeta, which are ACCUMULATED into (+=), so zero them first if
//     you want the plain gradient.
//   * Scratch: one file-scope array of MDL_LN_BWD_NOALLOC_SCRATCH_BYTES bytes
//     (2 MiB) per GPU, held by every GPU that loads the library until the
//     process exits. The number of CTAs is capped so that their partial sums
//     fit; D must be a multiple of 8 and at most 2048 (the same limits as the
//     regular path), and one CTA keeps ((mix ? T : 0) + 16) * D fp32 values in
//     shared memory (the token-mixing staging and the per-warp gamma/beta
//     partial sums), which must fit the device's per-block opt-in limit
//     (227 KB on B200: D <= 3,632 without mixing; (T + 16) * D <= 58,112 with
//     it, e.g. T = 16 at D = 1,816). Anything else is rejected with an error
//     message.
//   * The first call on a device looks up the device address of the array
//     (cudaGetSymbolAddress, with that device current) and caches it; make that
//     first call before any stream capture on that device.
//   * Every call shares the one array and the array keeps whatever the last call
//     left in it. Each call overwrites all partial rows it later reads, so no
//     zeroing is needed, but calls whose executions overlap on the GPU (two
//     streams, or two host threads using the same device) race on the array
//     and must be serialised by the caller.
//   * No cudaMalloc, cudaFree or allocating library routine is called.
//
// Return value: 0 on success, -1 when the arguments are rejected (see
// mdl_noalloc_last_error()), otherwise the cudaError_t of the failing call.
#pragma once

#include <cuda_runtime.h>

#define MDL_LN_BWD_NOALLOC_SCRATCH_BYTES (2u * 1024u * 1024u)

#ifdef __cplusplus
extern "C" {
#endif

int mdl_layernorm_bwd_noalloc(const void* dy, const void* dy_bcast, float bcast_scale, const void* a, const void* b,
                              const float* mean, const float* rstd, const float* gamma, void* dx, void* dx2,
                              float* dgamma, float* dbeta, int B, int T, int D, int mix, cudaStream_t stream);

// Message of the last rejected call on this host thread ("" if none).
const char* mdl_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
