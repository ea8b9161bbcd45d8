// Host interface of the NVLink symmetric-memory runtime and the fused
// collective kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "embedding.h"  // kMaxWorld

namespace mdl {

// ---- CUDA IPC buffers (one allocation per rank, mapped by every peer)
cudaError_t ipc_alloc(size_t bytes, void** ptr, cudaIpcMemHandle_t* handle);
cudaError_t ipc_open(const cudaIpcMemHandle_t& handle, void** ptr);
cudaError_t ipc_close(void* ptr);
cudaError_t ipc_free(void* ptr);

// ---- device-side barrier over peer signal words.
// signals[r] points at rank r's signal array (uint32[kMaxWorld]); counter is a
// local uint32 that the kernel increments, so the same launch can be replayed
// from a CUDA graph. Waits are bounded (error word + early return).
void set_barrier_limit_ns(uint64_t ns);
cudaError_t symm_barrier(unsigned* const* signals, unsigned* counter, int rank, int world, int* err,
                         cudaStream_t stream);

// ---- fused dense gradient all-reduce + optimizer (DDP replacement)
// Over the element range [begin, end) of a flat fp32 gradient buffer that
// every rank holds (grads[r] = rank r's buffer), rank `rank` owns the slice
// [begin + rank*chunk, ...) of each 1024-element-aligned partition. For each
// owned element it sums the peers' gradients (P2P loads over NVLink), scales by
// grad_scale, applies Adam or RMSprop to its fp32 master copy and optimizer
// state, and stores the updated bf16 shadow weight into EVERY rank's shadow
// buffer (P2P stores); elements >= fp32_from are also stored as fp32 into every
// rank's master copy. The result equals an all-reduce(mean) followed by the
// optimizer on every rank (DDP semantics, reference src/train.py:5311-5324).
struct DenseSyncArgs {
  float* grads[kMaxWorld] = {};
  float* params[kMaxWorld] = {};
  void* shadows[kMaxWorld] = {};   // bf16
  float* state1 = nullptr;         // local full-size state (only the owned slice is touched)
  float* state2 = nullptr;
  long long begin = 0, end = 0;
  long long fp32_from = 0;
  int world = 1, rank = 0;
  int optimizer = 0;               // 0 adam, 1 rmsprop
  float lr = 0.f, beta1 = 0.9f, beta2 = 0.999f, eps = 1e-8f, weight_decay = 0.f;
  float bias_correction1 = 1.f, bias_correction2 = 1.f, alpha = 0.99f;
  float grad_scale = 1.f;
  const float* clip = nullptr;
  float* sqnorm_out = nullptr;     // phase "norm": sum of squares of the reduced slice
  int phase = 0;                   // 0: fused update, 1: only reduce -> local grad slice + sqnorm
  int max_blocks = 0;              // grid cap (0: fill the GPU) when running beside other kernels
  // NVLS (NVSwitch multicast) variant: multicast addresses of the grad / master /
  // shadow buffers. When mc_grad is set, the owned slice's gradient is summed in the
  // switch (multimem.ld_reduce) and the updated weights are written to every rank
  // with one multicast store (multimem.st); grads/params/shadows then only need this
  // rank's own entries.
  float* mc_grad = nullptr;
  float* mc_master = nullptr;
  void* mc_shadow = nullptr;
};
cudaError_t dense_sync_update(const DenseSyncArgs& a, cudaStream_t stream);

// Sum-all-reduce of a small fp32 vector over peer buffers (one CTA, used for
// loss/label counts and clip norms). bufs[r] holds rank r's n values; every
// rank ends with the sum in its own buffer. Must be bracketed by barriers.
cudaError_t small_allreduce(float* const* bufs, float* out, int n, int world, cudaStream_t stream);

}  // namespace mdl
