// Single-query attention over a head-interleaved history (sqa.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace mdl {

struct SqaArgs {
  const float* q = nullptr;              // [B, N, D] fp32 queries (key weight applied)
  const __nv_bfloat16* hist = nullptr;   // [B, L, N, D] bf16 history
  const int* kstart = nullptr;           // [B] first valid event (events before it are padding)
  float* ctx = nullptr;                  // [B, N, D] fp32 output
  float* lse = nullptr;                  // [B, N] log-sum-exp of the scaled scores (-inf: no valid event)
  const float* dctx = nullptr;           // backward: [B, N, D] upstream gradient
  float* dq = nullptr;                   // backward: [B, N, D]
  __nv_bfloat16* dhist = nullptr;        // backward: [B, L, N, D] (every event written)
  int B = 0, L = 0, N = 0, D = 0;
  float scale = 1.f;
};

cudaError_t sqa_fwd(const SqaArgs& a, cudaStream_t stream);
cudaError_t sqa_bwd(const SqaArgs& a, cudaStream_t stream);

}  // namespace mdl
