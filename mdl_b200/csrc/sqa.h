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

// G queries per sample over one history that all of them share (keys = values = the
// history rows, no head slices): STCA's per-head score vectors W_K[g]^T (W_Q x)_g over the
// transformed history. dhist sums the G queries' gradients.
struct SqaSharedArgs {
  const float* q = nullptr;              // [B, G, D] fp32 queries
  const __nv_bfloat16* hist = nullptr;   // [B, L, D] bf16 history (D even)
  const int* kstart = nullptr;           // [B] first valid event
  float* ctx = nullptr;                  // [B, G, D] fp32 output
  float* lse = nullptr;                  // [B, G] log-sum-exp of the scaled scores (-inf: no valid event)
  const float* dctx = nullptr;           // backward: [B, G, D]
  float* dq = nullptr;                   // backward: [B, G, D]
  __nv_bfloat16* dhist = nullptr;        // backward: [B, L, D] (every event written)
  int B = 0, L = 0, G = 0, D = 0;
  float scale = 1.f;
};

// Shapes the shared-history kernels take: D even and at most 256, G at most 8, and
// G rounded up to 2, 4 or 8 times ceil(D / 64) rounded up to 1, 2 or 4 at most 16
// (register budget).
bool sqa_shared_supported(int G, int D);

cudaError_t sqa_fwd(const SqaArgs& a, cudaStream_t stream);
cudaError_t sqa_bwd(const SqaArgs& a, cudaStream_t stream);
cudaError_t sqa_shared_fwd(const SqaSharedArgs& a, cudaStream_t stream);
cudaError_t sqa_shared_bwd(const SqaSharedArgs& a, cudaStream_t stream);

}  // namespace mdl
