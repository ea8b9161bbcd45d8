// Host interface of the attention kernels.
#pragma once

#include <cuda_runtime.h>

namespace mdl {

// Few-query multi-head attention (MDL domain tokens over feature tokens,
// reference DomainAwareAttention src/modules/attention.py:425-512 via SDPA):
//   O[b, q, h*hd:(h+1)*hd] = softmax(Q_bh K_bh^T * scale [+ mask]) V_bh
// Q: [B, Nq, D] bf16 (row stride ldq), K/V: [B, Nk, D] bf16 (row stride ldk),
// O: [B, Nq, D] bf16, lse: [B, H, Nq] fp32 (saved for the backward).
// key_valid (optional): int32 [B] number of valid keys per sample (keys past it
// are masked; a sample with no valid key gets zeros).
// One CTA per (b, h); Nq, Nk <= 64, hd <= 128.
struct SmallAttnArgs {
  const void* q = nullptr;
  const void* k = nullptr;
  const void* v = nullptr;
  void* o = nullptr;
  float* lse = nullptr;
  const int* key_valid = nullptr;
  // backward
  const void* dout = nullptr;
  void* dq = nullptr;
  void* dk = nullptr;
  void* dv = nullptr;
  long long ldq = 0, ldk = 0, ldo = 0;      // row strides (elements) of Q, K/V, O
  long long bsq = 0, bsk = 0, bso = 0;      // batch strides
  int B = 0, Nq = 0, Nk = 0, H = 0, hd = 0;
  float scale = 1.f;
};
cudaError_t small_attention_fwd(const SmallAttnArgs& a, cudaStream_t stream);
cudaError_t small_attention_bwd(const SmallAttnArgs& a, cudaStream_t stream);

}  // namespace mdl
