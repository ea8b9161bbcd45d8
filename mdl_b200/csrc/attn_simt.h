// Suffix attention on the CUDA cores for head widths 8, 16 and 64 (attn_simt.cu);
// same layouts and visibility as the tcgen05 flash attention of fmha.h.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace mdl {

struct AttnSimtArgs {
  const __nv_bfloat16* qkv = nullptr;  // [B, Lk, 3 * H * hd]
  const int* kstart = nullptr;          // [B] first valid key
  __nv_bfloat16* out = nullptr;         // [B, Lq, H * hd]
  float* lse = nullptr;                 // [B, H, Lq] base-2 log-sum-exp (+inf: no visible key)
  const __nv_bfloat16* dout = nullptr;  // backward: [B, Lq, H * hd]
  __nv_bfloat16* dqkv = nullptr;        // backward: [B, Lk, 3 * H * hd], every element written
  float* dsum = nullptr;                // backward workspace [B, H, Lq]
  int B = 0, H = 0, hd = 0, Lk = 0, Lq = 0;
  int causal = 1, ktail = 0, kexcl = 0;
  float scale = 1.f;                    // softmax scale (1/sqrt(hd) by convention)
};

bool attn_simt_supported(int hd);
cudaError_t attn_simt_fwd(const AttnSimtArgs& a, cudaStream_t stream);
cudaError_t attn_simt_bwd(const AttnSimtArgs& a, cudaStream_t stream);

}  // namespace mdl
