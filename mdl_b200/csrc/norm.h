// Host interface of the fused normalisation kernels.
#pragma once

#include <cuda_runtime.h>

namespace mdl {

// Rows are grouped as [B, T, D] (T <= 32, D % 8 == 0, D <= 2048).
//   mix = 1: v[b,i,:] = mix(a)[b,i,:] + a[b,i,:]   (RankMixer token mixing, dh = D/T, dh % 8 == 0)
//            mix(a)[b,i,j*dh+w] = a[b,j,i*dh+w]
//   mix = 0: v = a + b (b may be null)
//   out = LayerNorm(v) * gamma + beta  (bf16), mean/rstd saved (fp32 [B*T]).
struct LNFwdArgs {
  const void* a = nullptr;
  const void* b = nullptr;
  const float* gamma = nullptr;
  const float* beta = nullptr;
  void* out = nullptr;
  float* mean = nullptr;
  float* rstd = nullptr;
  int B = 0, T = 0, D = 0, mix = 0;
  float eps = 1e-5f;
};
cudaError_t layernorm_fwd(const LNFwdArgs& a, cudaStream_t stream);

// Backward of the above. dy is [B,T,D] bf16, or (dy == null) dy[b,t,:] =
// dy_bcast[b,:] * bcast_scale (backward of a mean over tokens).
//   dx  = (mix ? dv + mix(dv) : dv) + res  (bf16; res optional, [B*T, D] bf16: a residual
//                                           gradient added in the same pass)
//   dx2 = dx without res (optional second copy, bf16)
// gamma/beta gradients are written as per-CTA partial sums into `partials`
// ([grid, 2 * D] fp32) and folded by a second kernel into dgamma and dbeta (+=).
struct LNBwdArgs {
  const void* dy = nullptr;
  const void* dy_bcast = nullptr;
  float bcast_scale = 1.f;
  const void* a = nullptr;
  const void* b = nullptr;
  const float* mean = nullptr;
  const float* rstd = nullptr;
  const float* gamma = nullptr;
  void* dx = nullptr;
  void* dx2 = nullptr;
  const void* res = nullptr;
  float* partials = nullptr;
  float* dgamma = nullptr;
  float* dbeta = nullptr;
  int B = 0, T = 0, D = 0, mix = 0;
  int grid = 0;  // number of CTAs (partials rows); 0 = choose
};
int layernorm_bwd_grid(int B);
// Dynamic shared memory of one backward CTA: the [T][D] dv staging of token mixing
// (mix only) plus the [8 warps][2][D] gamma/beta partial sums, fp32.
size_t layernorm_bwd_smem(int T, int D, int mix);
cudaError_t layernorm_bwd(const LNBwdArgs& a, cudaStream_t stream);

// RMSNorm over rows of width D (fp32 statistics, reference src/model.py:4550-4568):
//   out = x * rsqrt(mean(x^2) + eps) * weight
struct RMSArgs {
  const void* x = nullptr;
  const float* weight = nullptr;
  void* out = nullptr;
  float* rstd = nullptr;
  const void* dy = nullptr;
  void* dx = nullptr;
  float* dweight = nullptr;  // fp32 [D] (+=)
  // optional residual gradient added to dx: rows come in samples of res_period
  // rows; the last res_tail rows of each sample add dres row (sample * res_tail
  // + row - (res_period - res_tail)). res_period == 0: dres has dx's layout.
  const void* dres = nullptr;
  int res_period = 0, res_tail = 0;
  long long rows = 0;
  int D = 0;
  float eps = 1e-6f;
};
cudaError_t rmsnorm_fwd(const RMSArgs& a, cudaStream_t stream);
cudaError_t rmsnorm_bwd(const RMSArgs& a, cudaStream_t stream);

}  // namespace mdl
