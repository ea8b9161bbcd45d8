// Host interface of the small fused kernels: token mean, column sums, the
// task-head logit + BCE kernel and the dense optimizers.
#pragma once

#include <cuda_runtime.h>

namespace mdl {

// out[b, :] = mean_t x[b, t, :]     (bf16 [B,T,D] -> bf16 [B,D])
cudaError_t token_mean_fwd(const void* x, void* out, int B, int T, int D, cudaStream_t stream);

// out[g, n] += scale * sum_m x[g*gs + m*ld + n]  (bf16 x, fp32 out)
// gs_out: element distance between the outputs of consecutive groups (-1: N;
// 0: every group adds into the same N sums).
cudaError_t colsum_bf16(const void* x, float* out, int G, long long M, int N, long long ld, long long gs,
                        float scale, cudaStream_t stream, long long gs_out = -1);

// Learned absolute positions over a prefix-padded token sequence (reference
// OneTransBackbone._add_unified_position_embeddings src/model.py:6151-6179):
//   x[b, e, :] += pos[e - kstart[b], :] for e >= kstart[b]      (bf16 x [B, L, D], fp32 pos)
// and its gradient dpos[p, :] += sum_b dx[b, kstart[b] + p, :]. D % 8 == 0.
cudaError_t position_add(void* x, const float* pos, const int* kstart, int B, int L, int D, cudaStream_t stream);
cudaError_t position_grad(const void* dx, float* dpos, const int* kstart, int B, int L, int D, cudaStream_t stream);

// Task heads, last layer + BCE (reference TaskHead src/model.py:869-882 and
// _loss_terms_from_batch src/train.py:5890-6031), one launch for all tasks:
//   z[b,t]   = act[b, t*H:(t+1)*H] . w2[t] + b2[t]
//   loss    += task_scale[t] * mask[b,t] * BCE(z, y)
//   dz       = task_scale[t] * mask[b,t] * (sigmoid(z) - y)
//   dpre[b, t*H+k] = dz * w2[t,k] * act'(pre[b, t*H+k])      (gelu or relu)
//   dw2[t]  += sum_b dz * act[b, t*H:...];  db2[t] += sum_b dz
struct HeadArgs {
  const void* act = nullptr;   // bf16 [B, ntask*H]
  const void* pre = nullptr;   // bf16 [B, ntask*H]
  const float* w2 = nullptr;   // [ntask, H]
  const float* b2 = nullptr;   // [ntask]
  const float* labels = nullptr;   // [B, ntask]
  const float* mask = nullptr;     // [B, ntask] or null
  const float* task_scale = nullptr;  // [ntask] device
  float* logits = nullptr;     // [B, ntask]
  float* loss = nullptr;       // scalar (+=)
  void* dpre = nullptr;        // bf16 [B, ntask*H]; null -> forward only
  float* dw2 = nullptr;        // [ntask, H] (+=)
  float* db2 = nullptr;        // [ntask] (+=)
  int B = 0, ntask = 0, H = 0;
  int relu = 0;                // activation of the hidden layer: 0 gelu, 1 relu
};
cudaError_t head_bce(const HeadArgs& a, cudaStream_t stream);

// Dense optimizers over one flat fp32 parameter buffer with an optional bf16
// shadow copy (the GEMM operand). Gradient scale and clip factor are applied
// on the fly: g = grad * grad_scale * (clip ? *clip : 1).
struct OptimArgs {
  float* param = nullptr;
  const float* grad = nullptr;
  float* state1 = nullptr;  // Adam m / RMSprop square_avg
  float* state2 = nullptr;  // Adam v
  void* shadow = nullptr;   // bf16 copy of param (optional)
  long long n = 0;
  float lr = 0.f, beta1 = 0.9f, beta2 = 0.999f, eps = 1e-8f, weight_decay = 0.f;
  float bias_correction1 = 1.f, bias_correction2 = 1.f;  // 1 - beta^t
  float alpha = 0.99f;      // RMSprop smoothing
  float grad_scale = 1.f;
  const float* clip = nullptr;
  bool zero_grad = false;   // write 0 to the gradient after reading it (fused zero_grad)
  int max_blocks = 0;       // cap on the grid (0: enough to fill the GPU) for runs beside other kernels
};
cudaError_t adam_step(const OptimArgs& a, cudaStream_t stream);
cudaError_t rmsprop_step(const OptimArgs& a, cudaStream_t stream);
// out[0] += sum(grad^2) * grad_scale^2
cudaError_t grad_sqnorm(const float* grad, long long n, float grad_scale, float* out, cudaStream_t stream);
// clip[0] = min(1, max_norm / (sqrt(sum_sq[0]) + 1e-6))
cudaError_t clip_factor(const float* sum_sq, float max_norm, float* clip, cudaStream_t stream);
// dst(bf16) = src(fp32)
cudaError_t cast_f32_bf16(const float* src, void* dst, long long n, cudaStream_t stream);
// Waits on an mbarrier that never completes; the bounded wait records
// MDL_ERR_MBAR_TIMEOUT in *err and increments *returned (test of the timeout path).
cudaError_t mbar_timeout_selftest(int* err, int* returned, cudaStream_t stream);

}  // namespace mdl
