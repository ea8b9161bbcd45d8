// Single-query attention over a head-interleaved history (MixFormer cross attention).
//
// For sample b and head n: s_l = scale * (q[b,n,:] . h[b,l,n,:]) over the valid events
// l >= kstart[b], p = softmax(s), ctx[b,n,:] = sum_l p_l h[b,l,n,:] -- the reordered
// single-query form of the reference's MixFormerCrossAttention (src/modules/mixformer.py
// :226-784), with q already multiplied by the key weight.
//
// One warp per (b, n), lanes over the head width (element k on lane k % 32, slot k / 32),
// online softmax over the events; the bf16 history is read once, straight from its
// [B, L, N, D] layout (no transposed or fp32 copy). The backward recomputes p from the
// saved log-sum-exp and writes dh for every event (zero on padding) and dq.
#include "sqa.h"

#include <cuda_bf16.h>

namespace mdl {
namespace {

constexpr int kMaxSlots = 4;  // head width up to 128
constexpr int kWarps = 8;
constexpr int kUnroll = 4;    // events per loop iteration

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int S>
__global__ void __launch_bounds__(kWarps * 32) sqa_fwd_kernel(SqaArgs a) {
  const int lane = threadIdx.x & 31;
  const long long item = static_cast<long long>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (item >= static_cast<long long>(a.B) * a.N) return;
  const int b = static_cast<int>(item / a.N), n = static_cast<int>(item % a.N);
  const int D = a.D, L = a.L;
  float q[S], acc[S];
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const int k = lane + 32 * s;
    q[s] = k < D ? a.q[item * D + k] * a.scale : 0.f;
    acc[s] = 0.f;
  }
  int k0 = a.kstart[b];
  k0 = k0 < 0 ? 0 : (k0 > L ? L : k0);
  float m = -INFINITY, l = 0.f;
  const __nv_bfloat16* h = a.hist + (static_cast<long long>(b) * L * a.N + n) * D;
  const long long lstride = static_cast<long long>(a.N) * D;
  // kUnroll events per iteration: their loads and warp reductions are independent, so the
  // dependent load -> reduce -> exp chain of one event overlaps with the next ones
  for (int e0 = k0; e0 < L; e0 += kUnroll) {
    float hv[kUnroll][S];
    float dot[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int e = e0 + u;
      dot[u] = 0.f;
#pragma unroll
      for (int s = 0; s < S; ++s) {
        const int k = lane + 32 * s;
        hv[u][s] = (k < D && e < L) ? __bfloat162float(h[e * lstride + k]) : 0.f;
        dot[u] += q[s] * hv[u][s];
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) dot[u] = warp_sum(dot[u]);
    float mn = m;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      if (e0 + u < L) mn = fmaxf(mn, dot[u]);
    const float corr = expf(m - mn);  // 0 on the first chunk (m = -inf)
    l *= corr;
#pragma unroll
    for (int s = 0; s < S; ++s) acc[s] *= corr;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (e0 + u >= L) break;
      const float p = expf(dot[u] - mn);
      l += p;
#pragma unroll
      for (int s = 0; s < S; ++s) acc[s] += p * hv[u][s];
    }
    m = mn;
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const int k = lane + 32 * s;
    if (k < D) a.ctx[item * D + k] = acc[s] * inv;
  }
  if (lane == 0) a.lse[item] = l > 0.f ? m + logf(l) : -INFINITY;
}

template <int S>
__global__ void __launch_bounds__(kWarps * 32) sqa_bwd_kernel(SqaArgs a) {
  const int lane = threadIdx.x & 31;
  const long long item = static_cast<long long>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (item >= static_cast<long long>(a.B) * a.N) return;
  const int b = static_cast<int>(item / a.N), n = static_cast<int>(item % a.N);
  const int D = a.D, L = a.L;
  float q[S], dc[S], dq[S];
  float dsum = 0.f;
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const int k = lane + 32 * s;
    q[s] = k < D ? a.q[item * D + k] : 0.f;
    dc[s] = k < D ? a.dctx[item * D + k] : 0.f;
    dsum += k < D ? dc[s] * a.ctx[item * D + k] : 0.f;
    dq[s] = 0.f;
  }
  dsum = warp_sum(dsum);
  const float lse = a.lse[item];
  int k0 = a.kstart[b];
  k0 = k0 < 0 ? 0 : (k0 > L ? L : k0);
  const __nv_bfloat16* h = a.hist + (static_cast<long long>(b) * L * a.N + n) * D;
  __nv_bfloat16* dh = a.dhist + (static_cast<long long>(b) * L * a.N + n) * D;
  const long long lstride = static_cast<long long>(a.N) * D;
  const bool any = lse > -INFINITY;
  const int first = any ? k0 : L;
  for (int e = 0; e < first; ++e) {  // padding (or no valid event): zero gradient
#pragma unroll
    for (int s = 0; s < S; ++s) {
      const int k = lane + 32 * s;
      if (k < D) dh[e * lstride + k] = __float2bfloat16_rn(0.f);
    }
  }
  for (int e0 = first; e0 < L; e0 += kUnroll) {
    float hv[kUnroll][S];
    float dot[kUnroll], dp[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int e = e0 + u;
      dot[u] = 0.f;
      dp[u] = 0.f;
#pragma unroll
      for (int s = 0; s < S; ++s) {
        const int k = lane + 32 * s;
        hv[u][s] = (k < D && e < L) ? __bfloat162float(h[e * lstride + k]) : 0.f;
        dot[u] += q[s] * hv[u][s];
        dp[u] += dc[s] * hv[u][s];
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      dot[u] = warp_sum(dot[u]);
      dp[u] = warp_sum(dp[u]);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int e = e0 + u;
      if (e >= L) break;
      const float p = expf(dot[u] * a.scale - lse);
      const float ds = p * (dp[u] - dsum);
#pragma unroll
      for (int s = 0; s < S; ++s) {
        const int k = lane + 32 * s;
        dq[s] += ds * a.scale * hv[u][s];
        if (k < D) dh[e * lstride + k] = __float2bfloat16_rn(p * dc[s] + ds * a.scale * q[s]);
      }
    }
  }
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const int k = lane + 32 * s;
    if (k < D) a.dq[item * D + k] = dq[s];
  }
}

}  // namespace

cudaError_t sqa_fwd(const SqaArgs& a, cudaStream_t stream) {
  if (a.B <= 0 || a.N <= 0) return cudaSuccess;
  if (a.D <= 0 || a.D > 32 * kMaxSlots || a.L < 0) return cudaErrorInvalidValue;
  const long long items = static_cast<long long>(a.B) * a.N;
  const int grid = static_cast<int>((items + kWarps - 1) / kWarps);
  const int slots = (a.D + 31) / 32;
  if (slots == 1) sqa_fwd_kernel<1><<<grid, kWarps * 32, 0, stream>>>(a);
  else if (slots == 2) sqa_fwd_kernel<2><<<grid, kWarps * 32, 0, stream>>>(a);
  else if (slots == 3) sqa_fwd_kernel<3><<<grid, kWarps * 32, 0, stream>>>(a);
  else sqa_fwd_kernel<4><<<grid, kWarps * 32, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t sqa_bwd(const SqaArgs& a, cudaStream_t stream) {
  if (a.B <= 0 || a.N <= 0) return cudaSuccess;
  if (a.D <= 0 || a.D > 32 * kMaxSlots || a.L < 0) return cudaErrorInvalidValue;
  const long long items = static_cast<long long>(a.B) * a.N;
  const int grid = static_cast<int>((items + kWarps - 1) / kWarps);
  const int slots = (a.D + 31) / 32;
  if (slots == 1) sqa_bwd_kernel<1><<<grid, kWarps * 32, 0, stream>>>(a);
  else if (slots == 2) sqa_bwd_kernel<2><<<grid, kWarps * 32, 0, stream>>>(a);
  else if (slots == 3) sqa_bwd_kernel<3><<<grid, kWarps * 32, 0, stream>>>(a);
  else sqa_bwd_kernel<4><<<grid, kWarps * 32, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace mdl
