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

// ------------------------------------------------------------------ shared history
// One warp per sample runs all G queries over the sample's history, so every history row
// is read once for all of them (and dhist is written once, the sum over the queries).
// Lane `lane` holds the column pairs 64 * p + 2 * lane + {0, 1}, p < P (bf16x2 loads).
namespace {

constexpr int kSharedUnroll = 2;

__device__ __forceinline__ void load_pairs(const __nv_bfloat16* row, int D, int lane, int P, bool ok, float* v) {
  for (int p = 0; p < P; ++p) {
    const int k = 64 * p + 2 * lane;
    if (ok && k < D) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(row + k));
      v[2 * p] = f.x;
      v[2 * p + 1] = f.y;
    } else {
      v[2 * p] = 0.f;
      v[2 * p + 1] = 0.f;
    }
  }
}

template <int P, int G>
__global__ void __launch_bounds__(kWarps * 32) sqa_shared_fwd_kernel(SqaSharedArgs a) {
  const int lane = threadIdx.x & 31;
  const long long b = static_cast<long long>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (b >= a.B) return;
  const int D = a.D, L = a.L, NG = a.G;
  float q[G][2 * P], acc[G][2 * P], m[G], l[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const int k = 64 * p + 2 * lane;
      const bool ok = g < NG && k < D;
      const float* src = a.q + (b * NG + g) * D + k;
      q[g][2 * p] = ok ? src[0] * a.scale : 0.f;
      q[g][2 * p + 1] = ok ? src[1] * a.scale : 0.f;
      acc[g][2 * p] = acc[g][2 * p + 1] = 0.f;
    }
  }
  int k0 = a.kstart[b];
  k0 = k0 < 0 ? 0 : (k0 > L ? L : k0);
  const __nv_bfloat16* h = a.hist + b * L * D;
  for (int e0 = k0; e0 < L; e0 += kSharedUnroll) {
    float hv[kSharedUnroll][2 * P];
    float dot[kSharedUnroll][G];
#pragma unroll
    for (int u = 0; u < kSharedUnroll; ++u) load_pairs(h + static_cast<long long>(e0 + u) * D, D, lane, P,
                                                       e0 + u < L, hv[u]);
#pragma unroll
    for (int u = 0; u < kSharedUnroll; ++u)
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 2 * P; ++j) s = fmaf(q[g][j], hv[u][j], s);
        dot[u][g] = warp_sum(s);
      }
#pragma unroll
    for (int u = 0; u < kSharedUnroll; ++u) {
      if (e0 + u >= L) break;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float mn = fmaxf(m[g], dot[u][g]);
        const float corr = expf(m[g] - mn);  // 0 on the first event (m = -inf)
        const float pe = expf(dot[u][g] - mn);
        l[g] = l[g] * corr + pe;
#pragma unroll
        for (int j = 0; j < 2 * P; ++j) acc[g][j] = fmaf(acc[g][j], corr, pe * hv[u][j]);
        m[g] = mn;
      }
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (g >= NG) break;
    const float inv = l[g] > 0.f ? 1.f / l[g] : 0.f;
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const int k = 64 * p + 2 * lane;
      if (k < D)
        *reinterpret_cast<float2*>(a.ctx + (b * NG + g) * D + k) =
            make_float2(acc[g][2 * p] * inv, acc[g][2 * p + 1] * inv);
    }
    if (lane == 0) a.lse[b * NG + g] = l[g] > 0.f ? m[g] + logf(l[g]) : -INFINITY;
  }
}

template <int P, int G>
__global__ void __launch_bounds__(kWarps * 32) sqa_shared_bwd_kernel(SqaSharedArgs a) {
  const int lane = threadIdx.x & 31;
  const long long b = static_cast<long long>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (b >= a.B) return;
  const int D = a.D, L = a.L, NG = a.G;
  const float scale = a.scale;
  float q[G][2 * P], dc[G][2 * P], dq[G][2 * P], lse[G], delta[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    float dd = 0.f;
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const int k = 64 * p + 2 * lane;
      const bool ok = g < NG && k < D;
      const long long o = (b * NG + g) * D + k;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        q[g][2 * p + t] = ok ? a.q[o + t] : 0.f;
        dc[g][2 * p + t] = ok ? a.dctx[o + t] : 0.f;
        dq[g][2 * p + t] = 0.f;
        if (ok) dd = fmaf(dc[g][2 * p + t], a.ctx[o + t], dd);
      }
    }
    delta[g] = warp_sum(dd);
    lse[g] = g < NG ? a.lse[b * NG + g] : -INFINITY;
  }
  int k0 = a.kstart[b];
  k0 = k0 < 0 ? 0 : (k0 > L ? L : k0);
  const __nv_bfloat16* h = a.hist + b * L * D;
  __nv_bfloat16* dh = a.dhist + b * L * D;
  for (int e = 0; e < k0; ++e) {  // padding: zero gradient
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const int k = 64 * p + 2 * lane;
      if (k < D) *reinterpret_cast<__nv_bfloat162*>(dh + static_cast<long long>(e) * D + k) =
                     __floats2bfloat162_rn(0.f, 0.f);
    }
  }
  for (int e0 = k0; e0 < L; e0 += kSharedUnroll) {
    float hv[kSharedUnroll][2 * P];
    float sd[kSharedUnroll][G], pd[kSharedUnroll][G];
#pragma unroll
    for (int u = 0; u < kSharedUnroll; ++u) load_pairs(h + static_cast<long long>(e0 + u) * D, D, lane, P,
                                                       e0 + u < L, hv[u]);
#pragma unroll
    for (int u = 0; u < kSharedUnroll; ++u)
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float s = 0.f, d = 0.f;
#pragma unroll
        for (int j = 0; j < 2 * P; ++j) {
          s = fmaf(q[g][j], hv[u][j], s);
          d = fmaf(dc[g][j], hv[u][j], d);
        }
        sd[u][g] = warp_sum(s);
        pd[u][g] = warp_sum(d);
      }
#pragma unroll
    for (int u = 0; u < kSharedUnroll; ++u) {
      const int e = e0 + u;
      if (e >= L) break;
      float gh[2 * P];
#pragma unroll
      for (int j = 0; j < 2 * P; ++j) gh[j] = 0.f;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pr = lse[g] == -INFINITY ? 0.f : expf(sd[u][g] * scale - lse[g]);
        const float ds = pr * (pd[u][g] - delta[g]);
#pragma unroll
        for (int j = 0; j < 2 * P; ++j) {
          dq[g][j] = fmaf(ds, hv[u][j], dq[g][j]);
          gh[j] = fmaf(pr, dc[g][j], fmaf(scale * ds, q[g][j], gh[j]));
        }
      }
#pragma unroll
      for (int p = 0; p < P; ++p) {
        const int k = 64 * p + 2 * lane;
        if (k < D) *reinterpret_cast<__nv_bfloat162*>(dh + static_cast<long long>(e) * D + k) =
                       __floats2bfloat162_rn(gh[2 * p], gh[2 * p + 1]);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (g >= NG) break;
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const int k = 64 * p + 2 * lane;
      if (k < D)
        *reinterpret_cast<float2*>(a.dq + (b * NG + g) * D + k) =
            make_float2(dq[g][2 * p] * scale, dq[g][2 * p + 1] * scale);
    }
  }
}

int shared_pairs(int D) { return D <= 64 ? 1 : (D <= 128 ? 2 : 4); }
int shared_groups(int G) { return G <= 2 ? 2 : (G <= 4 ? 4 : 8); }

#define MDL_SQA_SHARED_DISPATCH(KERNEL, P, GT, grid, stream, a)       \
  do {                                                                \
    if (P == 1 && GT == 2) KERNEL<1, 2><<<grid, kWarps * 32, 0, stream>>>(a); \
    else if (P == 1 && GT == 4) KERNEL<1, 4><<<grid, kWarps * 32, 0, stream>>>(a); \
    else if (P == 1) KERNEL<1, 8><<<grid, kWarps * 32, 0, stream>>>(a); \
    else if (P == 2 && GT == 2) KERNEL<2, 2><<<grid, kWarps * 32, 0, stream>>>(a); \
    else if (P == 2 && GT == 4) KERNEL<2, 4><<<grid, kWarps * 32, 0, stream>>>(a); \
    else if (P == 2) KERNEL<2, 8><<<grid, kWarps * 32, 0, stream>>>(a); \
    else if (GT == 2) KERNEL<4, 2><<<grid, kWarps * 32, 0, stream>>>(a); \
    else KERNEL<4, 4><<<grid, kWarps * 32, 0, stream>>>(a);           \
  } while (0)

}  // namespace

bool sqa_shared_supported(int G, int D) {
  if (G <= 0 || G > 8 || D <= 0 || D > 256 || (D & 1)) return false;
  return shared_groups(G) * shared_pairs(D) <= 16;
}

cudaError_t sqa_shared_fwd(const SqaSharedArgs& a, cudaStream_t stream) {
  if (a.B <= 0) return cudaSuccess;
  if (!sqa_shared_supported(a.G, a.D) || a.L < 0) return cudaErrorInvalidValue;
  const int grid = (a.B + kWarps - 1) / kWarps;
  const int P = shared_pairs(a.D), GT = shared_groups(a.G);
  MDL_SQA_SHARED_DISPATCH(sqa_shared_fwd_kernel, P, GT, grid, stream, a);
  return cudaGetLastError();
}

cudaError_t sqa_shared_bwd(const SqaSharedArgs& a, cudaStream_t stream) {
  if (a.B <= 0) return cudaSuccess;
  if (!sqa_shared_supported(a.G, a.D) || a.L < 0) return cudaErrorInvalidValue;
  const int grid = (a.B + kWarps - 1) / kWarps;
  const int P = shared_pairs(a.D), GT = shared_groups(a.G);
  MDL_SQA_SHARED_DISPATCH(sqa_shared_bwd_kernel, P, GT, grid, stream, a);
  return cudaGetLastError();
}

}  // namespace mdl
