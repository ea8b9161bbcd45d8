// Few-query multi-head attention for sm_100a (MDL domain tokens attending to
// feature tokens: tens of queries over tens of keys per sample).
//
// Reference: DomainAwareAttention (src/modules/attention.py:425-512) runs
// scaled_dot_product_attention on [B, H, Nq, hd] x [B, H, Nk, hd]. With Nq, Nk of
// order 10-60 every (sample, head) fits in one CTA's shared memory, so each CTA
// loads its Q/K/V tiles once, forms scores, softmax and output in fp32, and the
// backward recomputes the probabilities from the saved log-sum-exp. No score
// matrix touches HBM.
#include "attention.h"
#include "common.cuh"

namespace mdl {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ void load_rows(float* dst, const __nv_bfloat16* src, int rows, int hd, long long ld,
                                          int pitch) {
  for (int e = threadIdx.x; e < rows * hd; e += blockDim.x) {
    const int r = e / hd, c = e - r * hd;
    dst[r * pitch + c] = __bfloat162float(src[r * ld + c]);
  }
}

__global__ void __launch_bounds__(kThreads) small_attn_fwd_kernel(const SmallAttnArgs a) {
  extern __shared__ float sm[];
  const int b = blockIdx.x / a.H, h = blockIdx.x - (blockIdx.x / a.H) * a.H;
  const int hd = a.hd, P = hd + 1, Nq = a.Nq, Nk = a.Nk;
  float* Qs = sm;
  float* Ks = Qs + Nq * P;
  float* Vs = Ks + Nk * P;
  float* S = Vs + Nk * P;  // [Nq][Nk]
  const auto* q = reinterpret_cast<const __nv_bfloat16*>(a.q) + b * a.bsq + h * hd;
  const auto* k = reinterpret_cast<const __nv_bfloat16*>(a.k) + b * a.bsk + h * hd;
  const auto* v = reinterpret_cast<const __nv_bfloat16*>(a.v) + b * a.bsk + h * hd;
  load_rows(Qs, q, Nq, hd, a.ldq, P);
  load_rows(Ks, k, Nk, hd, a.ldk, P);
  load_rows(Vs, v, Nk, hd, a.ldk, P);
  __syncthreads();
  const int valid = a.key_valid ? min(Nk, a.key_valid[b]) : Nk;
  for (int e = threadIdx.x; e < Nq * Nk; e += blockDim.x) {
    const int i = e / Nk, j = e - i * Nk;
    float s = 0.f;
    for (int d = 0; d < hd; ++d) s += Qs[i * P + d] * Ks[j * P + d];
    S[e] = s * a.scale;
  }
  __syncthreads();
  // row softmax: one warp per row
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = warp; i < Nq; i += kThreads / 32) {
    float m = -INFINITY;
    for (int j = lane; j < valid; j += 32) m = fmaxf(m, S[i * Nk + j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.f;
    for (int j = lane; j < Nk; j += 32) {
      const float p = j < valid ? expf(S[i * Nk + j] - m) : 0.f;
      S[i * Nk + j] = p;
      sum += p;
    }
    sum = warp_sum(sum);
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
    for (int j = lane; j < Nk; j += 32) S[i * Nk + j] *= inv;
    if (lane == 0 && a.lse) a.lse[(static_cast<long long>(b) * a.H + h) * Nq + i] = sum > 0.f ? m + logf(sum) : 0.f;
  }
  __syncthreads();
  auto* o = reinterpret_cast<__nv_bfloat16*>(a.o) + b * a.bso + h * hd;
  for (int e = threadIdx.x; e < Nq * hd; e += blockDim.x) {
    const int i = e / hd, d = e - i * hd;
    float acc = 0.f;
    for (int j = 0; j < valid; ++j) acc += S[i * Nk + j] * Vs[j * P + d];
    o[i * a.ldo + d] = __float2bfloat16_rn(acc);
  }
}

__global__ void __launch_bounds__(kThreads) small_attn_bwd_kernel(const SmallAttnArgs a) {
  extern __shared__ float sm[];
  const int b = blockIdx.x / a.H, h = blockIdx.x - (blockIdx.x / a.H) * a.H;
  const int hd = a.hd, P = hd + 1, Nq = a.Nq, Nk = a.Nk;
  float* Qs = sm;
  float* Ks = Qs + Nq * P;
  float* Vs = Ks + Nk * P;
  float* dOs = Vs + Nk * P;
  float* Pm = dOs + Nq * P;   // probabilities [Nq][Nk]
  float* dS = Pm + Nq * Nk;   // [Nq][Nk]
  float* Di = dS + Nq * Nk;   // [Nq]
  const auto* q = reinterpret_cast<const __nv_bfloat16*>(a.q) + b * a.bsq + h * hd;
  const auto* k = reinterpret_cast<const __nv_bfloat16*>(a.k) + b * a.bsk + h * hd;
  const auto* v = reinterpret_cast<const __nv_bfloat16*>(a.v) + b * a.bsk + h * hd;
  const auto* o = reinterpret_cast<const __nv_bfloat16*>(a.o) + b * a.bso + h * hd;
  const auto* dout = reinterpret_cast<const __nv_bfloat16*>(a.dout) + b * a.bso + h * hd;
  load_rows(Qs, q, Nq, hd, a.ldq, P);
  load_rows(Ks, k, Nk, hd, a.ldk, P);
  load_rows(Vs, v, Nk, hd, a.ldk, P);
  load_rows(dOs, dout, Nq, hd, a.ldo, P);
  const int valid = a.key_valid ? min(Nk, a.key_valid[b]) : Nk;
  __syncthreads();
  // D_i = rowsum(dO * O)
  for (int i = threadIdx.x; i < Nq; i += blockDim.x) {
    float s = 0.f;
    for (int d = 0; d < hd; ++d) s += dOs[i * P + d] * __bfloat162float(o[i * a.ldo + d]);
    Di[i] = s;
  }
  const float* lse = a.lse + (static_cast<long long>(b) * a.H + h) * Nq;
  for (int e = threadIdx.x; e < Nq * Nk; e += blockDim.x) {
    const int i = e / Nk, j = e - i * Nk;
    float p = 0.f;
    if (j < valid) {
      float s = 0.f;
      for (int d = 0; d < hd; ++d) s += Qs[i * P + d] * Ks[j * P + d];
      p = expf(s * a.scale - lse[i]);
    }
    Pm[e] = p;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < Nq * Nk; e += blockDim.x) {
    const int i = e / Nk, j = e - i * Nk;
    float dp = 0.f;
    for (int d = 0; d < hd; ++d) dp += dOs[i * P + d] * Vs[j * P + d];
    dS[e] = Pm[e] * (dp - Di[i]);
  }
  __syncthreads();
  auto* dq = reinterpret_cast<__nv_bfloat16*>(a.dq) + b * a.bsq + h * hd;
  auto* dk = reinterpret_cast<__nv_bfloat16*>(a.dk) + b * a.bsk + h * hd;
  auto* dv = reinterpret_cast<__nv_bfloat16*>(a.dv) + b * a.bsk + h * hd;
  for (int e = threadIdx.x; e < Nq * hd; e += blockDim.x) {
    const int i = e / hd, d = e - i * hd;
    float s = 0.f;
    for (int j = 0; j < Nk; ++j) s += dS[i * Nk + j] * Ks[j * P + d];
    dq[i * a.ldq + d] = __float2bfloat16_rn(s * a.scale);
  }
  for (int e = threadIdx.x; e < Nk * hd; e += blockDim.x) {
    const int j = e / hd, d = e - j * hd;
    float sk = 0.f, sv = 0.f;
    for (int i = 0; i < Nq; ++i) {
      sk += dS[i * Nk + j] * Qs[i * P + d];
      sv += Pm[i * Nk + j] * dOs[i * P + d];
    }
    dk[j * a.ldk + d] = __float2bfloat16_rn(sk * a.scale);
    dv[j * a.ldk + d] = __float2bfloat16_rn(sv);
  }
}

size_t fwd_smem(const SmallAttnArgs& a) {
  return sizeof(float) * (static_cast<size_t>(a.Nq + 2 * a.Nk) * (a.hd + 1) + static_cast<size_t>(a.Nq) * a.Nk);
}
size_t bwd_smem(const SmallAttnArgs& a) {
  return sizeof(float) * (static_cast<size_t>(2 * a.Nq + 2 * a.Nk) * (a.hd + 1) + 2 * static_cast<size_t>(a.Nq) * a.Nk +
                          a.Nq);
}

}  // namespace

cudaError_t small_attention_fwd(const SmallAttnArgs& a, cudaStream_t stream) {
  if (a.B == 0) return cudaSuccess;
  if (a.Nq <= 0 || a.Nk <= 0 || a.Nq > 64 || a.Nk > 64 || a.hd <= 0 || a.hd > 128) return cudaErrorInvalidValue;
  const size_t smem = fwd_smem(a);
  cudaFuncSetAttribute(small_attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  small_attn_fwd_kernel<<<a.B * a.H, kThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t small_attention_bwd(const SmallAttnArgs& a, cudaStream_t stream) {
  if (a.B == 0) return cudaSuccess;
  if (a.Nq <= 0 || a.Nk <= 0 || a.Nq > 64 || a.Nk > 64 || a.hd <= 0 || a.hd > 128) return cudaErrorInvalidValue;
  const size_t smem = bwd_smem(a);
  cudaFuncSetAttribute(small_attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  small_attn_bwd_kernel<<<a.B * a.H, kThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace mdl
