// Few-query multi-head attention for sm_100a (MDL domain tokens attending to
// feature tokens: tens of queries over tens of keys per sample).
//
// Reference: DomainAwareAttention (src/modules/attention.py:425-512) runs
// scaled_dot_product_attention on [B, H, Nq, hd] x [B, H, Nk, hd]. With Nq, Nk of
// order 10-60 every (sample, head) fits in one CTA's shared memory, so each CTA
// loads its Q/K/V tiles once (16-byte loads, all issued before the first use),
// forms scores, softmax and output in fp32, and the backward recomputes the
// probabilities from the saved log-sum-exp. No score matrix touches HBM; the
// kernels are bound by reading Q/K/V (and dO/O) once and writing O (dQ/dK/dV).
#include "attention.h"
#include "common.cuh"

namespace mdl {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

struct Tile {
  const __nv_bfloat16* src;
  long long ld;
  int rows;
  float* dst;
};

// Copy NT bf16 tiles [rows, hd] (row stride ld) into fp32 shared memory with row
// pitch `pitch`. 16-byte chunks; kUnroll loads in flight per thread.
template <int NT>
__device__ __forceinline__ void load_tiles(const Tile (&t)[NT], int hd, int pitch) {
  const int cpr = hd >> 3;
  int start[NT + 1];
  start[0] = 0;
#pragma unroll
  for (int k = 0; k < NT; ++k) start[k + 1] = start[k] + t[k].rows * cpr;
  const int total = start[NT];
  for (int base = threadIdx.x; base < total; base += kThreads * kUnroll) {
    uint4 v[kUnroll];
    float* dst[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int c = base + u * kThreads;
      dst[u] = nullptr;
      if (c < total) {
        // select the tile with compile-time indices only (keeps everything in registers)
        const __nv_bfloat16* src = t[0].src;
        long long ld = t[0].ld;
        float* d0 = t[0].dst;
        int cc = c;
#pragma unroll
        for (int kk = 1; kk < NT; ++kk) {
          if (c >= start[kk]) {
            src = t[kk].src;
            ld = t[kk].ld;
            d0 = t[kk].dst;
            cc = c - start[kk];
          }
        }
        const int r = cc / cpr, part = cc - r * cpr;
        v[u] = __ldg(reinterpret_cast<const uint4*>(src + r * ld + part * 8));
        dst[u] = d0 + r * pitch + part * 8;
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (dst[u] != nullptr) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[u]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          dst[u][2 * e] = f.x;
          dst[u][2 * e + 1] = f.y;
        }
      }
    }
  }
}

__device__ __forceinline__ float dot_rows(const float* a, const float* b, int hd) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  for (int d = 0; d < hd; d += 4) {
    s0 = fmaf(a[d], b[d], s0);
    s1 = fmaf(a[d + 1], b[d + 1], s1);
    s2 = fmaf(a[d + 2], b[d + 2], s2);
    s3 = fmaf(a[d + 3], b[d + 3], s3);
  }
  return (s0 + s1) + (s2 + s3);
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
  {
    const Tile tiles[3] = {{q, a.ldq, Nq, Qs}, {k, a.ldk, Nk, Ks}, {v, a.ldk, Nk, Vs}};
    load_tiles<3>(tiles, hd, P);
  }
  __syncthreads();
  const int valid = a.key_valid ? min(Nk, a.key_valid[b]) : Nk;
  for (int e = threadIdx.x; e < Nq * Nk; e += blockDim.x) {
    const int i = e / Nk, j = e - i * Nk;
    S[e] = dot_rows(Qs + i * P, Ks + j * P, hd) * a.scale;
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
  const int hd2 = hd >> 1;
  for (int e = threadIdx.x; e < Nq * hd2; e += blockDim.x) {
    const int i = e / hd2, d = 2 * (e - i * hd2);
    float acc0 = 0.f, acc1 = 0.f;
    for (int j = 0; j < valid; ++j) {
      const float p = S[i * Nk + j];
      acc0 = fmaf(p, Vs[j * P + d], acc0);
      acc1 = fmaf(p, Vs[j * P + d + 1], acc1);
    }
    *reinterpret_cast<__nv_bfloat162*>(o + i * a.ldo + d) = __floats2bfloat162_rn(acc0, acc1);
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
  float* Os = dOs + Nq * P;
  float* Pm = Os + Nq * P;    // probabilities [Nq][Nk]
  float* dS = Pm + Nq * Nk;   // [Nq][Nk]
  float* Di = dS + Nq * Nk;   // [Nq]
  const auto* q = reinterpret_cast<const __nv_bfloat16*>(a.q) + b * a.bsq + h * hd;
  const auto* k = reinterpret_cast<const __nv_bfloat16*>(a.k) + b * a.bsk + h * hd;
  const auto* v = reinterpret_cast<const __nv_bfloat16*>(a.v) + b * a.bsk + h * hd;
  const auto* o = reinterpret_cast<const __nv_bfloat16*>(a.o) + b * a.bso + h * hd;
  const auto* dout = reinterpret_cast<const __nv_bfloat16*>(a.dout) + b * a.bso + h * hd;
  {
    const Tile tiles[5] = {{q, a.ldq, Nq, Qs}, {k, a.ldk, Nk, Ks}, {v, a.ldk, Nk, Vs}, {dout, a.ldo, Nq, dOs},
                           {o, a.ldo, Nq, Os}};
    load_tiles<5>(tiles, hd, P);
  }
  const int valid = a.key_valid ? min(Nk, a.key_valid[b]) : Nk;
  const float* lse = a.lse + (static_cast<long long>(b) * a.H + h) * Nq;
  __syncthreads();
  // D_i = rowsum(dO * O): one warp per row
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = warp; i < Nq; i += kThreads / 32) {
    float s = 0.f;
    for (int d = lane; d < hd; d += 32) s = fmaf(dOs[i * P + d], Os[i * P + d], s);
    s = warp_sum(s);
    if (lane == 0) Di[i] = s;
  }
  for (int e = threadIdx.x; e < Nq * Nk; e += blockDim.x) {
    const int i = e / Nk, j = e - i * Nk;
    Pm[e] = j < valid ? expf(dot_rows(Qs + i * P, Ks + j * P, hd) * a.scale - lse[i]) : 0.f;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < Nq * Nk; e += blockDim.x) {
    const int i = e / Nk, j = e - i * Nk;
    dS[e] = Pm[e] * (dot_rows(dOs + i * P, Vs + j * P, hd) - Di[i]);
  }
  __syncthreads();
  auto* dq = reinterpret_cast<__nv_bfloat16*>(a.dq) + b * a.bsq + h * hd;
  auto* dk = reinterpret_cast<__nv_bfloat16*>(a.dk) + b * a.bsk + h * hd;
  auto* dv = reinterpret_cast<__nv_bfloat16*>(a.dv) + b * a.bsk + h * hd;
  const int hd2 = hd >> 1;
  for (int e = threadIdx.x; e < Nq * hd2; e += blockDim.x) {
    const int i = e / hd2, d = 2 * (e - i * hd2);
    float s0 = 0.f, s1 = 0.f;
    for (int j = 0; j < Nk; ++j) {
      const float w = dS[i * Nk + j];
      s0 = fmaf(w, Ks[j * P + d], s0);
      s1 = fmaf(w, Ks[j * P + d + 1], s1);
    }
    *reinterpret_cast<__nv_bfloat162*>(dq + i * a.ldq + d) = __floats2bfloat162_rn(s0 * a.scale, s1 * a.scale);
  }
  for (int e = threadIdx.x; e < Nk * hd2; e += blockDim.x) {
    const int j = e / hd2, d = 2 * (e - j * hd2);
    float k0 = 0.f, k1 = 0.f, v0 = 0.f, v1 = 0.f;
    for (int i = 0; i < Nq; ++i) {
      const float ds = dS[i * Nk + j], p = Pm[i * Nk + j];
      k0 = fmaf(ds, Qs[i * P + d], k0);
      k1 = fmaf(ds, Qs[i * P + d + 1], k1);
      v0 = fmaf(p, dOs[i * P + d], v0);
      v1 = fmaf(p, dOs[i * P + d + 1], v1);
    }
    *reinterpret_cast<__nv_bfloat162*>(dk + j * a.ldk + d) = __floats2bfloat162_rn(k0 * a.scale, k1 * a.scale);
    *reinterpret_cast<__nv_bfloat162*>(dv + j * a.ldk + d) = __floats2bfloat162_rn(v0, v1);
  }
}

size_t fwd_smem(const SmallAttnArgs& a) {
  return sizeof(float) * (static_cast<size_t>(a.Nq + 2 * a.Nk) * (a.hd + 1) + static_cast<size_t>(a.Nq) * a.Nk);
}
size_t bwd_smem(const SmallAttnArgs& a) {
  return sizeof(float) * (static_cast<size_t>(3 * a.Nq + 2 * a.Nk) * (a.hd + 1) + 2 * static_cast<size_t>(a.Nq) * a.Nk +
                          a.Nq);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

bool valid_args(const SmallAttnArgs& a, bool bwd) {
  if (a.Nq <= 0 || a.Nk <= 0 || a.Nq > 64 || a.Nk > 64 || a.hd <= 0 || a.hd > 128 || (a.hd % 8)) return false;
  if ((a.ldq % 8) || (a.ldk % 8) || (a.ldo % 8) || (a.bsq % 8) || (a.bsk % 8) || (a.bso % 8)) return false;
  if (!aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v) || !aligned16(a.o)) return false;
  if (bwd && (!aligned16(a.dout) || !aligned16(a.dq) || !aligned16(a.dk) || !aligned16(a.dv) || a.lse == nullptr))
    return false;
  return true;
}

}  // namespace

cudaError_t small_attention_fwd(const SmallAttnArgs& a, cudaStream_t stream) {
  if (a.B == 0) return cudaSuccess;
  if (!valid_args(a, false)) return cudaErrorInvalidValue;
  const size_t smem = fwd_smem(a);
  cudaFuncSetAttribute(small_attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  small_attn_fwd_kernel<<<a.B * a.H, kThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t small_attention_bwd(const SmallAttnArgs& a, cudaStream_t stream) {
  if (a.B == 0) return cudaSuccess;
  if (!valid_args(a, true)) return cudaErrorInvalidValue;
  const size_t smem = bwd_smem(a);
  cudaFuncSetAttribute(small_attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  small_attn_bwd_kernel<<<a.B * a.H, kThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace mdl
