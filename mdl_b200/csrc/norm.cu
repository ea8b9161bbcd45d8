// Fused normalisation kernels for sm_100a.
//
// RankMixer blocks compute LN(mix(x) + x) and LN(ffn + mixed)
// (reference src/model.py:6663-6665, token mixing src/modules/attention.py:354-363
// as permute(0,2,1,3).contiguous()). Here the token-mixing permutation is an
// index remap inside the LayerNorm kernel: no permuted copy is materialised.
// The backward recomputes the normalised row from the inputs and the saved
// (mean, rstd), so only those two floats per row are kept from the forward.
// gamma/beta and the per-token bias gradient of the producing layer are
// accumulated per CTA in registers and folded by a second small kernel.
#include <atomic>
#include "common.cuh"
#include "norm.h"

namespace mdl {
namespace {

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* v) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

// 8 consecutive fp32 values (32-byte aligned), or `fill` when p is null.
__device__ __forceinline__ void load_f8(const float* p, int c, float* v, float fill) {
  if (p == nullptr) {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = fill;
    return;
  }
  const float4 x = __ldg(reinterpret_cast<const float4*>(p + c));
  const float4 y = __ldg(reinterpret_cast<const float4*>(p + c + 4));
  v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
  v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
}

// Pre-norm value of row (b, i): mix(a)+a or a+b, 8 elements at column c.
template <bool MIX>
__device__ __forceinline__ void load_v(const __nv_bfloat16* a, const __nv_bfloat16* bsrc, long long b, int i,
                                       int T, int D, int c, float* v) {
  const long long row = (b * T + i) * static_cast<long long>(D);
  load8(a + row + c, v);
  float u[8];
  if (MIX) {
    const int dh = D / T;
    const int j = c / dh;
    const int w = c - j * dh;
    load8(a + (b * T + j) * static_cast<long long>(D) + i * dh + w, u);
  } else if (bsrc != nullptr) {
    load8(bsrc + row + c, u);
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) u[k] = 0.f;
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] += u[k];
}

template <int NCH, bool MIX>
__global__ void __launch_bounds__(256) ln_fwd_kernel(const LNFwdArgs p) {
  const long long r = (static_cast<long long>(blockIdx.x) * 256 + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= static_cast<long long>(p.B) * p.T) return;
  const long long b = r / p.T;
  const int i = static_cast<int>(r - b * p.T);
  const auto* a = reinterpret_cast<const __nv_bfloat16*>(p.a);
  const auto* bb = reinterpret_cast<const __nv_bfloat16*>(p.b);
  float v[NCH][8];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int c = (lane + 32 * k) * 8;
    if (c < p.D) {
      load_v<MIX>(a, bb, b, i, p.T, p.D, c, v[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) s += v[k][e];
    }
  }
  const float mean = warp_sum(s) / p.D;
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int c = (lane + 32 * k) * 8;
    if (c < p.D) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[k][e] - mean;
        q += d * d;
      }
    }
  }
  const float rstd = rsqrtf(warp_sum(q) / p.D + p.eps);
  auto* out = reinterpret_cast<__nv_bfloat16*>(p.out) + r * p.D;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int c = (lane + 32 * k) * 8;
    if (c < p.D) {
      float o[8], g[8], bt[8];
      load_f8(p.gamma, c, g, 1.f);
      load_f8(p.beta, c, bt, 0.f);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = (v[k][e] - mean) * rstd * g[e] + bt[e];
      store8(out + c, o);
    }
  }
  if (lane == 0) {
    if (p.mean) p.mean[r] = mean;
    if (p.rstd) p.rstd[r] = rstd;
  }
}

// CTAs of 8 warps. Non-mix: warps walk rows in a grid-stride loop. Mix: a CTA
// walks whole samples (all T rows of sample b are needed to undo the token
// permutation); the dv rows of the current sample are staged in shared memory.
// gamma/beta gradients are accumulated per warp in shared memory (each lane owns
// its columns of its warp's row, so no atomics) and written as one partial row per
// CTA. Keeping them out of registers lets two CTAs share an SM.
template <int NCH, bool MIX>
__global__ void __launch_bounds__(256, NCH <= 4 ? 2 : 1) ln_bwd_kernel(const LNBwdArgs p) {
  // MIX: [T][D] staging of the current sample's dv rows; then [8 warps][2][D] partial sums
  extern __shared__ float sm[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int T = p.T, D = p.D;
  const auto* a = reinterpret_cast<const __nv_bfloat16*>(p.a);
  const auto* bb = reinterpret_cast<const __nv_bfloat16*>(p.b);
  const auto* dy = reinterpret_cast<const __nv_bfloat16*>(p.dy);
  const auto* dyb = reinterpret_cast<const __nv_bfloat16*>(p.dy_bcast);
  auto* dx = reinterpret_cast<__nv_bfloat16*>(p.dx);
  auto* dx2 = reinterpret_cast<__nv_bfloat16*>(p.dx2);
  const auto* res = reinterpret_cast<const __nv_bfloat16*>(p.res);
  float* acc = sm + (MIX ? T * D : 0);
  float* my_dg = acc + warp * 2 * D;  // this warp's dgamma partials, then its dbeta partials
  float* my_db = my_dg + D;
  for (int c = lane * 4; c < 2 * D; c += 128) *reinterpret_cast<float4*>(my_dg + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  __syncwarp();

  // dv of row (b, i); returns via `dv` (registers); accumulates dg/db
  auto row_dv = [&](long long b, int i, float (*dv)[8]) {
    const long long r = b * T + i;
    const float mean = p.mean[r];
    const float rstd = p.rstd[r];
    float xh[NCH][8], gy[NCH][8], g[NCH][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int c = (lane + 32 * k) * 8;
      if (c < D) {
        load_v<MIX>(a, bb, b, i, T, D, c, xh[k]);
        if (dy != nullptr) {
          load8(dy + r * D + c, g[k]);
        } else {
          load8(dyb + b * D + c, g[k]);
#pragma unroll
          for (int e = 0; e < 8; ++e) g[k][e] *= p.bcast_scale;
        }
        float gm[8];
        load_f8(p.gamma, c, gm, 1.f);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          xh[k][e] = (xh[k][e] - mean) * rstd;
          gy[k][e] = g[k][e] * gm[e];
          s1 += gy[k][e];
          s2 += gy[k][e] * xh[k][e];
        }
      }
    }
    s1 = warp_sum(s1) / D;
    s2 = warp_sum(s2) / D;
#pragma unroll
    for (int k = 0; k < NCH; ++k) {
      const int c = (lane + 32 * k) * 8;
      if (c < D) {
        float4* pg = reinterpret_cast<float4*>(my_dg + c);
        float4* pb = reinterpret_cast<float4*>(my_db + c);
        float4 g0 = pg[0], g1 = pg[1], b0 = pb[0], b1 = pb[1];
        g0.x += g[k][0] * xh[k][0]; g0.y += g[k][1] * xh[k][1]; g0.z += g[k][2] * xh[k][2]; g0.w += g[k][3] * xh[k][3];
        g1.x += g[k][4] * xh[k][4]; g1.y += g[k][5] * xh[k][5]; g1.z += g[k][6] * xh[k][6]; g1.w += g[k][7] * xh[k][7];
        b0.x += g[k][0]; b0.y += g[k][1]; b0.z += g[k][2]; b0.w += g[k][3];
        b1.x += g[k][4]; b1.y += g[k][5]; b1.z += g[k][6]; b1.w += g[k][7];
        pg[0] = g0; pg[1] = g1; pb[0] = b0; pb[1] = b1;
#pragma unroll
        for (int e = 0; e < 8; ++e) dv[k][e] = rstd * (gy[k][e] - s1 - xh[k][e] * s2);
      }
    }
  };

  if (MIX) {
    const int dh = D / T;
    for (long long b = blockIdx.x; b < p.B; b += gridDim.x) {
      for (int i = warp; i < T; i += 8) {
        float dv[NCH][8];
        row_dv(b, i, dv);
#pragma unroll
        for (int k = 0; k < NCH; ++k) {
          const int c = (lane + 32 * k) * 8;
          if (c < D) {
            float4* d = reinterpret_cast<float4*>(sm + i * D + c);
            d[0] = make_float4(dv[k][0], dv[k][1], dv[k][2], dv[k][3]);
            d[1] = make_float4(dv[k][4], dv[k][5], dv[k][6], dv[k][7]);
          }
        }
      }
      __syncthreads();
      for (int i = warp; i < T; i += 8) {
        const long long r = b * T + i;
#pragma unroll
        for (int k = 0; k < NCH; ++k) {
          const int c = (lane + 32 * k) * 8;
          if (c < D) {
            const int j = c / dh;
            const int w = c - j * dh;
            const float4* d0 = reinterpret_cast<const float4*>(sm + i * D + c);
            const float4* d1 = reinterpret_cast<const float4*>(sm + j * D + i * dh + w);
            const float4 x0 = d0[0], x1 = d0[1], y0 = d1[0], y1 = d1[1];
            const float o[8] = {x0.x + y0.x, x0.y + y0.y, x0.z + y0.z, x0.w + y0.w,
                                x1.x + y1.x, x1.y + y1.y, x1.z + y1.z, x1.w + y1.w};
            if (dx2 != nullptr) store8(dx2 + r * D + c, o);
            if (res != nullptr) {
              float rv[8], o2[8];
              load8(res + r * D + c, rv);
#pragma unroll
              for (int e = 0; e < 8; ++e) o2[e] = o[e] + rv[e];
              store8(dx + r * D + c, o2);
            } else {
              store8(dx + r * D + c, o);
            }
          }
        }
      }
      __syncthreads();
    }
  } else {
    const long long rows = static_cast<long long>(p.B) * T;
    for (long long r = static_cast<long long>(blockIdx.x) * 8 + warp; r < rows; r += static_cast<long long>(gridDim.x) * 8) {
      const long long b = r / T;
      const int i = static_cast<int>(r - b * T);
      float dv[NCH][8];
      row_dv(b, i, dv);
#pragma unroll
      for (int k = 0; k < NCH; ++k) {
        const int c = (lane + 32 * k) * 8;
        if (c < D) {
          if (dx2 != nullptr) store8(dx2 + r * D + c, dv[k]);
          if (res != nullptr) {
            float rv[8];
            load8(res + r * D + c, rv);
#pragma unroll
            for (int e = 0; e < 8; ++e) dv[k][e] += rv[e];
          }
          store8(dx + r * D + c, dv[k]);
        }
      }
    }
  }
  // ---- fold the 8 warps' gamma/beta partials into this CTA's row of `partials`
  float* prow = p.partials + static_cast<long long>(blockIdx.x) * 2 * D;
  __syncthreads();
  for (int c = threadIdx.x; c < 2 * D; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += acc[w * 2 * D + c];
    prow[c] = t;
  }
}

// Column sums of `partials` [grid, 2D] into dgamma (first D) / dbeta (last D).
// Block = 32 columns x 8 warps; warp w sums rows w, w+8, ... (coalesced 128-byte
// rows), then the 8 warp sums are added in a fixed order (deterministic).
__global__ void __launch_bounds__(256) ln_partials_reduce_kernel(const float* partials, int grid, int D,
                                                                 float* dgamma, float* dbeta) {
  __shared__ float red[8][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (col < 2 * D) {
    int g = warp;
    for (; g + 24 < grid; g += 32) {
      const float a0 = partials[static_cast<long long>(g) * 2 * D + col];
      const float a1 = partials[static_cast<long long>(g + 8) * 2 * D + col];
      const float a2 = partials[static_cast<long long>(g + 16) * 2 * D + col];
      const float a3 = partials[static_cast<long long>(g + 24) * 2 * D + col];
      s += (a0 + a1) + (a2 + a3);
    }
    for (; g < grid; g += 8) s += partials[static_cast<long long>(g) * 2 * D + col];
  }
  red[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && col < 2 * D) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w][lane];
    if (col < D) {
      if (dgamma) dgamma[col] += t;
    } else if (dbeta) {
      dbeta[col - D] += t;
    }
  }
}

// ------------------------------------------------------------------ RMSNorm
template <int NCH>
__global__ void __launch_bounds__(256) rms_fwd_kernel(const RMSArgs p) {
  const long long r = (static_cast<long long>(blockIdx.x) * 256 + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= p.rows) return;
  const auto* x = reinterpret_cast<const __nv_bfloat16*>(p.x) + r * p.D;
  float v[NCH][8];
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int c = (lane + 32 * k) * 8;
    if (c < p.D) {
      load8(x + c, v[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) q += v[k][e] * v[k][e];
    }
  }
  const float rstd = rsqrtf(warp_sum(q) / p.D + p.eps);
  auto* out = reinterpret_cast<__nv_bfloat16*>(p.out) + r * p.D;
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int c = (lane + 32 * k) * 8;
    if (c < p.D) {
      float o[8], w[8];
      load_f8(p.weight, c, w, 1.f);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[k][e] * rstd * w[e];
      store8(out + c, o);
    }
  }
  if (lane == 0 && p.rstd) p.rstd[r] = rstd;
}

// Row of the residual gradient added to dx row r (nullptr: none).
__device__ __forceinline__ const __nv_bfloat16* rms_res_row(const RMSArgs& p, long long r) {
  if (p.dres == nullptr) return nullptr;
  long long rr = r;
  if (p.res_period > 0) {
    const long long smp = r / p.res_period;
    const int e = static_cast<int>(r - smp * p.res_period) - (p.res_period - p.res_tail);
    if (e < 0) return nullptr;
    rr = smp * p.res_tail + e;
  }
  return reinterpret_cast<const __nv_bfloat16*>(p.dres) + rr * p.D;
}

// One warp per row, two independent rows in flight per warp; the weight
// gradient is reduced over the block's warps in shared memory before one
// atomic add per column and block.
template <int NCH>
__global__ void __launch_bounds__(256) rms_bwd_kernel(const RMSArgs p) {
  constexpr int R = NCH <= 2 ? 2 : 1;  // rows in flight per warp (registers allow two for D <= 512)
  __shared__ float sdw[8][256];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const long long warps = static_cast<long long>(gridDim.x) * 8;
  constexpr bool kKeepW = NCH <= 2;  // weights stay in registers for small D, reloaded otherwise
  float wreg[kKeepW ? NCH : 1][8];
  float dw[NCH][8];
#pragma unroll
  for (int k = 0; k < NCH; ++k) {
    const int c = (lane + 32 * k) * 8;
    if (kKeepW && c < p.D) load_f8(p.weight, c, wreg[kKeepW ? k : 0], 1.f);
#pragma unroll
    for (int e = 0; e < 8; ++e) dw[k][e] = 0.f;
  }
  auto weights = [&](int k, int c, float* w) {
    if constexpr (kKeepW) {
#pragma unroll
      for (int e = 0; e < 8; ++e) w[e] = wreg[kKeepW ? k : 0][e];
    } else {
      load_f8(p.weight, c, w, 1.f);
    }
  };
  for (long long r0 = (static_cast<long long>(blockIdx.x) * 256 + threadIdx.x) >> 5; r0 < p.rows; r0 += R * warps) {
    long long rr[R];
#pragma unroll
    for (int u = 0; u < R; ++u) rr[u] = r0 + u * warps;
    float xv[R][NCH][8], gv[R][NCH][8], res[R][NCH][8];
    float s[R], rstd[R];
    bool has_res[R];
#pragma unroll
    for (int u = 0; u < R; ++u) {
      s[u] = 0.f;
      rstd[u] = 0.f;
      has_res[u] = false;
    }
#pragma unroll
    for (int u = 0; u < R; ++u) {
      if (rr[u] >= p.rows) continue;
      const auto* x = reinterpret_cast<const __nv_bfloat16*>(p.x) + rr[u] * p.D;
      const auto* dy = reinterpret_cast<const __nv_bfloat16*>(p.dy) + rr[u] * p.D;
      const __nv_bfloat16* rs = rms_res_row(p, rr[u]);
      has_res[u] = rs != nullptr;
      rstd[u] = p.rstd[rr[u]];
#pragma unroll
      for (int k = 0; k < NCH; ++k) {
        const int c = (lane + 32 * k) * 8;
        if (c < p.D) {
          load8(x + c, xv[u][k]);
          load8(dy + c, gv[u][k]);
          if (rs != nullptr) load8(rs + c, res[u][k]);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < R; ++u) {
      if (rr[u] >= p.rows) continue;
#pragma unroll
      for (int k = 0; k < NCH; ++k) {
        const int c = (lane + 32 * k) * 8;
        if (c < p.D) {
          float w[8];
          weights(k, c, w);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            s[u] += gv[u][k][e] * w[e] * xv[u][k][e];
            dw[k][e] += gv[u][k][e] * xv[u][k][e] * rstd[u];
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < R; ++u) s[u] += __shfl_xor_sync(0xffffffffu, s[u], o);
#pragma unroll
    for (int u = 0; u < R; ++u) {
      if (rr[u] >= p.rows) continue;
      const float su = s[u] / p.D;
      auto* dx = reinterpret_cast<__nv_bfloat16*>(p.dx) + rr[u] * p.D;
#pragma unroll
      for (int k = 0; k < NCH; ++k) {
        const int c = (lane + 32 * k) * 8;
        if (c < p.D) {
          float o[8], w[8];
          weights(k, c, w);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            o[e] = rstd[u] * (gv[u][k][e] * w[e] - xv[u][k][e] * rstd[u] * rstd[u] * su);
            if (has_res[u]) o[e] += res[u][k][e];
          }
          store8(dx + c, o);
        }
      }
    }
  }
  if (p.dweight) {
#pragma unroll
    for (int k = 0; k < NCH; ++k) {  // 256 columns at a time
#pragma unroll
      for (int e = 0; e < 8; ++e) sdw[wib][lane * 8 + e] = dw[k][e];
      __syncthreads();
      const int c = k * 256 + threadIdx.x;
      if (c < p.D) {
        float t = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) t += sdw[q][threadIdx.x];
        atomicAdd(p.dweight + c, t);
      }
      __syncthreads();
    }
  }
}

// SM count of the current device, cached per device (atomics: callers may run on
// any host thread, with any device current).
constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  int n = g_sm_count[dev].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
    g_sm_count[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}


}  // namespace

#define MDL_NCH_DISPATCH(D, MACRO) \
  if ((D) <= 256) { MACRO(1) } else if ((D) <= 512) { MACRO(2) } else if ((D) <= 768) { MACRO(3) } \
  else if ((D) <= 1024) { MACRO(4) } else if ((D) <= 2048) { MACRO(8) } else { return cudaErrorInvalidValue; }

cudaError_t layernorm_fwd(const LNFwdArgs& a, cudaStream_t stream) {
  if (a.D % 8 || a.T <= 0) return cudaErrorInvalidValue;
  if (a.mix && ((a.D % a.T) || ((a.D / a.T) % 8))) return cudaErrorInvalidValue;
  const long long rows = static_cast<long long>(a.B) * a.T;
  if (rows == 0) return cudaSuccess;
  const int grid = static_cast<int>((rows + 7) / 8);
#define LNF(N)                                                                   \
  if (a.mix) ln_fwd_kernel<N, true><<<grid, 256, 0, stream>>>(a);               \
  else ln_fwd_kernel<N, false><<<grid, 256, 0, stream>>>(a);
  MDL_NCH_DISPATCH(a.D, LNF)
#undef LNF
  return cudaGetLastError();
}

int layernorm_bwd_grid(int B) {
  const int cap = sm_count() * 4;  // 4 resident CTAs per SM (48 KB of staging each at D=768, T=16)
  return B < cap ? (B > 0 ? B : 1) : cap;
}

size_t layernorm_bwd_smem(int T, int D, int mix) {
  return static_cast<size_t>((mix ? T : 0) + 16) * D * sizeof(float);  // [T][D] staging + [8][2][D] partials
}

cudaError_t layernorm_bwd(const LNBwdArgs& a, cudaStream_t stream) {
  if (a.D % 8 || a.T <= 0) return cudaErrorInvalidValue;
  if (a.mix && ((a.D % a.T) || ((a.D / a.T) % 8))) return cudaErrorInvalidValue;
  if (a.B == 0) return cudaSuccess;
  const int grid = a.grid > 0 ? a.grid : layernorm_bwd_grid(a.B);
  const size_t smem = layernorm_bwd_smem(a.T, a.D, a.mix);
#define LNB(N)                                                                                         \
  {                                                                                                    \
    auto k = a.mix ? ln_bwd_kernel<N, true> : ln_bwd_kernel<N, false>;                                 \
    cudaError_t ea = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)); \
    if (ea != cudaSuccess) return ea;                                                                  \
    k<<<grid, 256, smem, stream>>>(a);                                                                 \
  }
  MDL_NCH_DISPATCH(a.D, LNB)
#undef LNB
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  ln_partials_reduce_kernel<<<(2 * a.D + 31) / 32, 256, 0, stream>>>(a.partials, grid, a.D, a.dgamma, a.dbeta);
  return cudaGetLastError();
}

cudaError_t rmsnorm_fwd(const RMSArgs& a, cudaStream_t stream) {
  if (a.D % 8) return cudaErrorInvalidValue;
  if (a.rows == 0) return cudaSuccess;
  const int grid = static_cast<int>((a.rows + 7) / 8);
#define RMF(N) rms_fwd_kernel<N><<<grid, 256, 0, stream>>>(a);
  MDL_NCH_DISPATCH(a.D, RMF)
#undef RMF
  return cudaGetLastError();
}

cudaError_t rmsnorm_bwd(const RMSArgs& a, cudaStream_t stream) {
  if (a.D % 8) return cudaErrorInvalidValue;
  if (a.rows == 0) return cudaSuccess;
  long long want = (a.rows + 15) / 16;  // two rows per warp per step
  const int grid = static_cast<int>(want < sm_count() * 8 ? want : sm_count() * 8);
#define RMB(N) rms_bwd_kernel<N><<<grid, 256, 0, stream>>>(a);
  MDL_NCH_DISPATCH(a.D, RMB)
#undef RMB
  return cudaGetLastError();
}

}  // namespace mdl

// ---------------------------------------------------------------------------
// LayerNorm backward for callers that cannot allocate (see norm_noalloc.h):
// the per-CTA partial sums live in a fixed file-scope device array instead of
// a caller-provided buffer. Builds on mdl::layernorm_bwd unchanged.
#include <cstdio>
#include <mutex>

#include "norm_noalloc.h"

namespace {

constexpr long long kNoAllocScratchFloats = MDL_LN_BWD_NOALLOC_SCRATCH_BYTES / sizeof(float);
static __device__ __align__(256) float g_ln_bwd_noalloc_scratch[kNoAllocScratchFloats];

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
float* g_noalloc_scratch_ptr[kNoAllocMaxDevices] = {};
thread_local char g_noalloc_message[256] = "";

int noalloc_reject(const char* msg) {
  std::snprintf(g_noalloc_message, sizeof(g_noalloc_message), "%s", msg);
  return -1;
}

// Device address of the scratch array on the current device, looked up once per
// device (host code only holds a stand-in for the symbol, never its address).
cudaError_t noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_ln_bwd_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" const char* mdl_noalloc_last_error(void) { return g_noalloc_message; }

extern "C" int mdl_layernorm_bwd_noalloc(const void* dy, const void* dy_bcast, float bcast_scale, const void* a,
                                         const void* b, const float* mean, const float* rstd, const float* gamma,
                                         void* dx, void* dx2, float* dgamma, float* dbeta, int B, int T, int D,
                                         int mix, cudaStream_t stream) {
  g_noalloc_message[0] = '\0';
  if (B < 0 || T <= 0 || D <= 0 || D % 8 != 0 || D > 2048)
    return noalloc_reject("mdl_layernorm_bwd_noalloc: need B >= 0, T >= 1 and D a multiple of 8 in [8, 2048]");
  if (mix && (D % T != 0 || (D / T) % 8 != 0))
    return noalloc_reject("mdl_layernorm_bwd_noalloc: token mixing needs D / T to be a multiple of 8");
  if (dy == nullptr && dy_bcast == nullptr)
    return noalloc_reject("mdl_layernorm_bwd_noalloc: one of dy / dy_bcast is required");
  const long long per_cta = 2LL * D;  // gamma and beta partial sums of one CTA
  const long long max_grid = kNoAllocScratchFloats / per_cta;
  if (max_grid < 1) return noalloc_reject("mdl_layernorm_bwd_noalloc: D exceeds the 2 MiB scratch array");
  if (B == 0) return 0;
  int dev = 0, smem_max = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (mdl::layernorm_bwd_smem(T, D, mix) > static_cast<size_t>(smem_max)) {
    char msg[200];
    std::snprintf(msg, sizeof(msg),
                  "mdl_layernorm_bwd_noalloc: ((mix ? T : 0) + 16) * D * 4 = %zu bytes of shared memory exceeds the "
                  "device's %d", mdl::layernorm_bwd_smem(T, D, mix), smem_max);
    return noalloc_reject(msg);
  }
  float* scratch = nullptr;
  e = noalloc_scratch(&scratch);
  if (e != cudaSuccess) return static_cast<int>(e);
  int grid = mdl::layernorm_bwd_grid(B);
  if (grid > max_grid) grid = static_cast<int>(max_grid);
  mdl::LNBwdArgs args;
  args.dy = dy;
  args.dy_bcast = dy_bcast;
  args.bcast_scale = bcast_scale;
  args.a = a;
  args.b = b;
  args.mean = mean;
  args.rstd = rstd;
  args.gamma = gamma;
  args.dx = dx;
  args.dx2 = dx2;
  args.partials = scratch;
  args.dgamma = dgamma;
  args.dbeta = dbeta;
  args.B = B;
  args.T = T;
  args.D = D;
  args.mix = mix ? 1 : 0;
  args.grid = grid;
  e = mdl::layernorm_bwd(args, stream);
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}
