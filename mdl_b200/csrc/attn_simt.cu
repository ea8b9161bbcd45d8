// Suffix attention for small head widths (8, 16; also 64) on the CUDA cores.
//
// Same contract as the tcgen05 flash attention (fmha.h): qkv [B, Lk, 3*D] bf16 with
// D = H * HD, the queries are the last Lq tokens, key j is visible to query row p iff
// kstart[b] <= j and (!causal or j <= p or j >= Lk - ktail or p >= Lk - ktail) and
// (j < Lk - kexcl or p >= Lk - kexcl); query rows before kstart[b] output zero. It
// serves the head widths the tensor-core kernel does not take -- the reference's
// production LONGER encoders run 32-wide tokens over 4 heads (head width 8) -- where an
// MMA tile would be mostly padding.
//
// Forward: a thread owns one query row of one head (128 rows per CTA); the CTA stages
// 64-key tiles of K and V (fp32) in shared memory and every thread runs an online
// softmax in base 2 over 16-key chunks (one rescale per chunk). Causal CTAs stop at their
// last query row and then visit only the trailing always-visible tokens.
// Few queries over many keys (Lq <= 64, head width <= 16): the key tiles are split over a
// CTA's four warps instead (see attn_simt_fwd_split_kernel).
// Backward (three launches): D_q = dO . O per query; dQ with a thread per query row
// (recomputing P from the saved log-sum-exp); dK and dV with a thread per key row over
// staged query tiles. Every element of dqkv is written by exactly one thread (no
// atomics); Q rows that are not queries get zero.
#include "attn_simt.h"

#include <cuda_bf16.h>
#include <math_constants.h>

namespace mdl {
namespace {

constexpr int kRows = 128;   // query (forward, dQ) or key (dK/dV) rows per CTA
constexpr int kTile = 64;    // staged rows of the other side
// keys per online-softmax rescale (fewer for wide heads, whose accumulators fill the registers)
template <int HD>
__host__ __device__ constexpr int chunk_of() { return HD >= 64 ? 4 : 16; }
constexpr float kLog2e = 1.4426950408889634f;
// threads per key row in the dK/dV kernel
template <int HD>
__host__ __device__ constexpr int keys_split() { return HD >= 64 ? 2 : 1; }

struct Vis {
  int Lk, Lq, kst, causal, tail0, excl0;
  __device__ __forceinline__ bool operator()(int p, int j) const {
    return j >= kst && (!causal || j <= p || j >= tail0 || p >= tail0) && (j < excl0 || p >= excl0);
  }
};

__device__ __forceinline__ Vis make_vis(const AttnSimtArgs& a, int b) {
  Vis v;
  v.Lk = a.Lk;
  v.Lq = a.Lq;
  int k = a.kstart[b];
  v.kst = k < 0 ? 0 : (k > a.Lk ? a.Lk : k);
  v.causal = a.causal;
  v.tail0 = a.causal ? a.Lk - a.ktail : a.Lk;
  v.excl0 = a.causal ? a.Lk - a.kexcl : a.Lk;
  return v;
}

// Rows [lo, hi) of head h's K (part 1) or V (part 2), or Q (part 0), as fp32 into s[kTile][HD].
template <int HD>
__device__ __forceinline__ void stage(float (*s)[HD], const __nv_bfloat16* base, long long row_stride, int col0,
                                      int lo, int hi) {
  for (int i = threadIdx.x; i < kTile * HD; i += blockDim.x) {
    const int r = i / HD, c = i % HD;
    const int j = lo + r;
    s[r][c] = j < hi ? __bfloat162float(base[static_cast<long long>(j) * row_stride + col0 + c]) : 0.f;
  }
}

// Grid: x = sample * row blocks + row block (samples can exceed the 65535 limit of y / z), y = head.
__device__ __forceinline__ void block_coords(int rows, int& b, int& blk) {
  const int nblk = (rows + kRows - 1) / kRows;
  b = static_cast<int>(blockIdx.x / nblk);
  blk = static_cast<int>(blockIdx.x - static_cast<unsigned>(b) * nblk);
}

template <int HD>
__global__ void __launch_bounds__(kRows) attn_simt_fwd_kernel(AttnSimtArgs a) {
  __shared__ float sK[kTile][HD];
  __shared__ float sV[kTile][HD];
  int b, blk;
  block_coords(a.Lq, b, blk);
  const int h = blockIdx.y;
  const int qi = blk * kRows + threadIdx.x;
  const int D = a.H * HD;
  const long long rs = 3LL * D;
  const __nv_bfloat16* base = a.qkv + static_cast<long long>(b) * a.Lk * rs;
  const Vis vis = make_vis(a, b);
  const int p = a.Lk - a.Lq + qi;
  const bool qvalid = qi < a.Lq && p >= vis.kst;
  float q[HD], o[HD];
#pragma unroll
  for (int d = 0; d < HD; ++d) {
    q[d] = qvalid ? __bfloat162float(base[static_cast<long long>(p) * rs + h * HD + d]) * a.scale * kLog2e : 0.f;
    o[d] = 0.f;
  }
  float m = -CUDART_INF_F, l = 0.f;
  // key ranges: [kst, hi) and, for causal CTAs, the trailing tokens after hi
  const int last_p = a.Lk - a.Lq + min(a.Lq, (blk + 1) * kRows) - 1;
  const int hi = a.causal ? min(a.Lk, last_p + 1) : a.Lk;
  const int tail_lo = a.causal ? max(hi, vis.tail0) : a.Lk;
  for (int range = 0; range < 2; ++range) {
    const int r0 = range == 0 ? vis.kst : max(tail_lo, vis.kst);
    const int r1 = range == 0 ? hi : a.Lk;
    for (int j0 = r0; j0 < r1; j0 += kTile) {
      __syncthreads();
      stage<HD>(sK, base, rs, D + h * HD, j0, r1);
      stage<HD>(sV, base, rs, 2 * D + h * HD, j0, r1);
      __syncthreads();
      if (!qvalid) continue;
      const int n = min(kTile, r1 - j0);
      constexpr int kChunk = chunk_of<HD>();
      for (int c0 = 0; c0 < n; c0 += kChunk) {
        float s[kChunk];
        float mc = m;
#pragma unroll
        for (int u = 0; u < kChunk; ++u) {
          const int jj = c0 + u;
          float t = -CUDART_INF_F;
          if (jj < n && vis(p, j0 + jj)) {
            t = 0.f;
#pragma unroll
            for (int d = 0; d < HD; ++d) t = fmaf(q[d], sK[jj][d], t);
          }
          s[u] = t;
          mc = fmaxf(mc, t);
        }
        if (mc == -CUDART_INF_F) continue;  // nothing visible in this chunk yet
        const float corr = exp2f(m - mc);   // 0 when m = -inf
        l *= corr;
#pragma unroll
        for (int d = 0; d < HD; ++d) o[d] *= corr;
#pragma unroll
        for (int u = 0; u < kChunk; ++u) {
          if (s[u] == -CUDART_INF_F) continue;
          const float pr = exp2f(s[u] - mc);
          l += pr;
#pragma unroll
          for (int d = 0; d < HD; ++d) o[d] = fmaf(pr, sV[c0 + u][d], o[d]);
        }
        m = mc;
      }
    }
  }
  if (qi >= a.Lq) return;
  const bool any = qvalid && l > 0.f;
  const float inv = any ? 1.f / l : 0.f;
  __nv_bfloat16* out = a.out + (static_cast<long long>(b) * a.Lq + qi) * D + h * HD;
#pragma unroll
  for (int d = 0; d < HD; ++d) out[d] = __float2bfloat16(o[d] * inv);
  a.lse[(static_cast<long long>(b) * a.H + h) * a.Lq + qi] = any ? m + log2f(l) : CUDART_INF_F;
}

// ---- few queries (LONGER cross blocks: R + G of a few dozen over thousands of keys)
// A CTA takes 32 query rows and splits the key tiles over its four warps (tile k to warp
// k % 4, each staging its own tiles: warp-local synchronisation only); the four partial
// (max, sum, accumulator) triples are merged through shared memory at the end, so all 128
// threads work although the query count is far below 128.
constexpr int kSplit = 4;
constexpr int kSplitRows = 32;

__device__ __forceinline__ void split_coords(int rows, int& b, int& blk) {
  const int nblk = (rows + kSplitRows - 1) / kSplitRows;
  b = static_cast<int>(blockIdx.x / nblk);
  blk = static_cast<int>(blockIdx.x - static_cast<unsigned>(b) * nblk);
}

template <int HD>
__device__ __forceinline__ void stage_warp(float (*s)[HD], const __nv_bfloat16* base, long long row_stride, int col0,
                                           int lo, int hi, int lane) {
  for (int i = lane; i < kTile * HD; i += 32) {
    const int r = i / HD, c = i % HD;
    const int j = lo + r;
    s[r][c] = j < hi ? __bfloat162float(base[static_cast<long long>(j) * row_stride + col0 + c]) : 0.f;
  }
}

template <int HD>
__global__ void __launch_bounds__(kSplit * 32) attn_simt_fwd_split_kernel(AttnSimtArgs a) {
  __shared__ float sK[kSplit][kTile][HD];
  __shared__ float sV[kSplit][kTile][HD];
  __shared__ float sM[kSplit][kSplitRows], sL[kSplit][kSplitRows];
  __shared__ float sO[kSplit][kSplitRows][HD + 1];
  int b, blk;
  split_coords(a.Lq, b, blk);
  const int h = blockIdx.y;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qi = blk * kSplitRows + lane;
  const int D = a.H * HD;
  const long long rs = 3LL * D;
  const __nv_bfloat16* base = a.qkv + static_cast<long long>(b) * a.Lk * rs;
  const Vis vis = make_vis(a, b);
  const int p = a.Lk - a.Lq + qi;
  const bool qvalid = qi < a.Lq && p >= vis.kst;
  float q[HD], o[HD];
#pragma unroll
  for (int d = 0; d < HD; ++d) {
    q[d] = qvalid ? __bfloat162float(base[static_cast<long long>(p) * rs + h * HD + d]) * a.scale * kLog2e : 0.f;
    o[d] = 0.f;
  }
  float m = -CUDART_INF_F, l = 0.f;
  const int last_p = a.Lk - a.Lq + min(a.Lq, (blk + 1) * kSplitRows) - 1;
  const int hi = a.causal ? min(a.Lk, last_p + 1) : a.Lk;
  const int tail_lo = a.causal ? max(hi, vis.tail0) : a.Lk;
  int idx = 0;
  for (int range = 0; range < 2; ++range) {
    const int r0 = range == 0 ? vis.kst : max(tail_lo, vis.kst);
    const int r1 = range == 0 ? hi : a.Lk;
    for (int j0 = r0; j0 < r1; j0 += kTile, ++idx) {
      if (idx % kSplit != w) continue;
      __syncwarp();
      stage_warp<HD>(sK[w], base, rs, D + h * HD, j0, r1, lane);
      stage_warp<HD>(sV[w], base, rs, 2 * D + h * HD, j0, r1, lane);
      __syncwarp();
      if (!qvalid) continue;
      const int n = min(kTile, r1 - j0);
      constexpr int kChunk = chunk_of<HD>();
      for (int c0 = 0; c0 < n; c0 += kChunk) {
        float s[kChunk];
        float mc = m;
#pragma unroll
        for (int u = 0; u < kChunk; ++u) {
          const int jj = c0 + u;
          float t = -CUDART_INF_F;
          if (jj < n && vis(p, j0 + jj)) {
            t = 0.f;
#pragma unroll
            for (int d = 0; d < HD; ++d) t = fmaf(q[d], sK[w][jj][d], t);
          }
          s[u] = t;
          mc = fmaxf(mc, t);
        }
        if (mc == -CUDART_INF_F) continue;
        const float corr = exp2f(m - mc);
        l *= corr;
#pragma unroll
        for (int d = 0; d < HD; ++d) o[d] *= corr;
#pragma unroll
        for (int u = 0; u < kChunk; ++u) {
          if (s[u] == -CUDART_INF_F) continue;
          const float pr = exp2f(s[u] - mc);
          l += pr;
#pragma unroll
          for (int d = 0; d < HD; ++d) o[d] = fmaf(pr, sV[w][c0 + u][d], o[d]);
        }
        m = mc;
      }
    }
  }
  sM[w][lane] = m;
  sL[w][lane] = l;
#pragma unroll
  for (int d = 0; d < HD; ++d) sO[w][lane][d] = o[d];
  __syncthreads();
  if (w != 0 || qi >= a.Lq) return;
  float M = -CUDART_INF_F;
#pragma unroll
  for (int g = 0; g < kSplit; ++g) M = fmaxf(M, sM[g][lane]);
  float L = 0.f, O[HD];
#pragma unroll
  for (int d = 0; d < HD; ++d) O[d] = 0.f;
  if (M != -CUDART_INF_F) {
#pragma unroll
    for (int g = 0; g < kSplit; ++g) {
      if (sM[g][lane] == -CUDART_INF_F) continue;
      const float f = exp2f(sM[g][lane] - M);
      L += sL[g][lane] * f;
#pragma unroll
      for (int d = 0; d < HD; ++d) O[d] = fmaf(sO[g][lane][d], f, O[d]);
    }
  }
  const bool any = qvalid && L > 0.f;
  const float inv = any ? 1.f / L : 0.f;
  __nv_bfloat16* out = a.out + (static_cast<long long>(b) * a.Lq + qi) * D + h * HD;
#pragma unroll
  for (int d = 0; d < HD; ++d) out[d] = __float2bfloat16(O[d] * inv);
  a.lse[(static_cast<long long>(b) * a.H + h) * a.Lq + qi] = any ? M + log2f(L) : CUDART_INF_F;
}

template <int HD>
__global__ void __launch_bounds__(kSplit * 32) attn_simt_dq_split_kernel(AttnSimtArgs a) {
  __shared__ float sK[kSplit][kTile][HD];
  __shared__ float sV[kSplit][kTile][HD];
  __shared__ float sQ[kSplit][kSplitRows][HD + 1];  // the warps' partial dQ
  int b, blk;
  split_coords(a.Lq, b, blk);
  const int h = blockIdx.y;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qi = blk * kSplitRows + lane;
  const int D = a.H * HD;
  const long long rs = 3LL * D;
  const __nv_bfloat16* base = a.qkv + static_cast<long long>(b) * a.Lk * rs;
  const Vis vis = make_vis(a, b);
  const int p = a.Lk - a.Lq + qi;
  const long long qoff = (static_cast<long long>(b) * a.H + h) * a.Lq + qi;
  const float lse = qi < a.Lq ? a.lse[qoff] : CUDART_INF_F;
  const bool qvalid = qi < a.Lq && p >= vis.kst && lse != CUDART_INF_F;
  const float c2 = a.scale * kLog2e;
  float q[HD], dO[HD], dq[HD];
  const long long ooff = (static_cast<long long>(b) * a.Lq + qi) * D + h * HD;
#pragma unroll
  for (int d = 0; d < HD; ++d) {
    q[d] = qvalid ? __bfloat162float(base[static_cast<long long>(p) * rs + h * HD + d]) * c2 : 0.f;
    dO[d] = qvalid ? __bfloat162float(a.dout[ooff + d]) : 0.f;
    dq[d] = 0.f;
  }
  const float Dq = qvalid ? a.dsum[qoff] : 0.f;
  const int last_p = a.Lk - a.Lq + min(a.Lq, (blk + 1) * kSplitRows) - 1;
  const int hi = a.causal ? min(a.Lk, last_p + 1) : a.Lk;
  const int tail_lo = a.causal ? max(hi, vis.tail0) : a.Lk;
  int idx = 0;
  for (int range = 0; range < 2; ++range) {
    const int r0 = range == 0 ? vis.kst : max(tail_lo, vis.kst);
    const int r1 = range == 0 ? hi : a.Lk;
    for (int j0 = r0; j0 < r1; j0 += kTile, ++idx) {
      if (idx % kSplit != w) continue;
      __syncwarp();
      stage_warp<HD>(sK[w], base, rs, D + h * HD, j0, r1, lane);
      stage_warp<HD>(sV[w], base, rs, 2 * D + h * HD, j0, r1, lane);
      __syncwarp();
      if (!qvalid) continue;
      const int n = min(kTile, r1 - j0);
      for (int jj = 0; jj < n; ++jj) {
        if (!vis(p, j0 + jj)) continue;
        float s = 0.f, dp = 0.f;
#pragma unroll
        for (int d = 0; d < HD; ++d) {
          s = fmaf(q[d], sK[w][jj][d], s);
          dp = fmaf(dO[d], sV[w][jj][d], dp);
        }
        const float ds = exp2f(s - lse) * (dp - Dq);
#pragma unroll
        for (int d = 0; d < HD; ++d) dq[d] = fmaf(ds, sK[w][jj][d], dq[d]);
      }
    }
  }
#pragma unroll
  for (int d = 0; d < HD; ++d) sQ[w][lane][d] = dq[d];
  __syncthreads();
  if (w != 0 || qi >= a.Lq) return;
  __nv_bfloat16* dst = a.dqkv + (static_cast<long long>(b) * a.Lk + p) * rs + h * HD;
#pragma unroll
  for (int d = 0; d < HD; ++d) {
    float t = 0.f;
#pragma unroll
    for (int g = 0; g < kSplit; ++g) t += sQ[g][lane][d];
    dst[d] = __float2bfloat16(t * a.scale);
  }
}

// D_q = sum_d dO[q, d] * O[q, d] per (b, h, q).
template <int HD>
__global__ void attn_simt_dsum_kernel(AttnSimtArgs a) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(a.B) * a.H * a.Lq;
  if (i >= total) return;
  const int qi = static_cast<int>(i % a.Lq);
  const long long bh = i / a.Lq;
  const int h = static_cast<int>(bh % a.H), b = static_cast<int>(bh / a.H);
  const long long off = (static_cast<long long>(b) * a.Lq + qi) * a.H * HD + h * HD;
  float s = 0.f;
#pragma unroll
  for (int d = 0; d < HD; ++d) s = fmaf(__bfloat162float(a.dout[off + d]), __bfloat162float(a.out[off + d]), s);
  a.dsum[i] = s;
}

template <int HD>
__global__ void __launch_bounds__(kRows) attn_simt_dq_kernel(AttnSimtArgs a) {
  __shared__ float sK[kTile][HD];
  __shared__ float sV[kTile][HD];
  int b, blk;
  block_coords(a.Lq, b, blk);
  const int h = blockIdx.y;
  const int qi = blk * kRows + threadIdx.x;
  const int D = a.H * HD;
  const long long rs = 3LL * D;
  const __nv_bfloat16* base = a.qkv + static_cast<long long>(b) * a.Lk * rs;
  const Vis vis = make_vis(a, b);
  const int p = a.Lk - a.Lq + qi;
  const long long qoff = (static_cast<long long>(b) * a.H + h) * a.Lq + qi;
  const float lse = qi < a.Lq ? a.lse[qoff] : CUDART_INF_F;
  const bool qvalid = qi < a.Lq && p >= vis.kst && lse != CUDART_INF_F;
  const float c2 = a.scale * kLog2e;
  float q[HD], dO[HD], dq[HD];
  const long long ooff = (static_cast<long long>(b) * a.Lq + qi) * D + h * HD;
#pragma unroll
  for (int d = 0; d < HD; ++d) {
    q[d] = qvalid ? __bfloat162float(base[static_cast<long long>(p) * rs + h * HD + d]) * c2 : 0.f;
    dO[d] = qvalid ? __bfloat162float(a.dout[ooff + d]) : 0.f;
    dq[d] = 0.f;
  }
  const float Dq = qvalid ? a.dsum[qoff] : 0.f;
  const int last_p = a.Lk - a.Lq + min(a.Lq, (blk + 1) * kRows) - 1;
  const int hi = a.causal ? min(a.Lk, last_p + 1) : a.Lk;
  const int tail_lo = a.causal ? max(hi, vis.tail0) : a.Lk;
  for (int range = 0; range < 2; ++range) {
    const int r0 = range == 0 ? vis.kst : max(tail_lo, vis.kst);
    const int r1 = range == 0 ? hi : a.Lk;
    for (int j0 = r0; j0 < r1; j0 += kTile) {
      __syncthreads();
      stage<HD>(sK, base, rs, D + h * HD, j0, r1);
      stage<HD>(sV, base, rs, 2 * D + h * HD, j0, r1);
      __syncthreads();
      if (!qvalid) continue;
      const int n = min(kTile, r1 - j0);
      for (int jj = 0; jj < n; ++jj) {
        if (!vis(p, j0 + jj)) continue;
        float s = 0.f, dp = 0.f;
#pragma unroll
        for (int d = 0; d < HD; ++d) {
          s = fmaf(q[d], sK[jj][d], s);
          dp = fmaf(dO[d], sV[jj][d], dp);
        }
        const float ds = exp2f(s - lse) * (dp - Dq);
#pragma unroll
        for (int d = 0; d < HD; ++d) dq[d] = fmaf(ds, sK[jj][d], dq[d]);
      }
    }
  }
  if (qi >= a.Lq) return;
  __nv_bfloat16* dst = a.dqkv + (static_cast<long long>(b) * a.Lk + p) * rs + h * HD;
#pragma unroll
  for (int d = 0; d < HD; ++d) dst[d] = __float2bfloat16(dq[d] * a.scale);
}

template <int HD>
__global__ void __launch_bounds__(kRows) attn_simt_dkv_kernel(AttnSimtArgs a) {
  // Wide heads (64) split a key's head dimension over TPK adjacent threads (dot products
  // completed with a shuffle), so each thread's K, V, dK and dV accumulators stay in registers.
  // The threads of a key take interleaved dimensions (hsel, hsel + TPK, ...): their shared-memory
  // reads of a staged row then fall in different banks (contiguous halves 32 words apart would
  // share a bank).
  constexpr int TPK = keys_split<HD>();
  constexpr int HW = HD / TPK;         // dimensions per thread
  constexpr int KPC = kRows / TPK;     // keys per CTA
  __shared__ float sQ[kTile][HD];
  __shared__ float sO[kTile][HD];  // dO of the staged queries
  __shared__ float sL[kTile];      // their log-sum-exp
  __shared__ float sD[kTile];      // their D_q
  const int nblk = (a.Lk + KPC - 1) / KPC;
  const int b = static_cast<int>(blockIdx.x / nblk);
  const int blk = static_cast<int>(blockIdx.x - static_cast<unsigned>(b) * nblk);
  const int h = blockIdx.y;
  const int j = blk * KPC + static_cast<int>(threadIdx.x) / TPK;  // key row
  const int hsel = static_cast<int>(threadIdx.x) % TPK;          // dimensions hsel + TPK * i
  const int D = a.H * HD;
  const long long rs = 3LL * D;
  const __nv_bfloat16* base = a.qkv + static_cast<long long>(b) * a.Lk * rs;
  const Vis vis = make_vis(a, b);
  const bool kvalid = j < a.Lk && j >= vis.kst;
  const float c2 = a.scale * kLog2e;
  float k[HW], v[HW], dk[HW], dv[HW];
#pragma unroll
  for (int d = 0; d < HW; ++d) {
    k[d] = kvalid ? __bfloat162float(base[static_cast<long long>(j) * rs + D + h * HD + hsel + TPK * d]) : 0.f;
    v[d] = kvalid ? __bfloat162float(base[static_cast<long long>(j) * rs + 2 * D + h * HD + hsel + TPK * d])
                  : 0.f;
    dk[d] = 0.f;
    dv[d] = 0.f;
  }
  // queries that may see keys of this CTA: rows >= the first key row (causal) or every
  // query when the CTA holds trailing tokens; all queries otherwise
  const int q_first = a.Lk - a.Lq;
  const int jmin = blk * KPC;
  const int jmax = min(a.Lk, jmin + KPC) - 1;
  int p_lo = max(q_first, vis.kst);
  if (a.causal && jmax < vis.tail0) p_lo = max(p_lo, jmin);
  const __nv_bfloat16* dO_base = a.dout + static_cast<long long>(b) * a.Lq * D + h * HD;
  const long long lbase = (static_cast<long long>(b) * a.H + h) * a.Lq;
  for (int p0 = p_lo; p0 < a.Lk; p0 += kTile) {
    __syncthreads();
    for (int i = threadIdx.x; i < kTile * HD; i += blockDim.x) {
      const int r = i / HD, c = i % HD;
      const int p = p0 + r;
      const bool ok = p < a.Lk;
      sQ[r][c] = ok ? __bfloat162float(base[static_cast<long long>(p) * rs + h * HD + c]) * c2 : 0.f;
      sO[r][c] = ok ? __bfloat162float(dO_base[static_cast<long long>(p - q_first) * D + c]) : 0.f;
    }
    for (int r = threadIdx.x; r < kTile; r += blockDim.x) {
      const int p = p0 + r;
      const bool ok = p < a.Lk;
      sL[r] = ok ? a.lse[lbase + (p - q_first)] : CUDART_INF_F;
      sD[r] = ok ? a.dsum[lbase + (p - q_first)] : 0.f;
    }
    __syncthreads();
    // threads of one key stay together (the partial dot products meet in a shuffle), so a
    // key group skips as a whole: j and the visibility are the same for its TPK threads
    if (!kvalid) continue;
    const int n = min(kTile, a.Lk - p0);
    for (int r = 0; r < n; ++r) {
      const int p = p0 + r;
      if (sL[r] == CUDART_INF_F || !vis(p, j)) continue;
      float s = 0.f, dp = 0.f;
#pragma unroll
      for (int d = 0; d < HW; ++d) {
        s = fmaf(sQ[r][hsel + TPK * d], k[d], s);
        dp = fmaf(sO[r][hsel + TPK * d], v[d], dp);
      }
      if constexpr (TPK > 1) {
        const unsigned grp = ((1u << TPK) - 1u) << ((threadIdx.x & 31) & ~(TPK - 1));
#pragma unroll
        for (int o = 1; o < TPK; o <<= 1) {
          s += __shfl_xor_sync(grp, s, o, TPK);
          dp += __shfl_xor_sync(grp, dp, o, TPK);
        }
      }
      const float pr = exp2f(s - sL[r]);
      const float ds = pr * (dp - sD[r]);
#pragma unroll
      for (int d = 0; d < HW; ++d) {
        dv[d] = fmaf(pr, sO[r][hsel + TPK * d], dv[d]);
        dk[d] = fmaf(ds, sQ[r][hsel + TPK * d], dk[d]);  // sQ holds q * scale * log2(e)
      }
    }
  }
  if (j >= a.Lk) return;
  __nv_bfloat16* dst = a.dqkv + (static_cast<long long>(b) * a.Lk + j) * rs + h * HD + hsel;
#pragma unroll
  for (int d = 0; d < HW; ++d) {
    dst[D + TPK * d] = __float2bfloat16(dk[d] / kLog2e);
    dst[2 * D + TPK * d] = __float2bfloat16(dv[d]);
    if (j < q_first) dst[TPK * d] = __float2bfloat16(0.f);  // Q rows that are not queries
  }
}

// Few queries per sample: the key-split kernels (every thread busy); otherwise a thread per query.
template <int HD>
bool use_split(const AttnSimtArgs& a) {
  return HD <= 16 && a.Lq <= 2 * kSplitRows && a.Lk >= 4 * kTile;
}

template <int HD>
cudaError_t launch_fwd(const AttnSimtArgs& a, cudaStream_t st) {
  if constexpr (HD <= 16) {
    if (use_split<HD>(a)) {
      const dim3 g(static_cast<unsigned>(a.B) * ((a.Lq + kSplitRows - 1) / kSplitRows), a.H);
      attn_simt_fwd_split_kernel<HD><<<g, kSplit * 32, 0, st>>>(a);
      return cudaGetLastError();
    }
  }
  const dim3 grid(static_cast<unsigned>(a.B) * ((a.Lq + kRows - 1) / kRows), a.H);
  attn_simt_fwd_kernel<HD><<<grid, kRows, 0, st>>>(a);
  return cudaGetLastError();
}

template <int HD>
cudaError_t launch_bwd(const AttnSimtArgs& a, cudaStream_t st) {
  const long long n = static_cast<long long>(a.B) * a.H * a.Lq;
  attn_simt_dsum_kernel<HD><<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  bool split = false;
  if constexpr (HD <= 16) {
    split = use_split<HD>(a);
    if (split)
      attn_simt_dq_split_kernel<HD>
          <<<dim3(static_cast<unsigned>(a.B) * ((a.Lq + kSplitRows - 1) / kSplitRows), a.H), kSplit * 32, 0, st>>>(a);
  }
  if (!split)
    attn_simt_dq_kernel<HD><<<dim3(static_cast<unsigned>(a.B) * ((a.Lq + kRows - 1) / kRows), a.H), kRows, 0, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  constexpr int kpc = kRows / keys_split<HD>();
  attn_simt_dkv_kernel<HD><<<dim3(static_cast<unsigned>(a.B) * ((a.Lk + kpc - 1) / kpc), a.H), kRows, 0, st>>>(a);
  return cudaGetLastError();
}

bool args_ok(const AttnSimtArgs& a) {
  return a.qkv != nullptr && a.kstart != nullptr && a.B > 0 && a.H > 0 && a.Lq > 0 && a.Lq <= a.Lk &&
         a.ktail >= 0 && a.ktail <= a.Lq && a.kexcl >= 0 && a.kexcl <= a.ktail && a.H <= 65535 &&
         static_cast<long long>(a.B) * ((a.Lk + kRows / 2 - 1) / (kRows / 2)) <= 0x7fffffffLL;
}

}  // namespace

bool attn_simt_supported(int hd) { return hd == 8 || hd == 16 || hd == 64; }

cudaError_t attn_simt_fwd(const AttnSimtArgs& a, cudaStream_t stream) {
  if (!args_ok(a) || a.out == nullptr || a.lse == nullptr) return cudaErrorInvalidValue;
  switch (a.hd) {
    case 8: return launch_fwd<8>(a, stream);
    case 16: return launch_fwd<16>(a, stream);
    case 64: return launch_fwd<64>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t attn_simt_bwd(const AttnSimtArgs& a, cudaStream_t stream) {
  if (!args_ok(a) || a.out == nullptr || a.lse == nullptr || a.dout == nullptr || a.dqkv == nullptr ||
      a.dsum == nullptr)
    return cudaErrorInvalidValue;
  switch (a.hd) {
    case 8: return launch_bwd<8>(a, stream);
    case 16: return launch_bwd<16>(a, stream);
    case 64: return launch_bwd<64>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace mdl
