// Small fused kernels for sm_100a: token mean, column sums, the task-head
// logit + BCE kernel and the dense optimizers.
#include "common.cuh"
#include "misc.h"

namespace mdl {
namespace {

__device__ __forceinline__ void ld8(const __nv_bfloat16* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void st8(__nv_bfloat16* p, const float* v) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

int sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// one thread per 8 output columns of one sample
__global__ void token_mean_kernel(const __nv_bfloat16* x, __nv_bfloat16* out, int B, int T, int D) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int per_row = D / 8;
  if (idx >= static_cast<long long>(B) * per_row) return;
  const long long b = idx / per_row;
  const int c = static_cast<int>(idx - b * per_row) * 8;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int t = 0; t < T; ++t) {
    float v[8];
    ld8(x + (b * T + t) * D + c, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += v[e];
  }
  const float inv = 1.f / T;
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] *= inv;
  st8(out + b * D + c, acc);
}

// grid (ceil(N/256), G, splits); each thread sums a strided range of rows for one column
__global__ void colsum_kernel(const __nv_bfloat16* x, float* out, long long M, int N, long long ld, long long gs,
                              long long gs_out, float scale) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int g = blockIdx.y;
  if (n >= N) return;
  const long long rows_per = (M + gridDim.z - 1) / gridDim.z;
  const long long m0 = blockIdx.z * rows_per;
  const long long m1 = min(M, m0 + rows_per);
  const __nv_bfloat16* p = x + g * gs + n;
  float s = 0.f;
  for (long long m = m0; m < m1; ++m) s += __bfloat162float(p[m * ld]);
  atomicAdd(out + g * gs_out + n, s * scale);
}

// One warp per (b, task); H % 256 == 0 handled by 8-wide chunks per lane.
// Block = 8 warps working on rows of one task (grid.y = task). dw2 partials are
// reduced in shared memory per block before one atomicAdd per element.
__global__ void __launch_bounds__(256) head_bce_kernel(const HeadArgs p) {
  extern __shared__ float sdw[];  // [H] block partial of dw2
  const int task = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  const int H = p.H;
  const int stride_all = p.ntask * H;
  for (int k = threadIdx.x; k < H; k += blockDim.x) sdw[k] = 0.f;
  __syncthreads();
  const auto* act = reinterpret_cast<const __nv_bfloat16*>(p.act);
  const auto* pre = reinterpret_cast<const __nv_bfloat16*>(p.pre);
  auto* dpre = reinterpret_cast<__nv_bfloat16*>(p.dpre);
  const float* w2 = p.w2 + static_cast<long long>(task) * H;
  const float scale = p.task_scale ? p.task_scale[task] : 1.f;
  float loss_acc = 0.f, db_acc = 0.f;
  for (long long b = static_cast<long long>(blockIdx.x) * 8 + w; b < p.B; b += static_cast<long long>(gridDim.x) * 8) {
    const __nv_bfloat16* arow = act + b * stride_all + static_cast<long long>(task) * H;
    float s = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
      float v[8];
      ld8(arow + c, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) s += v[e] * __ldg(w2 + c + e);
    }
    s = warp_sum(s);
    const float z = s + (p.b2 ? p.b2[task] : 0.f);
    const long long bt = b * p.ntask + task;
    if (lane == 0 && p.logits) p.logits[bt] = z;
    if (p.labels == nullptr) continue;
    const float y = p.labels[bt];
    const float m = p.mask ? p.mask[bt] : 1.f;
    const float wgt = scale * m;
    // numerically stable BCE with logits
    const float bce = fmaxf(z, 0.f) - z * y + log1pf(expf(-fabsf(z)));
    loss_acc += wgt * bce;
    const float sig = 1.f / (1.f + expf(-z));
    const float dz = wgt * (sig - y);
    db_acc += dz;
    if (dpre == nullptr) continue;
    const __nv_bfloat16* prow = pre + b * stride_all + static_cast<long long>(task) * H;
    __nv_bfloat16* drow = dpre + b * stride_all + static_cast<long long>(task) * H;
    for (int c = lane * 8; c < H; c += 256) {
      float pv[8], av[8], o[8];
      ld8(prow + c, pv);
      ld8(arow + c, av);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = p.relu ? (pv[e] > 0.f ? 1.f : 0.f) : gelu_erf_grad(pv[e]);
        o[e] = dz * __ldg(w2 + c + e) * d;
        atomicAdd(&sdw[c + e], dz * av[e]);  // shared-memory atomics, folded below
      }
      st8(drow + c, o);
    }
  }
  // z, the loss term and dz are identical in every lane of the warp: lane 0 reports them.
  if (lane == 0) {
    if (p.loss && p.labels) atomicAdd(p.loss, loss_acc);
    if (p.db2 && p.dpre) atomicAdd(p.db2 + task, db_acc);
  }
  __syncthreads();
  if (p.dw2 && p.dpre)
    for (int k = threadIdx.x; k < H; k += blockDim.x) atomicAdd(p.dw2 + static_cast<long long>(task) * H + k, sdw[k]);
}

__device__ __forceinline__ float clip_of(const float* clip) { return clip ? *clip : 1.f; }

// One optimizer element update; ALGO 0 = Adam, 1 = RMSprop.
template <int ALGO>
__device__ __forceinline__ float opt_elem(const OptimArgs& a, float g, float p, float& s1, float& s2, float step_size,
                                          float bc2_sqrt) {
  if (a.weight_decay != 0.f) g += a.weight_decay * p;
  if (ALGO == 0) {
    s1 = a.beta1 * s1 + (1.f - a.beta1) * g;
    s2 = a.beta2 * s2 + (1.f - a.beta2) * g * g;
    return p - step_size * s1 / (sqrtf(s2) / bc2_sqrt + a.eps);
  }
  s1 = a.alpha * s1 + (1.f - a.alpha) * g * g;
  return p - a.lr * g / (sqrtf(s1) + a.eps);
}

// Vectorised (4 elements per thread and iteration) when n and every buffer allow it.
template <int ALGO>
__global__ void __launch_bounds__(256) optim_kernel(const OptimArgs a) {
  const float gs = a.grad_scale * clip_of(a.clip);
  const float step_size = a.lr / a.bias_correction1;
  const float bc2_sqrt = sqrtf(a.bias_correction2);
  __nv_bfloat16* sh = reinterpret_cast<__nv_bfloat16*>(a.shadow);
  float* grad = const_cast<float*>(a.grad);
  const long long n4 = a.n / 4;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long v = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; v < n4; v += stride) {
    const long long i = v * 4;
    const float4 g4 = *reinterpret_cast<const float4*>(grad + i);
    const float4 p4 = *reinterpret_cast<const float4*>(a.param + i);
    const float4 s14 = *reinterpret_cast<const float4*>(a.state1 + i);
    float4 s24 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (ALGO == 0) s24 = *reinterpret_cast<const float4*>(a.state2 + i);
    float g[4] = {g4.x * gs, g4.y * gs, g4.z * gs, g4.w * gs};
    float p[4] = {p4.x, p4.y, p4.z, p4.w};
    float s1[4] = {s14.x, s14.y, s14.z, s14.w};
    float s2[4] = {s24.x, s24.y, s24.z, s24.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) p[k] = opt_elem<ALGO>(a, g[k], p[k], s1[k], s2[k], step_size, bc2_sqrt);
    *reinterpret_cast<float4*>(a.param + i) = make_float4(p[0], p[1], p[2], p[3]);
    *reinterpret_cast<float4*>(a.state1 + i) = make_float4(s1[0], s1[1], s1[2], s1[3]);
    if (ALGO == 0) *reinterpret_cast<float4*>(a.state2 + i) = make_float4(s2[0], s2[1], s2[2], s2[3]);
    if (a.zero_grad) *reinterpret_cast<float4*>(grad + i) = make_float4(0.f, 0.f, 0.f, 0.f);
    if (sh) {
      const __nv_bfloat162 h0 = __floats2bfloat162_rn(p[0], p[1]);
      const __nv_bfloat162 h1 = __floats2bfloat162_rn(p[2], p[3]);
      uint2 u;
      u.x = *reinterpret_cast<const uint32_t*>(&h0);
      u.y = *reinterpret_cast<const uint32_t*>(&h1);
      *reinterpret_cast<uint2*>(sh + i) = u;
    }
  }
  // tail
  for (long long i = n4 * 4 + static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < a.n; i += stride) {
    float s1 = a.state1[i], s2 = ALGO == 0 ? a.state2[i] : 0.f;
    const float p = opt_elem<ALGO>(a, grad[i] * gs, a.param[i], s1, s2, step_size, bc2_sqrt);
    a.param[i] = p;
    a.state1[i] = s1;
    if (ALGO == 0) a.state2[i] = s2;
    if (a.zero_grad) grad[i] = 0.f;
    if (sh) sh[i] = __float2bfloat16_rn(p);
  }
}

__global__ void sqnorm_kernel(const float* g, long long n, float scale, float* out) {
  float s = 0.f;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float v = g[i];
    s += v * v;
  }
  s = warp_sum(s) * scale * scale;
  if ((threadIdx.x & 31) == 0) atomicAdd(out, s);
}

__global__ void clip_factor_kernel(const float* sum_sq, float max_norm, float* clip) {
  const float norm = sqrtf(*sum_sq);
  *clip = fminf(1.f, max_norm / (norm + 1e-6f));
}

__global__ void cast_kernel(const float* s, __nv_bfloat16* d, long long n) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    d[i] = __float2bfloat16_rn(s[i]);
}

int grid_for(long long n) {
  const long long want = (n + 255) / 256;
  const long long cap = static_cast<long long>(sms()) * 8;
  return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

}  // namespace

__global__ void __launch_bounds__(256) position_add_kernel(__nv_bfloat16* x, const float* __restrict__ pos,
                                                           const int* __restrict__ kstart, int B, int L, int D) {
  const long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (i >= static_cast<long long>(B) * L * D) return;
  const long long row = i / D;
  const int c = static_cast<int>(i - row * D);
  const int b = static_cast<int>(row / L);
  const int p = static_cast<int>(row - static_cast<long long>(b) * L) - kstart[b];
  if (p < 0) return;
  uint4* xp = reinterpret_cast<uint4*>(x + i);
  uint4 v = *xp;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
  const float4 a = *reinterpret_cast<const float4*>(pos + static_cast<long long>(p) * D + c);
  const float4 e = *reinterpret_cast<const float4*>(pos + static_cast<long long>(p) * D + c + 4);
  const float add[8] = {a.x, a.y, a.z, a.w, e.x, e.y, e.z, e.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = __bfloat1622float2(h[k]);
    h[k] = __floats2bfloat162_rn(f.x + add[2 * k], f.y + add[2 * k + 1]);
  }
  *xp = v;
}

// grid: (positions x D/8 threads, sample chunks); each thread sums its chunk of samples.
constexpr int kPosChunk = 64;
__global__ void __launch_bounds__(256) position_grad_kernel(const __nv_bfloat16* __restrict__ dx, float* dpos,
                                                            const int* __restrict__ kstart, int B, int L, int D) {
  const long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (i >= static_cast<long long>(L) * D) return;
  const int p = static_cast<int>(i / D);
  const int c = static_cast<int>(i - static_cast<long long>(p) * D);
  const int b0 = blockIdx.y * kPosChunk;
  const int b1 = min(B, b0 + kPosChunk);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  bool any = false;
  for (int b = b0; b < b1; ++b) {
    const int e = kstart[b] + p;
    if (e >= L) continue;
    any = true;
    const uint4 v = *reinterpret_cast<const uint4*>(dx + (static_cast<long long>(b) * L + e) * D + c);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __bfloat1622float2(h[k]);
      acc[2 * k] += f.x;
      acc[2 * k + 1] += f.y;
    }
  }
  if (!any) return;
#pragma unroll
  for (int k = 0; k < 8; ++k) atomicAdd(dpos + i + k, acc[k]);
}

cudaError_t position_add(void* x, const float* pos, const int* kstart, int B, int L, int D, cudaStream_t stream) {
  if (D % 8 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(pos) & 15))
    return cudaErrorInvalidValue;
  const long long vec = static_cast<long long>(B) * L * D / 8;
  if (vec == 0) return cudaSuccess;
  position_add_kernel<<<static_cast<unsigned>((vec + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<__nv_bfloat16*>(x), pos, kstart, B, L, D);
  return cudaGetLastError();
}

cudaError_t position_grad(const void* dx, float* dpos, const int* kstart, int B, int L, int D, cudaStream_t stream) {
  if (D % 8 || (reinterpret_cast<uintptr_t>(dx) & 15)) return cudaErrorInvalidValue;
  const long long vec = static_cast<long long>(L) * D / 8;
  if (vec == 0 || B == 0) return cudaSuccess;
  dim3 grid(static_cast<unsigned>((vec + 255) / 256), static_cast<unsigned>((B + kPosChunk - 1) / kPosChunk));
  position_grad_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(dx), dpos, kstart, B, L, D);
  return cudaGetLastError();
}

cudaError_t token_mean_fwd(const void* x, void* out, int B, int T, int D, cudaStream_t stream) {
  if (D % 8) return cudaErrorInvalidValue;
  const long long n = static_cast<long long>(B) * (D / 8);
  if (n == 0) return cudaSuccess;
  token_mean_kernel<<<static_cast<int>((n + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<__nv_bfloat16*>(out), B, T, D);
  return cudaGetLastError();
}

cudaError_t colsum_bf16(const void* x, float* out, int G, long long M, int N, long long ld, long long gs, float scale,
                        cudaStream_t stream, long long gs_out) {
  if (G <= 0 || M <= 0 || N <= 0) return cudaSuccess;
  const int bx = (N + 255) / 256;
  long long splits = (static_cast<long long>(sms()) * 4) / (static_cast<long long>(bx) * G);
  if (splits < 1) splits = 1;
  if (splits > M) splits = M;
  if (splits > 65535) splits = 65535;
  dim3 grid(bx, G, static_cast<unsigned>(splits));
  colsum_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const __nv_bfloat16*>(x), out, M, N, ld, gs,
                                          gs_out < 0 ? N : gs_out, scale);
  return cudaGetLastError();
}

cudaError_t head_bce(const HeadArgs& a, cudaStream_t stream) {
  if (a.H % 8 || a.B <= 0) return a.B <= 0 ? cudaSuccess : cudaErrorInvalidValue;
  int bx = (a.B + 7) / 8;
  const int cap = sms() * 2;
  if (bx > cap) bx = cap;
  dim3 grid(bx, a.ntask);
  const size_t smem = static_cast<size_t>(a.H) * sizeof(float);
  cudaFuncSetAttribute(head_bce_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  head_bce_kernel<<<grid, 256, smem, stream>>>(a);
  return cudaGetLastError();
}

namespace {
bool optim_aligned(const OptimArgs& a) {
  auto al = [](const void* p, uintptr_t m) { return (reinterpret_cast<uintptr_t>(p) & m) == 0; };
  return al(a.param, 15) && al(a.grad, 15) && al(a.state1, 15) && (a.state2 == nullptr || al(a.state2, 15)) &&
         (a.shadow == nullptr || al(a.shadow, 7));
}
int optim_grid(const OptimArgs& a) {
  int g = grid_for((a.n + 3) / 4);
  if (a.max_blocks > 0 && g > a.max_blocks) g = a.max_blocks;
  return g;
}
}  // namespace

cudaError_t adam_step(const OptimArgs& a, cudaStream_t stream) {
  if (a.n == 0) return cudaSuccess;
  if (!optim_aligned(a)) return cudaErrorInvalidValue;
  optim_kernel<0><<<optim_grid(a), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t rmsprop_step(const OptimArgs& a, cudaStream_t stream) {
  if (a.n == 0) return cudaSuccess;
  if (!optim_aligned(a)) return cudaErrorInvalidValue;
  optim_kernel<1><<<optim_grid(a), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t grad_sqnorm(const float* grad, long long n, float grad_scale, float* out, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  sqnorm_kernel<<<grid_for(n), 256, 0, stream>>>(grad, n, grad_scale, out);
  return cudaGetLastError();
}

cudaError_t clip_factor(const float* sum_sq, float max_norm, float* clip, cudaStream_t stream) {
  clip_factor_kernel<<<1, 1, 0, stream>>>(sum_sq, max_norm, clip);
  return cudaGetLastError();
}

namespace {
// One thread waits on an mbarrier that nothing arrives on: the bounded wait runs
// out, records MDL_ERR_MBAR_TIMEOUT and the kernel returns (self-test of the
// timeout path every tcgen05 pipeline in this library relies on).
__global__ void mbar_timeout_selftest_kernel(int* err, int* returned) {
  __shared__ __align__(8) uint64_t bar;
  mbar_init(&bar, 1);
  fence_barrier_init();
  if (!mbar_wait(&bar, 0, err, nullptr)) atomicAdd(returned, 1);
}
}  // namespace

cudaError_t mbar_timeout_selftest(int* err, int* returned, cudaStream_t stream) {
  mbar_timeout_selftest_kernel<<<1, 1, 0, stream>>>(err, returned);
  return cudaGetLastError();
}

cudaError_t cast_f32_bf16(const float* src, void* dst, long long n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  cast_kernel<<<grid_for(n), 256, 0, stream>>>(src, reinterpret_cast<__nv_bfloat16*>(dst), n);
  return cudaGetLastError();
}

}  // namespace mdl
