// NVLink symmetric-memory runtime and fused collectives for sm_100a.
//
// One process per GPU. Each rank cudaMalloc's its buffers, exports CUDA IPC
// handles once (exchanged over torch.distributed at setup), and maps every
// peer's buffers. Kernels then reach peer HBM with plain loads/stores/reductions
// over NVLink 5 / NVSwitch. No TMA is used on peer memory.
//
// dense_sync_update replaces the reference's DDP reducer + RMSprop step
// (src/train.py:5311-5324, :4826-4893): a reduce-scatter of the fp32 gradient
// (peer loads), the optimizer on the owned slice, and an all-gather of the
// updated bf16 weights (peer stores), fused in one kernel per bucket. On
// NVSwitch systems with multicast the same kernel shape runs on multimem
// instructions: the switch sums the gradient slice (ld_reduce) and replicates
// the updated weights (st), so each element crosses NVLink once.
#include "comm.h"
#include "common.cuh"

namespace mdl {

cudaError_t ipc_alloc(size_t bytes, void** ptr, cudaIpcMemHandle_t* handle) {
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return e;
  return cudaIpcGetMemHandle(handle, *ptr);
}
cudaError_t ipc_open(const cudaIpcMemHandle_t& handle, void** ptr) {
  return cudaIpcOpenMemHandle(ptr, handle, cudaIpcMemLazyEnablePeerAccess);
}
cudaError_t ipc_close(void* ptr) { return cudaIpcCloseMemHandle(ptr); }
cudaError_t ipc_free(void* ptr) { return cudaFree(ptr); }

namespace {

struct SigPtrs {
  unsigned* p[kMaxWorld];
};

__device__ __forceinline__ void st_release_sys(unsigned* addr, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* addr) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

__global__ void barrier_kernel(SigPtrs sig, unsigned* counter, int rank, int world, int* err, uint64_t limit_ns) {
  __shared__ unsigned epoch;
  if (threadIdx.x == 0) {
    epoch = *counter + 1u;
    *counter = epoch;
  }
  __syncthreads();
  const int t = threadIdx.x;
  if (t < world) {
    __threadfence_system();
    st_release_sys(sig.p[t] + rank, epoch);
    const uint64_t start = globaltimer_ns();
    // wrap-safe comparison of epochs
    while (static_cast<int>(ld_acquire_sys(sig.p[rank] + t) - epoch) < 0) {
      if (globaltimer_ns() - start > limit_ns) {
        record_error(err, MDL_ERR_PEER_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
}

struct SyncPtrs {
  float* grads[kMaxWorld];
  float* params[kMaxWorld];
  __nv_bfloat16* shadows[kMaxWorld];
};

__device__ __forceinline__ void opt_update(const DenseSyncArgs& a, float& p, float g, float& s1, float& s2) {
  if (a.weight_decay != 0.f) g += a.weight_decay * p;
  if (a.optimizer == 0) {
    s1 = a.beta1 * s1 + (1.f - a.beta1) * g;
    s2 = a.beta2 * s2 + (1.f - a.beta2) * g * g;
    p -= (a.lr / a.bias_correction1) * s1 / (sqrtf(s2) / sqrtf(a.bias_correction2) + a.eps);
  } else {
    s1 = a.alpha * s1 + (1.f - a.alpha) * g * g;
    p -= a.lr * g / (sqrtf(s1) + a.eps);
  }
}

__global__ void __launch_bounds__(256) dense_sync_kernel(const DenseSyncArgs a, const SyncPtrs ptr) {
  const long long total = a.end - a.begin;
  const long long chunk = ((total / a.world) + 3) / 4 * 4;
  const long long lo = a.begin + chunk * a.rank;
  const long long hi = min(a.end, lo + chunk);
  const float scale = a.grad_scale * (a.clip != nullptr && a.phase != 1 ? *a.clip : 1.f);
  float sq = 0.f;
  const long long nvec = (hi > lo) ? (hi - lo) / 4 : 0;
  for (long long v = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; v < nvec;
       v += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long i = lo + v * 4;
    float4 g;
    if (a.phase == 2) {
      g = *reinterpret_cast<const float4*>(ptr.grads[a.rank] + i);
    } else {
      g = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < kMaxWorld; ++r) {
        if (r < a.world) {
          const float4 x = *reinterpret_cast<const float4*>(ptr.grads[r] + i);
          g.x += x.x; g.y += x.y; g.z += x.z; g.w += x.w;
        }
      }
    }
    if (a.phase == 1) {
      *reinterpret_cast<float4*>(ptr.grads[a.rank] + i) = g;
      const float s = a.grad_scale;
      sq += (g.x * g.x + g.y * g.y + g.z * g.z + g.w * g.w) * s * s;
      continue;
    }
    const float gv[4] = {g.x * scale, g.y * scale, g.z * scale, g.w * scale};
    float4 p = *reinterpret_cast<const float4*>(ptr.params[a.rank] + i);
    float pv[4] = {p.x, p.y, p.z, p.w};
    float4 s1 = *reinterpret_cast<const float4*>(a.state1 + i);
    float s1v[4] = {s1.x, s1.y, s1.z, s1.w};
    float s2v[4] = {0.f, 0.f, 0.f, 0.f};
    if (a.optimizer == 0) {
      const float4 s2 = *reinterpret_cast<const float4*>(a.state2 + i);
      s2v[0] = s2.x; s2v[1] = s2.y; s2v[2] = s2.z; s2v[3] = s2.w;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) opt_update(a, pv[k], gv[k], s1v[k], s2v[k]);
    p = make_float4(pv[0], pv[1], pv[2], pv[3]);
    *reinterpret_cast<float4*>(ptr.params[a.rank] + i) = p;
    *reinterpret_cast<float4*>(a.state1 + i) = make_float4(s1v[0], s1v[1], s1v[2], s1v[3]);
    if (a.optimizer == 0) *reinterpret_cast<float4*>(a.state2 + i) = make_float4(s2v[0], s2v[1], s2v[2], s2v[3]);
    __nv_bfloat162 h0 = __floats2bfloat162_rn(pv[0], pv[1]);
    __nv_bfloat162 h1 = __floats2bfloat162_rn(pv[2], pv[3]);
    uint2 hb;
    hb.x = *reinterpret_cast<uint32_t*>(&h0);
    hb.y = *reinterpret_cast<uint32_t*>(&h1);
    const bool bcast_fp32 = i >= a.fp32_from;
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r) {
      if (r < a.world) {
        if (ptr.shadows[r] != nullptr) *reinterpret_cast<uint2*>(ptr.shadows[r] + i) = hb;
        if (bcast_fp32 && r != a.rank) *reinterpret_cast<float4*>(ptr.params[r] + i) = p;
      }
    }
  }
  if (a.phase == 1 && a.sqnorm_out != nullptr) {
    sq = warp_sum(sq);
    if ((threadIdx.x & 31) == 0) atomicAdd(a.sqnorm_out, sq);
  }
}

// ---- NVLS variant: the switch reduces, the switch replicates ----------------
// Per owned element: NVLink ingress of 4 bytes (one reduced fp32 value instead of
// W-1 peer loads) and egress of 2 bytes (one multicast bf16 store instead of W-1
// peer stores); fp32-broadcast elements add a 4-byte multicast store.
__device__ __forceinline__ float4 mc_ld_reduce_f32x4(const float* mc) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
__device__ __forceinline__ void mc_st_f32x4(float* mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void mc_st_b32x2(void* mc, uint32_t a, uint32_t b) {
  asm volatile("multimem.st.relaxed.sys.global.v2.f32 [%0], {%1, %2};" ::"l"(mc), "f"(__uint_as_float(a)),
               "f"(__uint_as_float(b))
               : "memory");
}

// Multicast loads and stores travel through the switch and have long latency: each
// thread keeps kNvlsUnroll reductions in flight before it updates any of them.
constexpr int kNvlsUnroll = 4;

__global__ void __launch_bounds__(256) dense_sync_nvls_kernel(const DenseSyncArgs a) {
  const long long total = a.end - a.begin;
  const long long chunk = ((total / a.world) + 3) / 4 * 4;
  const long long lo = a.begin + chunk * a.rank;
  const long long hi = min(a.end, lo + chunk);
  const float scale = a.grad_scale * (a.clip != nullptr && a.phase != 1 ? *a.clip : 1.f);
  float* grads = a.grads[a.rank];
  float* params = a.params[a.rank];
  float sq = 0.f;
  const long long nvec = (hi > lo) ? (hi - lo) / 4 : 0;
  const long long step = static_cast<long long>(gridDim.x) * blockDim.x * kNvlsUnroll;
  for (long long base = static_cast<long long>(blockIdx.x) * blockDim.x * kNvlsUnroll + threadIdx.x; base < nvec;
       base += step) {
    float4 g[kNvlsUnroll];
#pragma unroll
    for (int u = 0; u < kNvlsUnroll; ++u) {
      const long long v = base + static_cast<long long>(u) * blockDim.x;
      if (v < nvec) {
        const long long i = lo + v * 4;
        g[u] = a.phase == 2 ? *reinterpret_cast<const float4*>(grads + i) : mc_ld_reduce_f32x4(a.mc_grad + i);
      }
    }
#pragma unroll
    for (int u = 0; u < kNvlsUnroll; ++u) {
      const long long v = base + static_cast<long long>(u) * blockDim.x;
      if (v >= nvec) continue;
      const long long i = lo + v * 4;
      if (a.phase == 1) {
        *reinterpret_cast<float4*>(grads + i) = g[u];
        const float s = a.grad_scale;
        sq += (g[u].x * g[u].x + g[u].y * g[u].y + g[u].z * g[u].z + g[u].w * g[u].w) * s * s;
        continue;
      }
      const float gv[4] = {g[u].x * scale, g[u].y * scale, g[u].z * scale, g[u].w * scale};
      float4 p = *reinterpret_cast<const float4*>(params + i);
      float pv[4] = {p.x, p.y, p.z, p.w};
      float4 s1 = *reinterpret_cast<const float4*>(a.state1 + i);
      float s1v[4] = {s1.x, s1.y, s1.z, s1.w};
      float s2v[4] = {0.f, 0.f, 0.f, 0.f};
      if (a.optimizer == 0) {
        const float4 s2 = *reinterpret_cast<const float4*>(a.state2 + i);
        s2v[0] = s2.x; s2v[1] = s2.y; s2v[2] = s2.z; s2v[3] = s2.w;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) opt_update(a, pv[k], gv[k], s1v[k], s2v[k]);
      p = make_float4(pv[0], pv[1], pv[2], pv[3]);
      *reinterpret_cast<float4*>(a.state1 + i) = make_float4(s1v[0], s1v[1], s1v[2], s1v[3]);
      if (a.optimizer == 0) *reinterpret_cast<float4*>(a.state2 + i) = make_float4(s2v[0], s2v[1], s2v[2], s2v[3]);
      if (i >= a.fp32_from) {
        mc_st_f32x4(a.mc_master + i, p);  // every rank's master (this rank's included)
      } else {
        *reinterpret_cast<float4*>(params + i) = p;
      }
      __nv_bfloat162 h0 = __floats2bfloat162_rn(pv[0], pv[1]);
      __nv_bfloat162 h1 = __floats2bfloat162_rn(pv[2], pv[3]);
      mc_st_b32x2(reinterpret_cast<__nv_bfloat16*>(a.mc_shadow) + i, *reinterpret_cast<uint32_t*>(&h0),
                  *reinterpret_cast<uint32_t*>(&h1));
    }
  }
  if (a.phase == 1 && a.sqnorm_out != nullptr) {
    sq = warp_sum(sq);
    if ((threadIdx.x & 31) == 0) atomicAdd(a.sqnorm_out, sq);
  }
}

struct SmallPtrs {
  float* p[kMaxWorld];
};

__global__ void small_allreduce_kernel(SmallPtrs bufs, float* out, int n, int world) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < world; ++r) s += bufs.p[r][i];
    out[i] = s;
  }
}

}  // namespace

static uint64_t g_barrier_limit_ns = 10000000000ull;  // 10 s default

void set_barrier_limit_ns(uint64_t ns) { g_barrier_limit_ns = ns; }

cudaError_t symm_barrier(unsigned* const* signals, unsigned* counter, int rank, int world, int* err,
                         cudaStream_t stream) {
  SigPtrs s{};
  for (int r = 0; r < world && r < kMaxWorld; ++r) s.p[r] = signals[r];
  barrier_kernel<<<1, 32, 0, stream>>>(s, counter, rank, world, err, g_barrier_limit_ns);
  return cudaGetLastError();
}

cudaError_t dense_sync_update(const DenseSyncArgs& a, cudaStream_t stream) {
  if (a.end <= a.begin) return cudaSuccess;
  if (((a.end - a.begin) % (4 * a.world)) != 0 || (a.begin % 4) != 0) return cudaErrorInvalidValue;
  SyncPtrs p{};
  for (int r = 0; r < a.world; ++r) {
    p.grads[r] = a.grads[r];
    p.params[r] = a.params[r];
    p.shadows[r] = reinterpret_cast<__nv_bfloat16*>(a.shadows[r]);
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long per_rank_vec = (a.end - a.begin) / a.world / 4 + 1;
  long long blocks = (per_rank_vec + 255) / 256;
  if (blocks > sms * 4) blocks = sms * 4;
  if (a.max_blocks > 0 && blocks > a.max_blocks) blocks = a.max_blocks;
  if (blocks < 1) blocks = 1;
  if (a.mc_grad != nullptr) {
    if (a.mc_shadow == nullptr || a.mc_master == nullptr || a.params[a.rank] == nullptr || a.grads[a.rank] == nullptr)
      return cudaErrorInvalidValue;
    dense_sync_nvls_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(a);
  } else {
    dense_sync_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(a, p);
  }
  return cudaGetLastError();
}

cudaError_t small_allreduce(float* const* bufs, float* out, int n, int world, cudaStream_t stream) {
  SmallPtrs s{};
  for (int r = 0; r < world && r < kMaxWorld; ++r) s.p[r] = bufs[r];
  small_allreduce_kernel<<<1, 256, 0, stream>>>(s, out, n, world);
  return cudaGetLastError();
}

}  // namespace mdl
