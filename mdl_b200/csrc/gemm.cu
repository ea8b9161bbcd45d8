// Persistent, warp-specialised batched GEMM for sm_100a on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in TMEM, operands staged by TMA).
//
// It serves every GEMM-shaped op of the framework: the RankMixer per-token FFN
// (one group per token), the per-token tokenizer projection, the task-head
// towers and all their backward (dgrad / wgrad) products. The reference runs
// these as cuBLAS strided-batched GEMMs through torch.bmm
// (src/modules/mlp.py:187-207, PerTokenLinear src/modules/mlp.py:30-42).
//
// Roles inside one CTA (576 threads, one CTA per SM):
//   warp 0      : TMA producer (one lane) filling a STAGES-deep smem ring
//   warp 1      : MMA issuer (one lane) + TMEM allocator
//   warps 2..17 : epilogue; warp w reads TMEM lane quarter (w % 4) and one
//                 quarter (64 columns) of the 256-column accumulator
// The accumulator is double-buffered in TMEM (2 x 256 fp32 columns) so the
// epilogue of tile i overlaps the main loop of tile i+1.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "gemm.h"

namespace mdl {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;   // 64 bf16 = 128 bytes = one swizzle row
constexpr int STAGES = 4;
constexpr int A_STAGE_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_STAGE_BYTES = BN * BK * 2;  // 32 KB
constexpr int TMEM_COLS = 2 * BN;           // double-buffered accumulator
constexpr int NUM_EPI_WARPS = 16;                // four warps per TMEM lane quarter
constexpr int NUM_THREADS = 64 + NUM_EPI_WARPS * 32;
constexpr int MN_CHUNK_BYTES = BK * 128;    // one 64-wide MN chunk of BK rows (MN-major)
constexpr int SMEM_BYTES =
    1024 + STAGES * (A_STAGE_BYTES + B_STAGE_BYTES) + (2 * STAGES + 4) * 8 + 16;

struct EpiParams {
  void* out;
  long long ldc, gsC;
  int out_fp32, accumulate;
  __nv_bfloat16* out2;
  const float* bias;
  long long gs_bias;
  const __nv_bfloat16* aux;
  long long ld_aux, gs_aux;
  float* colsum;
  long long gs_colsum;
  int act;
  float alpha;
  int M, N, K, G;
  int* err;
};

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void unpack_bf16x8(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// Reduce v[0..31] across the 32 lanes so that lane l ends with the column-l sum
// in v[0] (recursive halving, 31 shuffles).
__device__ __forceinline__ void warp_transpose_reduce32(float* v, int lane) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = upper ? v[i] : v[i + o];
      const float keep = upper ? v[i + o] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
}

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const EpiParams ep) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * B_STAGE_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (ep.M + BM - 1) / BM;
  const int n_tiles = (ep.N + BN - 1) / BN;
  const int tiles_per_group = m_tiles * n_tiles;
  const int num_tiles = tiles_per_group * ep.G;
  const int k_blocks = (ep.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], NUM_EPI_WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;  // stages filled but possibly not yet consumed
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int g = tile / tiles_per_group;
        const int rem = tile - g * tiles_per_group;
        const int mb = rem / n_tiles;
        const int nb = rem - mb * n_tiles;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, ep.err, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], A_STAGE_BYTES + B_STAGE_BYTES);
          const int k0 = kb * BK;
          uint8_t* a_dst = sA + stage * A_STAGE_BYTES;
          uint8_t* b_dst = sB + stage * B_STAGE_BYTES;
          if (!A_MN) {
            tma_load_3d(a_dst, &tmA, &full[stage], k0, mb * BM, g);
          } else {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c)
              tma_load_3d(a_dst + c * MN_CHUNK_BYTES, &tmA, &full[stage], mb * BM + c * 64, k0, g);
          }
          if (!B_MN) {
            tma_load_3d(b_dst, &tmB, &full[stage], k0, nb * BN, g);
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_3d(b_dst + c * MN_CHUNK_BYTES, &tmB, &full[stage], nb * BN + c * 64, k0, g);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Drain copies still in flight into this CTA's smem before exiting.
        int s = stage, p = phase;
        for (int i = 0; i < STAGES && i < issued; ++i) {
          s = (s + STAGES - 1) % STAGES;
          if (s == STAGES - 1) p ^= 1;
          mbar_wait(&full[s], p, nullptr, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN, A_MN, B_MN);
      const uint32_t a_base = smem_u32(sA);
      const uint32_t b_base = smem_u32(sB);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, ep.err, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, ep.err, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_stage = a_base + stage * A_STAGE_BYTES;
          const uint32_t b_stage = b_base + stage * B_STAGE_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // K-major: advance 16 elements = 32 bytes inside the 128-byte swizzle row.
            // MN-major: advance 16 K-rows = two 1024-byte swizzle atoms.
            const uint64_t adesc = A_MN ? make_smem_desc(a_stage + kk * 2048, MN_CHUNK_BYTES, 1024)
                                        : make_smem_desc(a_stage + kk * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? make_smem_desc(b_stage + kk * 2048, MN_CHUNK_BYTES, 1024)
                                        : make_smem_desc(b_stage + kk * 32, 16, 1024);
            tc_mma_bf16(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;            // TMEM lane quarter this warp may read
    const int cgroup = (warp - 2) / 4;       // which 64-column group of the tile
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      if (!mbar_wait(&tfull[acc], acc_phase, ep.err, abort_flag)) break;
      tc_fence_after();
      const int g = tile / tiles_per_group;
      const int rem = tile - g * tiles_per_group;
      const int mb = rem / n_tiles;
      const int nb = rem - mb * n_tiles;
      const int row = mb * BM + quarter * 32 + lane;
      const bool row_ok = row < ep.M;
      for (int c0 = cgroup * (BN / 4); c0 < (cgroup + 1) * (BN / 4); c0 += 32) {
        const int col0 = nb * BN + c0;
        if (col0 >= ep.N) break;  // warp-uniform
        float v[32];
        tmem_ld_32x32b_x32(
            tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN + c0),
            v);
        const bool full_chunk = col0 + 32 <= ep.N;
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= ep.alpha;
        if (ep.bias != nullptr) {
          const float* bp = ep.bias + g * ep.gs_bias + col0;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (full_chunk || col0 + i < ep.N) v[i] += __ldg(bp + i);
        }
        if (ep.act == GEMM_ACT_DGELU || ep.act == GEMM_ACT_DRELU) {
          if (row_ok) {
            const __nv_bfloat16* ap = ep.aux + g * ep.gs_aux + static_cast<long long>(row) * ep.ld_aux + col0;
            float a[32];
            if (full_chunk) {
              const uint4* ap4 = reinterpret_cast<const uint4*>(ap);
#pragma unroll
              for (int q = 0; q < 4; ++q) unpack_bf16x8(__ldg(ap4 + q), a + 8 * q);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) a[i] = (col0 + i < ep.N) ? __bfloat162float(ap[i]) : 0.f;
            }
            if (ep.act == GEMM_ACT_DGELU) {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] *= gelu_erf_grad(a[i]);
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = a[i] > 0.f ? v[i] : 0.f;
            }
          }
        }
        if (ep.act == GEMM_ACT_RELU) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.f);
        }
        if (row_ok) {
          const long long off = g * ep.gsC + static_cast<long long>(row) * ep.ldc + col0;
          if (ep.out_fp32) {
            float* op = reinterpret_cast<float*>(ep.out) + off;
            if (full_chunk) {
              float4* op4 = reinterpret_cast<float4*>(op);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                float4 t = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                if (ep.accumulate) {
                  const float4 o = op4[q];
                  t.x += o.x; t.y += o.y; t.z += o.z; t.w += o.w;
                }
                op4[q] = t;
              }
            } else {
              for (int i = 0; i < 32; ++i)
                if (col0 + i < ep.N) op[i] = ep.accumulate ? op[i] + v[i] : v[i];
            }
          } else {
            __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(ep.out) + off;
            __nv_bfloat16* op2 = ep.out2 != nullptr ? ep.out2 + off : nullptr;
            if (full_chunk) {
              uint4* o4 = reinterpret_cast<uint4*>(op);
              if (ep.accumulate) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  float old[8];
                  unpack_bf16x8(o4[q], old);
#pragma unroll
                  for (int e = 0; e < 8; ++e) v[8 * q + e] += old[e];
                }
              }
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                uint4 t;
                t.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
                t.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
                t.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
                t.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
                o4[q] = t;
              }
              if (ep.act == GEMM_ACT_GELU) {
                uint4* o24 = reinterpret_cast<uint4*>(op2);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  uint4 t;
                  t.x = pack_bf16x2(gelu_erf(v[8 * q + 0]), gelu_erf(v[8 * q + 1]));
                  t.y = pack_bf16x2(gelu_erf(v[8 * q + 2]), gelu_erf(v[8 * q + 3]));
                  t.z = pack_bf16x2(gelu_erf(v[8 * q + 4]), gelu_erf(v[8 * q + 5]));
                  t.w = pack_bf16x2(gelu_erf(v[8 * q + 6]), gelu_erf(v[8 * q + 7]));
                  o24[q] = t;
                }
              }
            } else {
              for (int i = 0; i < 32; ++i) {
                if (col0 + i < ep.N) {
                  if (ep.accumulate) v[i] += __bfloat162float(op[i]);
                  op[i] = __float2bfloat16_rn(v[i]);
                  if (ep.act == GEMM_ACT_GELU) op2[i] = __float2bfloat16_rn(gelu_erf(v[i]));
                }
              }
            }
          }
        }
        if (ep.colsum != nullptr) {
          // Column sums of what this epilogue produced (gelu output excluded).
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (!row_ok) v[i] = 0.f;
          warp_transpose_reduce32(v, lane);
          if (col0 + lane < ep.N) atomicAdd(ep.colsum + g * ep.gs_colsum + col0 + lane, v[0]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3D bf16 map: dims {inner, outer, G}; box {box_inner(=64), box_outer, 1}; 128-byte swizzle.
bool encode_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t groups,
                uint64_t outer_stride_elems, uint64_t group_stride_elems, uint32_t box_outer) {
  auto fn = get_encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {inner, outer, groups};
  uint64_t gstride = group_stride_elems * 2;
  if (groups <= 1) gstride = ((outer * outer_stride_elems * 2) + 15) & ~uint64_t(15);
  cuuint64_t strides[2] = {outer_stride_elems * 2, gstride};
  cuuint32_t box[3] = {64, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <bool A_MN, bool B_MN>
cudaError_t launch(const CUtensorMap& ta, const CUtensorMap& tb, const EpiParams& ep, int grid,
                   cudaStream_t stream) {
  auto kern = gemm_tcgen05_kernel<A_MN, B_MN>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  kern<<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(ta, tb, ep);
  return cudaGetLastError();
}

}  // namespace

cudaError_t gemm_bf16_tcgen05(const GemmArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0 || a.G <= 0) return cudaSuccess;
  if ((a.lda % 8) || (a.ldb % 8) || (a.G > 1 && ((a.gsA % 8) || (a.gsB % 8))) ||
      (reinterpret_cast<uintptr_t>(a.A) & 15) || (reinterpret_cast<uintptr_t>(a.B) & 15))
    return cudaErrorInvalidValue;
  if (!a.out_fp32 && (a.ldc % 8)) return cudaErrorInvalidValue;
  if (a.out_fp32 && (a.ldc % 4)) return cudaErrorInvalidValue;
  CUtensorMap ta, tb;
  bool ok;
  if (!a.a_mn_major)
    ok = encode_map(&ta, a.A, a.K, a.M, a.G, a.lda, a.gsA, BM);
  else
    ok = encode_map(&ta, a.A, a.M, a.K, a.G, a.lda, a.gsA, BK);
  if (!ok) return cudaErrorInvalidValue;
  if (!a.b_mn_major)
    ok = encode_map(&tb, a.B, a.K, a.N, a.G, a.ldb, a.gsB, BN);
  else
    ok = encode_map(&tb, a.B, a.N, a.K, a.G, a.ldb, a.gsB, BK);
  if (!ok) return cudaErrorInvalidValue;

  EpiParams ep;
  ep.out = a.out;
  ep.ldc = a.ldc;
  ep.gsC = a.gsC;
  ep.out_fp32 = a.out_fp32 ? 1 : 0;
  ep.accumulate = a.accumulate ? 1 : 0;
  ep.out2 = reinterpret_cast<__nv_bfloat16*>(a.out2);
  ep.bias = a.bias;
  ep.gs_bias = a.gs_bias;
  ep.aux = reinterpret_cast<const __nv_bfloat16*>(a.aux);
  ep.ld_aux = a.ld_aux;
  ep.gs_aux = a.gs_aux;
  ep.colsum = a.colsum;
  ep.gs_colsum = a.gs_colsum;
  ep.act = a.act;
  ep.alpha = a.alpha;
  ep.M = a.M;
  ep.N = a.N;
  ep.K = a.K;
  ep.G = a.G;
  ep.err = a.err;
  const long long tiles =
      static_cast<long long>((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN) * static_cast<long long>(a.G);
  int grid = num_sms();
  if (a.max_ctas > 0 && a.max_ctas < grid) grid = a.max_ctas;
  if (tiles < grid) grid = static_cast<int>(tiles);
  if (a.a_mn_major) {
    return a.b_mn_major ? launch<true, true>(ta, tb, ep, grid, stream)
                        : launch<true, false>(ta, tb, ep, grid, stream);
  }
  return a.b_mn_major ? launch<false, true>(ta, tb, ep, grid, stream)
                      : launch<false, false>(ta, tb, ep, grid, stream);
}

}  // namespace mdl
