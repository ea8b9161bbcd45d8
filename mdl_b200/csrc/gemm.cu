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
//
// Epilogue data path: tcgen05.ld gives each lane one ROW of a 32x32 chunk, so
// direct stores would touch 32 rows per instruction. Each warp instead stages
// the chunk in shared memory 16 columns at a time (fp32, 64-byte rows whose four
// 16-byte slots are XOR-swizzled by row pair: conflict-free writes by row and
// reads by column group) and writes it back eight rows x 32 bytes per
// instruction; the aux operand of the activation-derivative epilogues is read
// the same way. The 32 KB staging buffer leaves room for a 4-stage (single CTA)
// or 6-stage (CTA pair) operand ring.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "gemm.h"

// Pipeline wait counters for tuning builds (-DMDL_GEMM_STATS): clock cycles the producer
// waits for free stages, the MMA issuer for loaded stages and free accumulators, and one
// epilogue lane for finished accumulators, summed over CTAs. Off in the library build.
#ifdef MDL_GEMM_STATS
__device__ unsigned long long g_gemm_stats[8];
#define GSTAT_DECL(v) long long v = 0
#define GSTAT_WAIT(v, expr) \
  ([&]() { const long long t0_ = clock64(); const bool r_ = (expr); v += clock64() - t0_; return r_; }())
#define GSTAT_FLUSH(i, v) atomicAdd(&g_gemm_stats[i], static_cast<unsigned long long>(v))
#else
#define GSTAT_DECL(v)
#define GSTAT_WAIT(v, expr) (expr)
#define GSTAT_FLUSH(i, v)
#endif

namespace mdl {
namespace {

void bind_context_once() {
  thread_local bool bound = false;
  if (!bound) {
    cudaFree(nullptr);  // makes the device's primary context current on this thread
    bound = true;
  }
}

constexpr int BM = 128;  // accumulator rows per CTA (TMEM lanes)
constexpr int BN = 256;
constexpr int BK = 64;   // 64 bf16 = 128 bytes = one swizzle row
constexpr int A_STAGE_BYTES = BM * BK * 2;  // 16 KB
constexpr int TMEM_COLS = 2 * BN;           // double-buffered accumulator
constexpr int NUM_EPI_WARPS = 16;                // four warps per TMEM lane quarter
constexpr int NUM_THREADS = 64 + NUM_EPI_WARPS * 32;
constexpr int MN_CHUNK_BYTES = BK * 128;    // one 64-wide MN chunk of BK rows (MN-major)
constexpr int EPI_PITCH = 16;               // floats per staged row (16 columns, float4 slots swizzled)
constexpr int EPI_WARP_FLOATS = 32 * EPI_PITCH;
constexpr int EPI_BYTES = NUM_EPI_WARPS * EPI_WARP_FLOATS * 4;  // 32 KB

// Single CTA: a 128 x 256 tile per CTA, all of B's 256 rows staged per k-block.
// CTA pair (cta_group::2, cluster of two): a 256 x 256 tile per pair; each CTA stages
// 128 rows of A and 128 rows of B per k-block (32 KB instead of 48 KB per 128 x 256 of
// output), which leaves room for a fourth pipeline stage.
// Epilogues that read global memory per element (aux operands) or compute GELU keep
// a shallower ring: the shared-memory carve-out then leaves more of the SM's unified
// L1 for their loads, and their time is set by the epilogue, not by operand latency.
template <bool PAIR, bool HEAVY_EPI = false>
struct Cfg {
  static constexpr int TILE_M = PAIR ? 2 * BM : BM;
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;
  static constexpr int B_STAGE_BYTES = B_ROWS * BK * 2;
  static constexpr int STAGES = HEAVY_EPI ? (PAIR ? 4 : 3) : (PAIR ? 6 : 4);
  static constexpr int SMEM_BYTES =
      1024 + STAGES * (A_STAGE_BYTES + B_STAGE_BYTES) + EPI_BYTES + (2 * STAGES + 4) * 8 + 16;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

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
  int KG;                  // K-range groups (G == 1 when KG > 1)
  int splits;              // K slices per output tile (> 1: fp32 output reduced with atomics)
  int kb_per_split;
  int a_shared, b_shared;  // operand shared by every group (batch stride 0)
  int* err;
};

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Epilogue kinds (compile-time, so each instantiation carries only its own path).
constexpr int EPI_PLAIN = 0;     // bf16 out, optional bias / ReLU / column sums
constexpr int EPI_GELU = 1;      // bf16 pre-activation (or GELU'(pre)) + bf16 GELU(pre)
constexpr int EPI_AUX = 2;       // bf16 out scaled by GELU'(aux), ReLU'(aux) or aux, or plus aux; optional column sums
constexpr int EPI_ACC_BF16 = 3;  // bf16 out += result
constexpr int EPI_F32 = 4;       // fp32 out (= or +=)

template <bool A_MN, bool B_MN, int EPI, bool PAIR>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const EpiParams ep) {
  using C = Cfg<PAIR, EPI == EPI_GELU || EPI == EPI_AUX>;
  constexpr int STAGES = C::STAGES;
  constexpr int B_STAGE_BYTES = C::B_STAGE_BYTES;
  constexpr int TILE_M = C::TILE_M;
  constexpr int B_ROWS = C::B_ROWS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
  float* sEpi = reinterpret_cast<float*>(sB + STAGES * B_STAGE_BYTES);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sEpi + NUM_EPI_WARPS * EPI_WARP_FLOATS);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // pair rank (0 = leader: issues the MMAs, owns the full / tempty barriers); units are
  // distributed over pairs
  const uint32_t cr = PAIR ? cluster_ctarank() : 0u;
  const int unit0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int unit_step = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const int m_tiles = (ep.M + TILE_M - 1) / TILE_M;
  const int n_tiles = (ep.N + BN - 1) / BN;
  const int tiles_per_group = m_tiles * n_tiles;
  const int num_tiles = tiles_per_group * ep.G;
  const int num_units = num_tiles * ep.splits;  // work unit = (output tile, K slice)
  const int kb_per_range = (ep.K + BK - 1) / BK;
  const int k_blocks = kb_per_range * ep.KG;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], PAIR ? 2 * NUM_EPI_WARPS : NUM_EPI_WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR) {
    cluster_sync();  // both CTAs' barriers initialised before any cross-CTA signal
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // the leader's full / tempty barriers as cluster addresses (TMA completion, epilogue release)
  const uint32_t full_lead = PAIR ? mapa_shared(smem_u32(full), 0) : smem_u32(full);
  const uint32_t tempty_lead = PAIR ? mapa_shared(smem_u32(tempty), 0) : smem_u32(tempty);

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;  // stages filled but possibly not yet consumed
      bool ok = true;
      GSTAT_DECL(w_empty);
      for (int unit = unit0; unit < num_units && ok; unit += unit_step) {
        const int tile = unit / ep.splits;
        const int kb0 = (unit - tile * ep.splits) * ep.kb_per_split;
        const int kb1 = min(k_blocks, kb0 + ep.kb_per_split);
        const int g = tile / tiles_per_group;
        const int rem = tile - g * tiles_per_group;
        const int mb = rem / n_tiles;
        const int nb = rem - mb * n_tiles;
        const int a_row0 = mb * TILE_M + static_cast<int>(cr) * BM;     // this CTA's A rows
        const int b_row0 = nb * BN + static_cast<int>(cr) * B_ROWS;     // this CTA's B rows
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!GSTAT_WAIT(w_empty, mbar_wait(&empty[stage], phase ^ 1u, ep.err, abort_flag))) {
            ok = false;
            break;
          }
          // the leader expects the bytes of both CTAs' copies on its own barrier
          if (cr == 0) mbar_arrive_expect_tx(&full[stage], (PAIR ? 2 : 1) * (A_STAGE_BYTES + B_STAGE_BYTES));
          // third map coordinate: the batch group, or the K range when KG > 1
          const int kr = ep.KG > 1 ? kb / kb_per_range : 0;
          const int k0 = (kb - kr * kb_per_range) * BK;
          const int za = ep.KG > 1 ? kr : (ep.a_shared ? 0 : g);
          const int zb = ep.KG > 1 ? kr : (ep.b_shared ? 0 : g);
          uint8_t* a_dst = sA + stage * A_STAGE_BYTES;
          uint8_t* b_dst = sB + stage * B_STAGE_BYTES;
          const uint32_t fb = full_lead + static_cast<uint32_t>(stage) * 8u;
          auto load = [&](uint8_t* dst, const CUtensorMap* map, int c0, int c1, int c2) {
            if constexpr (PAIR) {
              tma_load_3d_pair(dst, map, fb, c0, c1, c2);
            } else {
              tma_load_3d(dst, map, &full[stage], c0, c1, c2);
            }
          };
          if (!A_MN) {
            load(a_dst, &tmA, k0, a_row0, za);
          } else {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c) load(a_dst + c * MN_CHUNK_BYTES, &tmA, a_row0 + c * 64, k0, za);
          }
          if (!B_MN) {
            load(b_dst, &tmB, k0, b_row0, zb);
          } else {
#pragma unroll
            for (int c = 0; c < B_ROWS / 64; ++c) load(b_dst + c * MN_CHUNK_BYTES, &tmB, b_row0 + c * 64, k0, zb);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Drain copies still in flight into this CTA's smem before exiting (their bytes
        // count on the leader's barriers, so a pair member waits a fixed 2 ms instead).
        if (PAIR && cr != 0) {
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 2000000ull) {
          }
        } else {
          int s = stage, p = phase;
          for (int i = 0; i < STAGES && i < issued; ++i) {
            s = (s + STAGES - 1) % STAGES;
            if (s == STAGES - 1) p ^= 1;
            mbar_wait(&full[s], p, nullptr, nullptr);
          }
        }
      }
      GSTAT_FLUSH(0, w_empty);
    }
  } else if (warp == 1) {
    if (lane == 0 && cr == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(TILE_M, BN, A_MN, B_MN);
      const uint32_t a_base = smem_u32(sA);
      const uint32_t b_base = smem_u32(sB);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      GSTAT_DECL(w_full);
      GSTAT_DECL(w_tempty);
#ifdef MDL_GEMM_STATS
      const long long t_start = clock64();
#endif
      for (int unit = unit0; unit < num_units && ok; unit += unit_step) {
        const int tile = unit / ep.splits;
        const int kb0 = (unit - tile * ep.splits) * ep.kb_per_split;
        const int kb1 = min(k_blocks, kb0 + ep.kb_per_split);
        if (!GSTAT_WAIT(w_tempty, mbar_wait(&tempty[acc], acc_phase ^ 1u, ep.err, abort_flag))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!GSTAT_WAIT(w_full, mbar_wait(&full[stage], phase, ep.err, abort_flag))) {
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
            if constexpr (PAIR) {
              tc_mma_bf16_pair(d_tmem, adesc, bdesc, idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
            } else {
              tc_mma_bf16(d_tmem, adesc, bdesc, idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
            }
          }
          if constexpr (PAIR) {
            tc_commit_pair(&empty[stage]);  // frees the stage in both CTAs
          } else {
            tc_commit(&empty[stage]);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (PAIR) {
          tc_commit_pair(&tfull[acc]);  // both CTAs' epilogues may read their halves
        } else {
          tc_commit(&tfull[acc]);
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      GSTAT_FLUSH(1, w_full);
      GSTAT_FLUSH(2, w_tempty);
#ifdef MDL_GEMM_STATS
      GSTAT_FLUSH(3, clock64() - t_start);
      GSTAT_FLUSH(5, 1);
#endif
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Per 32x32 chunk: tcgen05.ld (lane = row) -> stage in smem -> write-back where
    // lane l owns columns 4*(l%8)..+3 of rows it*4 + l/8 (it = 0..7): bias,
    // activation, accumulate and column sums act on 4 consecutive columns, and
    // every global access is a coalesced 4-row x 128/64-byte pattern.
    constexpr bool kF32 = EPI == EPI_F32;
    constexpr bool kGelu = EPI == EPI_GELU;
    constexpr bool kAux = EPI == EPI_AUX;
    const bool accumulate = EPI == EPI_ACC_BF16 || (kF32 && ep.accumulate);
    const bool relu = EPI == EPI_PLAIN && ep.act == GEMM_ACT_RELU;
    const bool affine = ep.alpha != 1.f || ep.bias != nullptr;
    const bool store_grad = kGelu && ep.act == GEMM_ACT_GELU_GRAD;
    const int quarter = warp & 3;            // TMEM lane quarter this warp may read
    const int cgroup = (warp - 2) / 4;       // which 64-column group of the tile
    float* stg = sEpi + (warp - 2) * EPI_WARP_FLOATS;
    const int q4 = lane & 3;                 // 4-column group in a 16-column half (write-back)
    const int rq = lane >> 2;                // row within each 8-row step (write-back)
    int acc = 0;
    uint32_t acc_phase = 0;
    const bool atomic_out = ep.splits > 1;  // K slices of one tile add into the fp32 output
    GSTAT_DECL(w_tfull);
    for (int unit = unit0; unit < num_units; unit += unit_step) {
      const int tile = unit / ep.splits;
      // warp-uniform outcome: the tcgen05.ld below must be executed by the whole warp
      if (!__all_sync(0xffffffffu, GSTAT_WAIT(w_tfull, mbar_wait(&tfull[acc], acc_phase, ep.err, abort_flag)))) break;
      tc_fence_after();
      const int g = tile / tiles_per_group;
      const int rem = tile - g * tiles_per_group;
      const int mb = rem / n_tiles;
      const int nb = rem - mb * n_tiles;
      const int row0 = mb * TILE_M + static_cast<int>(cr) * BM + quarter * 32;  // this warp's 32-row slab
      for (int c0 = cgroup * (BN / 4); c0 < (cgroup + 1) * (BN / 4); c0 += 32) {
        const int col0 = nb * BN + c0;
        if (col0 >= ep.N) break;  // warp-uniform
        constexpr bool need_aux = kAux;
        // Steps s = 0..7 cover the 32 x 32 chunk: half h = s / 4 (16 columns), rows
        // it * 8 + rq (it = s % 4); lane owns columns 4 * q4 .. +3 of the half.
        auto gcol_of = [&](int h) { return col0 + h * 16 + q4 * 4; };
        // Global reads of the chunk (aux or old output) run PF steps ahead: steps 0..PF-1
        // are requested before the TMEM load, step s+PF as soon as step s is consumed.
        const bool need_read = need_aux || (accumulate && !atomic_out);
        constexpr int PF = kF32 ? 2 : 4;  // steps in flight (fp32 rows need 4 registers each)
        uint4 pf[PF];
        auto prefetch = [&](int st) -> uint4 {
          uint4 r4 = make_uint4(0u, 0u, 0u, 0u);
          const int grow = row0 + (st & 3) * 8 + rq;
          const int gc = gcol_of(st >> 2);
          if (grow < ep.M && gc + 4 <= ep.N) {
            if constexpr (need_aux) {
              const uint2 a2 = __ldg(reinterpret_cast<const uint2*>(ep.aux + g * ep.gs_aux +
                                                                   static_cast<long long>(grow) * ep.ld_aux + gc));
              r4 = make_uint4(a2.x, a2.y, 0u, 0u);
            } else if (accumulate) {
              const long long off = g * ep.gsC + static_cast<long long>(grow) * ep.ldc + gc;
              if (kF32) {
                r4 = *reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(ep.out) + off);
              } else {
                const uint2 o = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(ep.out) + off);
                r4 = make_uint4(o.x, o.y, 0u, 0u);
              }
            }
          }
          return r4;
        };
#pragma unroll
        for (int st = 0; st < PF; ++st) pf[st] = need_read ? prefetch(st) : make_uint4(0u, 0u, 0u, 0u);
        float4 bias4[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          bias4[h] = make_float4(0.f, 0.f, 0.f, 0.f);
          const int gc = gcol_of(h);
          const int nc = gc + 4 <= ep.N ? 4 : max(0, ep.N - gc);
          if (ep.bias != nullptr && nc > 0) {
            const float* bp = ep.bias + g * ep.gs_bias + gc;
            if (nc == 4 && ((reinterpret_cast<uintptr_t>(bp) & 15) == 0)) {
              bias4[h] = __ldg(reinterpret_cast<const float4*>(bp));
            } else {
              float b4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
              for (int e = 0; e < 4; ++e)
                if (e < nc) b4[e] = __ldg(bp + e);
              bias4[h] = make_float4(b4[0], b4[1], b4[2], b4[3]);
            }
          }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          {
            // stage this half: lane = row, four float4 slots swizzled by row pair (conflict-free
            // 16-byte writes by row and reads by column group)
            float v[16];
            tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc * BN + c0 + h * 16),
                               v);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              reinterpret_cast<float4*>(stg + lane * EPI_PITCH)[k ^ ((lane >> 1) & 3)] =
                  make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
          }
          __syncwarp();
          const int gcol = gcol_of(h);
          const bool col_vec = gcol + 4 <= ep.N;
          const int ncols = col_vec ? 4 : max(0, ep.N - gcol);
          float csum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            const int st = h * 4 + it;
            const int r = it * 8 + rq;
            const int grow = row0 + r;
            const uint4 cur = pf[st % PF];
            if (st + PF < 8 && need_read) pf[st % PF] = prefetch(st + PF);
            if (grow >= ep.M || ncols == 0) continue;
            const float4 s4 = reinterpret_cast<const float4*>(stg + r * EPI_PITCH)[q4 ^ ((r >> 1) & 3)];
            float t[4] = {s4.x, s4.y, s4.z, s4.w};
            if (affine) {
              t[0] = fmaf(t[0], ep.alpha, bias4[h].x);
              t[1] = fmaf(t[1], ep.alpha, bias4[h].y);
              t[2] = fmaf(t[2], ep.alpha, bias4[h].z);
              t[3] = fmaf(t[3], ep.alpha, bias4[h].w);
            }
            const long long off = g * ep.gsC + static_cast<long long>(grow) * ep.ldc + gcol;
            if constexpr (need_aux) {
              uint32_t abits[4] = {cur.x & 0xFFFFu, cur.x >> 16, cur.y & 0xFFFFu, cur.y >> 16};
              if (!col_vec) {
                const __nv_bfloat16* ap = ep.aux + g * ep.gs_aux + static_cast<long long>(grow) * ep.ld_aux + gcol;
#pragma unroll
                for (int e = 0; e < 4; ++e) abits[e] = e < ncols ? __bfloat16_as_ushort(ap[e]) : 0u;
              }
              if (ep.act == GEMM_ACT_DMUL) {
#pragma unroll
                for (int e = 0; e < 4; ++e) t[e] *= bf16_bits_to_float(abits[e]);
              } else if (ep.act == GEMM_ACT_ADD) {
#pragma unroll
                for (int e = 0; e < 4; ++e) t[e] += bf16_bits_to_float(abits[e]);
              } else if (ep.act == GEMM_ACT_DGELU) {
#pragma unroll
                for (int e = 0; e < 4; ++e) t[e] *= gelu_grad_fast(bf16_bits_to_float(abits[e]));
              } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) t[e] = bf16_bits_to_float(abits[e]) > 0.f ? t[e] : 0.f;
              }
            } else if (relu) {
#pragma unroll
              for (int e = 0; e < 4; ++e) t[e] = fmaxf(t[e], 0.f);
            }
            if (ep.colsum != nullptr) {  // column sums of the product (before any accumulate)
#pragma unroll
              for (int e = 0; e < 4; ++e) csum[e] += t[e];
            }
            if (kF32 && atomic_out) {
              float* op = reinterpret_cast<float*>(ep.out) + off;
              if (col_vec) {
                asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(op), "f"(t[0]), "f"(t[1]),
                             "f"(t[2]), "f"(t[3])
                             : "memory");
              } else {
  #pragma unroll
                for (int e = 0; e < 4; ++e)
                  if (e < ncols) atomicAdd(op + e, t[e]);
              }
            } else if (kF32) {
              float* op = reinterpret_cast<float*>(ep.out) + off;
              if (col_vec) {
                float4 o4 = make_float4(t[0], t[1], t[2], t[3]);
                if (accumulate) {
                  const uint4 o = need_aux ? *reinterpret_cast<const uint4*>(op) : cur;
                  o4.x += __uint_as_float(o.x);
                  o4.y += __uint_as_float(o.y);
                  o4.z += __uint_as_float(o.z);
                  o4.w += __uint_as_float(o.w);
                }
                *reinterpret_cast<float4*>(op) = o4;
              } else {
  #pragma unroll
                for (int e = 0; e < 4; ++e)
                  if (e < ncols) op[e] = accumulate ? op[e] + t[e] : t[e];
              }
            } else {
              __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(ep.out) + off;
              if (accumulate) {
                if (col_vec) {
                  const uint2 o = need_aux ? *reinterpret_cast<const uint2*>(op) : make_uint2(cur.x, cur.y);
                  t[0] += bf16_bits_to_float(o.x & 0xFFFFu);
                  t[1] += bf16_bits_to_float(o.x >> 16);
                  t[2] += bf16_bits_to_float(o.y & 0xFFFFu);
                  t[3] += bf16_bits_to_float(o.y >> 16);
                } else {
  #pragma unroll
                  for (int e = 0; e < 4; ++e)
                    if (e < ncols) t[e] += __bfloat162float(op[e]);
                }
              }
              const uint32_t p01 = pack_bf16x2(t[0], t[1]), p23 = pack_bf16x2(t[2], t[3]);
              if constexpr (kGelu) {
                // GELU (and optionally GELU') of the bf16 pre-activation
                const float x[4] = {bf16_bits_to_float(p01 & 0xFFFFu), bf16_bits_to_float(p01 >> 16),
                                    bf16_bits_to_float(p23 & 0xFFFFu), bf16_bits_to_float(p23 >> 16)};
                float a[4], d[4];
  #pragma unroll
                for (int e = 0; e < 4; ++e) gelu_and_grad_fast(x[e], a[e], d[e], store_grad);
                const uint32_t o01 = store_grad ? pack_bf16x2(d[0], d[1]) : p01;
                const uint32_t o23 = store_grad ? pack_bf16x2(d[2], d[3]) : p23;
                if (col_vec) {
                  *reinterpret_cast<uint2*>(op) = make_uint2(o01, o23);
                } else {
                  const float ov[4] = {store_grad ? d[0] : t[0], store_grad ? d[1] : t[1], store_grad ? d[2] : t[2],
                                       store_grad ? d[3] : t[3]};
  #pragma unroll
                  for (int e = 0; e < 4; ++e)
                    if (e < ncols) op[e] = __float2bfloat16_rn(ov[e]);
                }
                const float a0 = a[0], a1 = a[1], a2 = a[2], a3 = a[3];
                if (col_vec) {
                  *reinterpret_cast<uint2*>(ep.out2 + off) = make_uint2(pack_bf16x2(a0, a1), pack_bf16x2(a2, a3));
                } else {
                  const float av[4] = {a0, a1, a2, a3};
  #pragma unroll
                  for (int e = 0; e < 4; ++e)
                    if (e < ncols) ep.out2[off + e] = __float2bfloat16_rn(av[e]);
                }
              } else {
                if (col_vec) {
                  *reinterpret_cast<uint2*>(op) = make_uint2(p01, p23);
                } else {
  #pragma unroll
                  for (int e = 0; e < 4; ++e)
                    if (e < ncols) op[e] = __float2bfloat16_rn(t[e]);
                }
              }
            }
          }
          if (ep.colsum != nullptr) {
            // lanes q4, q4+4, ..., q4+28 hold the same four columns: reduce, then lanes 0..3 add
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              csum[e] += __shfl_xor_sync(0xffffffffu, csum[e], 4);
              csum[e] += __shfl_xor_sync(0xffffffffu, csum[e], 8);
              csum[e] += __shfl_xor_sync(0xffffffffu, csum[e], 16);
            }
            if (rq == 0) {
              float* cp = ep.colsum + g * ep.gs_colsum + gcol;
#pragma unroll
              for (int e = 0; e < 4; ++e)
                if (e < ncols) atomicAdd(cp + e, csum[e]);
            }
          }
          __syncwarp();  // the staging buffer is rewritten by the next half / chunk
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) {
          mbar_arrive_cluster(tempty_lead + static_cast<uint32_t>(acc) * 8u);  // the leader's barrier
        } else {
          mbar_arrive(&tempty[acc]);
        }
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
#ifdef MDL_GEMM_STATS
    if (warp == 2 && lane == 0) GSTAT_FLUSH(4, w_tfull);
#endif
  }
  if constexpr (PAIR) {
    tc_fence_before();
    cluster_sync();  // no CTA leaves while its partner still reads its smem or signals its barriers
  } else {
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) {
      tmem_dealloc_pair(tmem_base, TMEM_COLS);
    } else {
      tmem_dealloc(tmem_base, TMEM_COLS);
    }
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
  // The encoder is a driver call: it needs this thread's context current (an
  // autograd worker thread may not have made any runtime call yet).
  bind_context_once();
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

template <bool A_MN, bool B_MN, int EPI, bool PAIR>
cudaError_t launch_kind(const CUtensorMap& ta, const CUtensorMap& tb, const EpiParams& ep, int grid,
                        cudaStream_t stream) {
  auto kern = gemm_tcgen05_kernel<A_MN, B_MN, EPI, PAIR>;
  constexpr int smem = Cfg<PAIR, EPI == EPI_GELU || EPI == EPI_AUX>::SMEM_BYTES;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  if constexpr (PAIR) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // A persistent grid must be co-resident: clusters beyond what the GPCs can hold at
    // once would only start after the others finish.
    static int max_clusters = 0;
    if (max_clusters == 0) {
      cfg.gridDim = dim3(static_cast<unsigned>(2 * (num_sms() / 2)), 1, 1);
      int n = 0;
      cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
      if (e != cudaSuccess || n <= 0) return e != cudaSuccess ? e : cudaErrorInvalidConfiguration;
      max_clusters = n;
    }
    if (grid > 2 * max_clusters) grid = 2 * max_clusters;
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    return cudaLaunchKernelEx(&cfg, kern, ta, tb, ep);
  } else {
    kern<<<grid, NUM_THREADS, smem, stream>>>(ta, tb, ep);
    return cudaGetLastError();
  }
}

template <bool A_MN, bool B_MN, bool PAIR>
cudaError_t launch(const CUtensorMap& ta, const CUtensorMap& tb, const EpiParams& ep, int epi, int grid,
                   cudaStream_t stream) {
  switch (epi) {
    case EPI_PLAIN: return launch_kind<A_MN, B_MN, EPI_PLAIN, PAIR>(ta, tb, ep, grid, stream);
    case EPI_GELU: return launch_kind<A_MN, B_MN, EPI_GELU, PAIR>(ta, tb, ep, grid, stream);
    case EPI_AUX: return launch_kind<A_MN, B_MN, EPI_AUX, PAIR>(ta, tb, ep, grid, stream);
    case EPI_ACC_BF16: return launch_kind<A_MN, B_MN, EPI_ACC_BF16, PAIR>(ta, tb, ep, grid, stream);
    default: return launch_kind<A_MN, B_MN, EPI_F32, PAIR>(ta, tb, ep, grid, stream);
  }
}

template <bool PAIR>
cudaError_t launch_any(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const EpiParams& ep,
                       int epi, int grid, cudaStream_t stream) {
  if (a_mn) {
    return b_mn ? launch<true, true, PAIR>(ta, tb, ep, epi, grid, stream)
                : launch<true, false, PAIR>(ta, tb, ep, epi, grid, stream);
  }
  return b_mn ? launch<false, true, PAIR>(ta, tb, ep, epi, grid, stream)
              : launch<false, false, PAIR>(ta, tb, ep, epi, grid, stream);
}

// CTA pairs for GEMMs with enough 256 x 256 tiles to fill the GPU (MDL_B200_GEMM_PAIR=0
// turns them off, =1 forces them where the shape allows; gemm_pair_mode() overrides).
std::atomic<int> g_pair_mode{-2};  // -2: not read from the environment yet

int pair_mode() {
  int m = g_pair_mode.load();
  if (m == -2) {
    const char* e = std::getenv("MDL_B200_GEMM_PAIR");
    int want = e == nullptr ? -1 : std::atoi(e);
    g_pair_mode.compare_exchange_strong(m, want);
    m = g_pair_mode.load();
  }
  return m;
}

// By shape: at least two waves of pairs and a main loop of at least 8 k-blocks per tile
// (short-K products such as OneTrans' d=256 projections are bound by their epilogue,
// and the pair's cross-CTA handshakes then cost more than the halved B traffic saves).
bool use_pair(long long pair_tiles, int splits, int k_per_tile) {
  const int mode = pair_mode();
  if (mode == 0 || splits > 1) return false;
  if (mode == 1) return true;
  return pair_tiles >= num_sms() && k_per_tile >= 8 * BK;
}

// Epilogue kind of a call; -1 for a combination no kernel implements.
int epilogue_kind(const GemmArgs& a) {
  const bool aux_act =
      a.act == GEMM_ACT_DGELU || a.act == GEMM_ACT_DRELU || a.act == GEMM_ACT_DMUL || a.act == GEMM_ACT_ADD;
  if (a.out_fp32) return (a.act == GEMM_ACT_NONE && a.out2 == nullptr && a.colsum == nullptr) ? EPI_F32 : -1;
  if (a.act == GEMM_ACT_GELU || a.act == GEMM_ACT_GELU_GRAD)
    return (!a.accumulate && a.out2 != nullptr) ? EPI_GELU : -1;
  if (aux_act) return (!a.accumulate && a.aux != nullptr) ? EPI_AUX : -1;
  if (a.accumulate) return a.act == GEMM_ACT_NONE ? EPI_ACC_BF16 : -1;
  return EPI_PLAIN;
}

}  // namespace

int gemm_pair_mode(int mode) {
  const int prev = pair_mode();
  if (mode >= -1 && mode <= 1) g_pair_mode.store(mode);
  return prev;
}

cudaError_t gemm_bf16_tcgen05(const GemmArgs& a, cudaStream_t stream) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0 || a.G <= 0 || a.KG <= 0) return cudaSuccess;
  if (a.KG > 1 && (a.G != 1 || (a.ksA % 8) || (a.ksB % 8) || a.ksA <= 0 || a.ksB <= 0))
    return cudaErrorInvalidValue;
  if ((a.lda % 8) || (a.ldb % 8) || (a.G > 1 && ((a.gsA % 8) || (a.gsB % 8))) ||
      (reinterpret_cast<uintptr_t>(a.A) & 15) || (reinterpret_cast<uintptr_t>(a.B) & 15))
    return cudaErrorInvalidValue;
  if (!a.out_fp32 && (a.ldc % 8)) return cudaErrorInvalidValue;
  if (a.out_fp32 && (a.ldc % 4)) return cudaErrorInvalidValue;
  // vector epilogue stores: 16 bytes (fp32) / 8 bytes (bf16) per lane; aux read 16 bytes per lane
  if (a.G > 1 && (a.gsC % 4)) return cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(a.out) & (a.out_fp32 ? 15 : 7)) return cudaErrorInvalidValue;
  if (a.out2 != nullptr && (reinterpret_cast<uintptr_t>(a.out2) & 7)) return cudaErrorInvalidValue;
  if (a.aux != nullptr && ((a.ld_aux % 8) || (a.G > 1 && (a.gs_aux % 8)) || (reinterpret_cast<uintptr_t>(a.aux) & 15)))
    return cudaErrorInvalidValue;
  const int epi = epilogue_kind(a);
  if (epi < 0) return cudaErrorInvalidValue;
  const long long pair_tiles =
      static_cast<long long>((a.M + 2 * BM - 1) / (2 * BM)) * ((a.N + BN - 1) / BN) * static_cast<long long>(a.G);
  CUtensorMap ta, tb;
  bool ok;
  // third map dimension: K ranges (KG > 1), batch groups, or 1 for a shared operand
  const bool a_shared = a.G > 1 && a.gsA == 0;
  const bool b_shared = a.G > 1 && a.gsB == 0;
  const uint64_t za = a.KG > 1 ? a.KG : (a_shared ? 1 : a.G);
  const uint64_t zb = a.KG > 1 ? a.KG : (b_shared ? 1 : a.G);
  const long long sa = a.KG > 1 ? a.ksA : a.gsA;
  const long long sb = a.KG > 1 ? a.ksB : a.gsB;
  if (!a.a_mn_major)
    ok = encode_map(&ta, a.A, a.K, a.M, za, a.lda, sa, BM);
  else
    ok = encode_map(&ta, a.A, a.M, a.K, za, a.lda, sa, BK);
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
  ep.KG = a.KG;
  ep.a_shared = a_shared ? 1 : 0;
  ep.b_shared = b_shared ? 1 : 0;
  ep.err = a.err;
  long long tiles =
      static_cast<long long>((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN) * static_cast<long long>(a.G);
  // Split K across CTAs when the output has too few tiles to fill the GPU (weight
  // gradients: a few output tiles over a K of many thousand rows). Only for an fp32
  // output that is accumulated into, which the slices then add to atomically.
  const int total_kb = ((a.K + BK - 1) / BK) * a.KG;
  ep.splits = 1;
  ep.kb_per_split = total_kb;
  if (epi == EPI_F32 && a.accumulate && tiles * 2 <= num_sms() && total_kb >= 8) {
    long long want = (num_sms() + tiles - 1) / tiles;
    want = std::min<long long>(want, total_kb / 4);
    if (want > 1) {
      ep.kb_per_split = static_cast<int>((total_kb + want - 1) / want);
      ep.splits = (total_kb + ep.kb_per_split - 1) / ep.kb_per_split;
    }
  }
  const bool pair = use_pair(pair_tiles, ep.splits, ep.kb_per_split * BK) && a.max_ctas <= 0;
  // B operand map: each CTA of a pair stages half of the tile's 256 B rows
  const uint32_t b_box = pair ? BN / 2 : BN;
  if (!a.b_mn_major)
    ok = encode_map(&tb, a.B, a.K, a.N, zb, a.ldb, sb, b_box);
  else
    ok = encode_map(&tb, a.B, a.N, a.K, zb, a.ldb, sb, BK);
  if (!ok) return cudaErrorInvalidValue;
  if (pair) {
    tiles = pair_tiles;
    int clusters = num_sms() / 2;
    if (tiles < clusters) clusters = static_cast<int>(tiles);
    return launch_any<true>(a.a_mn_major, a.b_mn_major, ta, tb, ep, epi, 2 * clusters, stream);
  }
  const long long units = tiles * ep.splits;
  int grid = num_sms();
  if (a.max_ctas > 0 && a.max_ctas < grid) grid = a.max_ctas;
  if (units < grid) grid = static_cast<int>(units);
  return launch_any<false>(a.a_mn_major, a.b_mn_major, ta, tb, ep, epi, grid, stream);
}

}  // namespace mdl
