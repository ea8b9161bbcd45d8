// Flash attention for sm_100a on the 5th-generation tensor cores: scores and
// products in TMEM (tcgen05.mma), operands staged by TMA with 128-byte swizzle,
// softmax in registers, one warp-specialised CTA per tile.
//
// Serves the OneTrans mixed causal attention (queries = the pyramid-pruned
// suffix of the [S; NS] token sequence, bottom-right causal, prefix padding
// given as a per-sample first valid key; reference
// MixedCausalAttention.attend_causal_suffix src/model.py:5617-5695, which
// packs the valid tokens and calls flash_attn_varlen_func,
// src/attention.py:103-162). Padding is never packed away here: a sample's
// prefix of invalid keys is skipped a whole 128-key tile at a time and masked
// inside the boundary tile.
//
// Tiling. Query and key tiles are 128 token rows aligned to the END of the
// sequence (tile t = rows Lk-128(t+1) .. Lk-128t-1), so query tile i meets key
// tile i on the diagonal (the only tile with a causal mask) and key tiles
// t > i in full. Rows before the first token read as zeros (TMA fill).
//
// Forward (192 threads, 2 persistent CTAs/SM, 256 TMEM columns each): a work
// item = one sample, one head, one query tile. TMA boxes are 64 columns (one 128-byte
// swizzled row) starting at the head, so the MMAs read the head's 32 columns.
//   warp 0      TMA: Q once, K and V tiles into 2-stage rings
//   warp 1      MMA: S = Q K^T (M=128, N=128, K=32) into TMEM, then
//               PV = P V (M=128, N=64, K=128) into a TMEM double buffer
//   warps 2-5   softmax: thread = query row; online max / sum in base 2, P as
//               bf16 into swizzled smem; the PV of tile j-1 is folded into the
//               register accumulator while the tensor core works on tile j.
// Backward (320 threads, one persistent CTA per SM): a work item = one sample,
// one head, one key tile; it walks the query tiles that see those keys:
//   S^T = K Q^T and dP^T = V dO^T (thread = key row), P^T = exp2(S^T*c - lse),
//   dS^T = P^T (dP^T - D) * scale, dV += P^T dO, dK += dS^T Q (accumulated in
//   TMEM), dQ_tile = dS K (same smem dS^T read as an MN-major operand) added
//   to an fp32 buffer with vector reductions.
//
// Every wait is bounded (error word + abort flag) and every role drains what
// it has in flight before the CTA exits.
//
// Registers: 10 warps (backward) or 2 x 6 warps (forward) spread at most 3 per
// SM sub-partition, each with 16K registers, so a thread may hold at most 168.
#include <cudaTypedefs.h>

#include <math_constants.h>

#include <algorithm>
#include <climits>
#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "fmha.h"

namespace mdl {
namespace {

void bind_context_once() {
  thread_local bool bound = false;
  if (!bound) {
    cudaFree(nullptr);  // makes the device's primary context current on this thread
    bound = true;
  }
}

constexpr int HD = 32;
constexpr int TILE = 128;
constexpr int TILE_BYTES = TILE * 128;  // 128 rows x 128 bytes (64 bf16 = two heads)
constexpr int P_BYTES = 2 * TILE_BYTES; // 128 x 128 bf16 as two 64-column swizzled blocks
constexpr int NUM_THREADS = 320;
constexpr int TMEM_COLS = 512;
constexpr float kLog2e = 1.4426950408889634f;

// forward (one head per CTA, two CTAs per SM): Q | K[2] | V[2] | P | barriers. Two
// CTAs fit in the SM's shared memory only without alignment slack: the kernel
// relies on the dynamic shared memory base being 1024-byte aligned (it is when
// the kernel has no static shared memory) and checks it.
constexpr int F_THREADS = 192;
constexpr int F_TMEM = 256;
constexpr int F_SMEM = TILE_BYTES * 5 + P_BYTES + 256;
// backward smem: K[2] | V[2] | Q[2] | dO[2] | P^T | dS^T | lse[2][128] | D[2][128] | barriers
constexpr int B_SMEM = 1024 + TILE_BYTES * 8 + 2 * P_BYTES + 4 * TILE * 4 + 256;
static_assert(F_SMEM <= 232448 && B_SMEM <= 232448, "shared memory budget");

struct Params {
  void* out;
  float* lse;
  const int* kstart;
  float* dq_acc;
  const float* dsum;
  void* dqkv;
  int B, H, Lk, Lq, D, causal;
  int ktail;  // the last ktail tokens see and are seen by every token (causal only)
  int kexcl;  // of those, the last kexcl are seen only by themselves (causal only)
  float scale, scale2;
  int* err;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA / integer pipes, for x <= 0: Cody-Waite style split x = j + f with
// j = round(x) taken from the low mantissa bits of x + 1.5*2^23, 2^f by a degree-3
// polynomial on [-0.5, 0.5] (fitted here to 2^f with near-minimax relative weighting;
// largest relative error 7.5e-5 in fp32, far below bf16 rounding), and 2^j added to
// the exponent bits; x < -125 (masked scores included) gives 0. Used for part of the
// softmax exponentials so that they do not all queue on the special-function unit.
__device__ __forceinline__ float ex2_fma(float x) {
  const float shift = 12582912.f;  // 1.5 * 2^23
  const float t = x + shift;
  const float j = t - shift;
  const float f = x - j;
  float q = fmaf(0.0551716648f, f, 0.2426111251f);
  q = fmaf(q, f, 0.6932609677f);
  q = fmaf(q, f, 0.9999280572f);
  const int ji = __float_as_int(t) - 0x4B400000;
  const float r = __int_as_float(__float_as_int(q) + (ji << 23));
  return x < -125.f ? 0.f : r;
}

// Element k (0..7) of an 8-wide chunk: polynomial when EXPV > 0 and k % EXPV == 0.
template <int EXPV>
__device__ __forceinline__ float ex2_mix(float x, int k) {
  if constexpr (EXPV > 0) {
    if (k % EXPV == 0) return ex2_fma(x);
  }
  return ex2(x);
}

__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void st_smem_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Round-to-nearest-even bf16 pair of two finite floats with integer ops only (keeps
// the conversions off the special-function pipe, which the exponentials saturate):
// add 0x7FFF plus the lowest kept bit, keep the high halves.
__device__ __forceinline__ uint32_t pack2_int(float a, float b) {
  uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
  ua += 0x7FFFu + ((ua >> 16) & 1u);
  ub += 0x7FFFu + ((ub >> 16) & 1u);
  return __byte_perm(ua, ub, 0x7632);
}

template <bool INT_PACK>
__device__ __forceinline__ uint32_t packp(float a, float b) {
  if constexpr (INT_PACK) return pack2_int(a, b);
  return pack2(a, b);
}

// 32 consecutive fp32 TMEM columns of this thread's lane, no wait.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// K-major operand, 128-byte swizzle: `k_bytes` selects the 16-element K step inside the row.
__device__ __forceinline__ uint64_t desc_k(uint32_t base, uint32_t k_bytes) {
  return make_smem_desc(base + k_bytes, 16, 1024);
}
// 128 x 128 operand stored as two 64-column K-major blocks: K step s (16 columns).
__device__ __forceinline__ uint64_t desc_k128(uint32_t base, int s) {
  return make_smem_desc(base + (s >> 2) * TILE_BYTES + (s & 3) * 32, 16, 1024);
}
// MN-major operand (rows = K, 64 contiguous MN elements per 128-byte row; a
// second 64-wide MN block TILE_BYTES further): K step s = 16 rows.
__device__ __forceinline__ uint64_t desc_mn(uint32_t base, int s) {
  return make_smem_desc(base + s * 2048, TILE_BYTES, 1024);
}

// Byte offset of 16-byte chunk `c` (0..15) of row `r` in a 128 x 128 bf16 block pair.
__device__ __forceinline__ uint32_t swz_off(int r, int c) {
  return (c >> 3) * TILE_BYTES + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

// A wait whose outcome is the same on every lane of the warp: the tcgen05.ld /
// wait::ld that follow are .sync.aligned and must be executed by the whole warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag) {
  const bool ok = mbar_wait(bar, parity, err, abort_flag);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void red_add_v4(float* dst, float a, float b, float c, float d) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(dst), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

// Bits [l, h] (inclusive, clipped) of 32-column word w of a 128-column tile.
__device__ __forceinline__ uint32_t range_bits(int l, int h, int w) {
  const int a = max(l - 32 * w, 0), b = min(h - 32 * w, 31);
  if (a > b) return 0u;
  const uint32_t upto = b == 31 ? 0xFFFFFFFFu : ((1u << (b + 1)) - 1u);
  return upto & (0xFFFFFFFFu << a);
}

// ============================================================================ forward
// Work item = (sample, head, query tile); items are numbered heaviest first (query
// tile 0 = the last 128 rows sees the most key tiles under causality).
struct FwdItem {
  int b, h, i, t0, n, kst, extra0;
};

__device__ __forceinline__ FwdItem fwd_item(const Params& p, int w) {
  FwdItem it;
  it.h = w % p.H;
  const int rest = w / p.H;
  it.b = rest % p.B;
  it.i = rest / p.B;
  it.kst = min(max(p.kstart[it.b], 0), p.Lk);
  const int tmax = (p.Lk - it.kst + TILE - 1) / TILE - 1;
  it.t0 = p.causal ? it.i : 0;
  // trailing always-visible tokens live in key tile 0, which a causal query tile
  // i > 0 would otherwise skip: visit it first
  it.extra0 = (p.causal && p.ktail > 0 && it.i > 0 && tmax >= 0) ? 1 : 0;
  it.n = max(0, tmax - it.t0 + 1) + it.extra0;  // key tiles visited
  return it;
}

// Key tile of the j-th visited tile of an item.
__device__ __forceinline__ int fwd_tile(const FwdItem& it, int j) {
  return it.extra0 ? (j == 0 ? 0 : it.t0 + j - 1) : it.t0 + j;
}

// Persistent: each CTA walks items blockIdx.x, +gridDim.x, ...; the K/V rings and
// every barrier phase run on across items (global tile counter g), so the loads of
// the next item overlap the softmax of the current one.
template <bool INT_PACK, int EXPV>
__global__ void __launch_bounds__(F_THREADS, 2)
    fmha_fwd_kernel(const __grid_constant__ CUtensorMap tm, const Params p, int num_items) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023) {  // uniform across the CTA: nothing has been touched yet
    if (threadIdx.x == 0) record_error(p.err, MDL_ERR_BAD_ARG);
    return;
  }
  uint8_t* sQ = smem_raw;
  uint8_t* sK = sQ + TILE_BYTES;      // [2]
  uint8_t* sV = sK + 2 * TILE_BYTES;  // [2]
  uint8_t* sP = sV + 2 * TILE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;      // [2]
  uint64_t* k_empty = bars + 4;     // [2]
  uint64_t* v_full = bars + 6;      // [2]
  uint64_t* v_empty = bars + 8;     // [2]
  uint64_t* s_full = bars + 10;
  uint64_t* s_empty = bars + 11;
  uint64_t* p_full = bars + 12;
  uint64_t* p_empty = bars + 13;
  uint64_t* pv_full = bars + 14;    // [2]
  uint64_t* pv_empty = bars + 16;   // [2]
  uint64_t* done = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int Lk = p.Lk;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&pv_full[s], 1);
      mbar_init(&pv_empty[s], 4);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, 4);
    mbar_init(p_full, 4);
    mbar_init(p_empty, 1);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, F_TMEM);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm);
      int items = 0, g = 0;  // items with work, tiles issued (global)
      int k_issued = 0, v_issued = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < num_items && ok; w += gridDim.x) {
        const FwdItem it = fwd_item(p, w);
        if (it.n == 0) continue;
        if (items >= 1 && !mbar_wait(q_empty, (items - 1) & 1, p.err, abort_flag)) break;
        mbar_arrive_expect_tx(q_full, TILE_BYTES);
        tma_load_3d(sQ, &tm, q_full, it.h * HD, Lk - TILE * (it.i + 1), it.b);
        ++items;
        for (int j = 0; j < it.n; ++j, ++g) {
          const int st = g & 1;
          const int y = Lk - TILE * (fwd_tile(it, j) + 1);
          if (g >= 2 && !mbar_wait(&k_empty[st], ((g >> 1) - 1) & 1, p.err, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&k_full[st], TILE_BYTES);
          tma_load_3d(sK + st * TILE_BYTES, &tm, &k_full[st], p.D + it.h * HD, y, it.b);
          k_issued = g + 1;
          if (g >= 2 && !mbar_wait(&v_empty[st], ((g >> 1) - 1) & 1, p.err, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&v_full[st], TILE_BYTES);
          tma_load_3d(sV + st * TILE_BYTES, &tm, &v_full[st], 2 * p.D + it.h * HD, y, it.b);
          v_issued = g + 1;
        }
      }
      // every copy into this CTA's smem has landed before the CTA may exit
      if (items > 0) mbar_wait(q_full, (items - 1) & 1, nullptr, nullptr);
      for (int j = max(0, k_issued - 2); j < k_issued; ++j) mbar_wait(&k_full[j & 1], (j >> 1) & 1, nullptr, nullptr);
      for (int j = max(0, v_issued - 2); j < v_issued; ++j) mbar_wait(&v_full[j & 1], (j >> 1) & 1, nullptr, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(TILE, TILE, false, false);
      constexpr uint32_t idesc_pv = make_idesc_bf16(TILE, 64, false, true);
      const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV), p_base = smem_u32(sP);
      bool ok = true;
      int items = 0, g0 = 0;
      // S(g) = Q K(g)^T; the item's last S releases Q
      auto issue_s = [&](int g, bool last) -> bool {
        if (!mbar_wait(&k_full[g & 1], (g >> 1) & 1, p.err, abort_flag) ||
            (g > 0 && !mbar_wait(s_empty, (g - 1) & 1, p.err, abort_flag)))
          return false;
        tc_fence_after();
        const uint32_t kb = k_base + (g & 1) * TILE_BYTES;
        for (int ks = 0; ks < 2; ++ks)
          tc_mma_bf16(tmem, desc_k(q_base, ks * 32), desc_k(kb, ks * 32), idesc_s, ks);
        tc_commit(&k_empty[g & 1]);
        tc_commit(s_full);
        if (last) tc_commit(q_empty);
        return true;
      };
      for (int w = blockIdx.x; w < num_items && ok; w += gridDim.x) {
        const FwdItem it = fwd_item(p, w);
        if (it.n == 0) continue;
        if (!mbar_wait(q_full, items & 1, p.err, abort_flag) || !issue_s(g0, it.n == 1)) break;
        ++items;
        for (int j = 0; j < it.n; ++j) {
          const int g = g0 + j;
          if (j + 1 < it.n && !issue_s(g + 1, j + 2 == it.n)) {
            ok = false;
            break;
          }
          const int buf = g & 1;
          if (!mbar_wait(p_full, g & 1, p.err, abort_flag) ||
              !mbar_wait(&v_full[buf], (g >> 1) & 1, p.err, abort_flag) ||
              (g >= 2 && !mbar_wait(&pv_empty[buf], ((g >> 1) - 1) & 1, p.err, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int ks = 0; ks < 8; ++ks)
            tc_mma_bf16(tmem + 128 + buf * 64, desc_k128(p_base, ks), desc_mn(v_base + buf * TILE_BYTES, ks),
                        idesc_pv, ks);
          tc_commit(&pv_full[buf]);
          tc_commit(p_empty);
          tc_commit(&v_empty[buf]);
        }
        g0 += it.n;
      }
      // all MMAs have finished before TMEM is released
      tc_commit(done);
      mbar_wait(done, 0, nullptr, nullptr);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t p_base = smem_u32(sP);
    bool ok = true;
    int g0 = 0;
    for (int w = blockIdx.x; w < num_items && ok; w += gridDim.x) {
      const FwdItem it = fwd_item(p, w);
      const int qrow = Lk - TILE * (it.i + 1) + r;
      float m = -CUDART_INF_F, l = 0.f, alpha_prev = 1.f;
      float o[HD];
#pragma unroll
      for (int d = 0; d < HD; ++d) o[d] = 0.f;
      auto fold_pv = [&](int gg) -> bool {
        const int buf = gg & 1;
        if (!warp_wait(&pv_full[buf], (gg >> 1) & 1, p.err, abort_flag)) return false;
        tc_fence_after();
        uint32_t pv[HD];
        tmem_ld32(t_lane + 128 + buf * 64, pv);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pv_empty[buf]);
#pragma unroll
        for (int d = 0; d < HD; ++d) o[d] = fmaf(o[d], alpha_prev, __uint_as_float(pv[d]));
        return true;
      };
      for (int j = 0; j < it.n; ++j) {
        const int g = g0 + j;
        const int t = fwd_tile(it, j);
        const int kbase = Lk - TILE * (t + 1);
        if (!warp_wait(s_full, g & 1, p.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[TILE];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(t_lane + c * 32, sr + c * 32);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_empty);
        // padding, the diagonal tile and the tile of the trailing tokens need a per-column mask
        if (p.ktail == 0) {
          const int lo = it.kst - kbase;                         // columns < lo are padding
          const int hi = (p.causal && t == it.i) ? r : TILE - 1;  // columns > hi are in the future
          if (lo > 0 || hi < TILE - 1) {
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              const uint32_t vm = range_bits(lo, hi, w);
#pragma unroll
              for (int c = 0; c < 32; ++c)
                if (!((vm >> c) & 1u)) sr[32 * w + c] = __float_as_uint(-CUDART_INF_F);
            }
          }
        } else if (it.kst > kbase || t == it.i || t == 0) {
          // (ktail > 0 implies causal.) The row's visible columns are at most two intervals:
          // [lo, h1] (the causal part, or everything a global query sees) and [l2, h2] (the
          // trailing global keys a sequence query sees). They become a 128-bit mask, so each
          // column costs a bit test and a select instead of the full visibility expression.
          const int tail0 = Lk - p.ktail;
          const int excl0 = Lk - p.kexcl;  // keys from here on: only queries from here on see them
          const int lo = it.kst - kbase;
          int h1, l2 = TILE, h2 = -1;
          if (qrow >= excl0) {
            h1 = TILE - 1;
          } else if (qrow >= tail0) {
            h1 = excl0 - 1 - kbase;
          } else {
            h1 = qrow - kbase;
            l2 = max(lo, tail0 - kbase);
            h2 = excl0 - 1 - kbase;
          }
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const uint32_t vm = range_bits(lo, h1, w) | range_bits(l2, h2, w);
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (!((vm >> c) & 1u)) sr[32 * w + c] = __float_as_uint(-CUDART_INF_F);
          }
        }
        float mx8[8];  // eight independent partial maxima (short dependency chains)
#pragma unroll
        for (int k = 0; k < 8; ++k) mx8[k] = __uint_as_float(sr[k]);
#pragma unroll
        for (int c = 8; c < TILE; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], __uint_as_float(sr[c]));
        const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        const float m_new = fmaxf(m, mx * p.scale2);
        const float m_use = m_new == -CUDART_INF_F ? 0.f : m_new;
        const float alpha = ex2(m - m_use);
        if (g > 0 && !warp_wait(p_empty, (g - 1) & 1, p.err, abort_flag)) {  // P(g-1) consumed
          ok = false;
          break;
        }
        float sum8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          float e[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            e[k] = ex2_mix<EXPV>(fmaf(__uint_as_float(sr[c * 8 + k]), p.scale2, -m_use), k);
            sum8[k] += e[k];
          }
          st_smem_v4(p_base + swz_off(r, c), packp<INT_PACK>(e[0], e[1]), packp<INT_PACK>(e[2], e[3]),
                     packp<INT_PACK>(e[4], e[5]), packp<INT_PACK>(e[6], e[7]));
        }
        const float sum = ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) + ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        l = fmaf(l, alpha, sum);
        m = m_new;
        if (j > 0 && !fold_pv(g - 1)) {
          ok = false;
          break;
        }
        alpha_prev = alpha;
      }
      if (ok && it.n > 0) ok = fold_pv(g0 + it.n - 1);
      if (!ok) break;
      g0 += it.n;
      const int qi = qrow - (Lk - p.Lq);
      if (qi >= 0) {
        const bool valid = qrow >= it.kst && l > 0.f;
        const float inv = valid ? 1.f / l : 0.f;
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) +
                                              (static_cast<long long>(it.b) * p.Lq + qi) * p.D + it.h * HD);
#pragma unroll
        for (int c = 0; c < HD / 8; ++c)
          dst[c] = make_uint4(pack2(o[c * 8] * inv, o[c * 8 + 1] * inv), pack2(o[c * 8 + 2] * inv, o[c * 8 + 3] * inv),
                              pack2(o[c * 8 + 4] * inv, o[c * 8 + 5] * inv), pack2(o[c * 8 + 6] * inv, o[c * 8 + 7] * inv));
        p.lse[(static_cast<long long>(it.b) * p.H + it.h) * p.Lq + qi] = valid ? m + lg2(l) : CUDART_INF_F;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, F_TMEM);
  }
}

// ============================================================================ backward
// D[b,h,q] = sum_d dO*O over the head; zero the dQ accumulator row.
__global__ void __launch_bounds__(256) fmha_bwd_pre_kernel(const __nv_bfloat16* __restrict__ out,
                                                           const __nv_bfloat16* __restrict__ dout,
                                                           float* __restrict__ dsum, float* __restrict__ dq_acc,
                                                           int B, int Lq, int H, int D) {
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= static_cast<long long>(B) * Lq) return;
  const int b = static_cast<int>(row / Lq);
  const int q = static_cast<int>(row - static_cast<long long>(b) * Lq);
  for (int base = 0; base < D; base += 256) {  // warp-uniform trip count (shuffles below)
    const int c = base + lane * 8;
    const bool active = c < D;
    float acc = 0.f;
    if (active) {
      const uint4 ov = *reinterpret_cast<const uint4*>(out + row * D + c);
      const uint4 gv = *reinterpret_cast<const uint4*>(dout + row * D + c);
      const uint32_t* o32 = reinterpret_cast<const uint32_t*>(&ov);
      const uint32_t* g32 = reinterpret_cast<const uint32_t*>(&gv);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        acc = fmaf(bf16_bits_to_float(o32[k] & 0xFFFFu), bf16_bits_to_float(g32[k] & 0xFFFFu), acc);
        acc = fmaf(bf16_bits_to_float(o32[k] >> 16), bf16_bits_to_float(g32[k] >> 16), acc);
      }
      *reinterpret_cast<float4*>(dq_acc + row * D + c) = make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(dq_acc + row * D + c + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // four lanes hold one head (32 elements)
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if (active && (lane & 3) == 0) dsum[(static_cast<long long>(b) * H + c / HD) * Lq + q] = acc;
  }
}

// Work item = (sample, head, key tile); items with the most query tiles come first.
struct BwdItem {
  int b, h, kbase, kst, qlo, n;
};

__device__ __forceinline__ BwdItem bwd_item(const Params& p, int w) {
  BwdItem it;
  const int nkt = (p.Lk + TILE - 1) / TILE;
  it.h = w % p.H;
  const int rest = w / p.H;
  it.b = rest % p.B;
  const int t = nkt - 1 - rest / p.B;
  it.kbase = p.Lk - TILE * (t + 1);
  it.kst = min(max(p.kstart[it.b], 0), p.Lk);
  it.qlo = max(it.kst, p.Lk - p.Lq);  // first row that is a query with a visible key
  const int nq = (p.Lq + TILE - 1) / TILE;
  // key tile 0 holds the trailing always-visible tokens: every query tile sees it
  int imax = (p.causal && !(p.ktail > 0 && t == 0)) ? min(t, nq - 1) : nq - 1;
  imax = min(imax, (p.Lk - 1 - it.qlo) / TILE);
  it.n = (it.kbase + TILE - 1 >= it.kst && it.qlo < p.Lk) ? max(0, imax + 1) : 0;  // query tiles visited
  return it;
}

// Persistent: K/V of successive items in a 2-stage ring, Q/dO/lse/D of successive
// query tiles in a 2-stage ring; barrier phases run on across items (item counter
// for K/V and dK/dV, global query-tile counter for the rest).
template <bool INT_PACK, int EXPV>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    fmha_bwd_kernel(const __grid_constant__ CUtensorMap tm, const __grid_constant__ CUtensorMap tm_do,
                    const Params p, int num_items) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sK = smem;                   // [2]
  uint8_t* sV = sK + 2 * TILE_BYTES;    // [2]
  uint8_t* sQ = sV + 2 * TILE_BYTES;    // [2]
  uint8_t* sdO = sQ + 2 * TILE_BYTES;   // [2]
  uint8_t* sPT = sdO + 2 * TILE_BYTES;
  uint8_t* sdST = sPT + P_BYTES;
  float* sLse = reinterpret_cast<float*>(sdST + P_BYTES);  // [2][128]
  float* sDs = sLse + 2 * TILE;                            // [2][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDs + 2 * TILE);
  uint64_t* kv_full = bars;        // [2]
  uint64_t* kv_empty = bars + 2;   // [2]
  uint64_t* qd_full = bars + 4;    // [2]
  uint64_t* qd_empty = bars + 6;   // [2]
  uint64_t* st_full = bars + 8;
  uint64_t* st_empty = bars + 9;
  uint64_t* pds_full = bars + 10;
  uint64_t* pds_empty = bars + 11;
  uint64_t* dq_full = bars + 12;
  uint64_t* dq_empty = bars + 13;
  uint64_t* dkv_full = bars + 14;
  uint64_t* dkv_empty = bars + 15;
  uint64_t* done = bars + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int Lk = p.Lk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&qd_full[s], 33);  // TMA bytes + the 32 lanes that stage lse / D
      mbar_init(&qd_empty[s], 1);
    }
    mbar_init(st_full, 1);
    mbar_init(st_empty, 8);
    mbar_init(pds_full, 8);
    mbar_init(pds_empty, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 8);
    mbar_init(dkv_full, 1);
    mbar_init(dkv_empty, 8);
    mbar_init(done, 1);
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
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm);
      tma_prefetch_desc(&tm_do);
    }
    int items = 0, gq = 0, kv_issued = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < num_items && ok; w += gridDim.x) {
      const BwdItem it = bwd_item(p, w);
      if (it.n == 0) continue;
      const int stk = items & 1;
      if (lane == 0) {
        if (items >= 2 && !mbar_wait(&kv_empty[stk], ((items >> 1) - 1) & 1, p.err, abort_flag)) ok = false;
        if (ok) {
          mbar_arrive_expect_tx(&kv_full[stk], 2 * TILE_BYTES);
          tma_load_3d(sK + stk * TILE_BYTES, &tm, &kv_full[stk], p.D + it.h * HD, it.kbase, it.b);
          tma_load_3d(sV + stk * TILE_BYTES, &tm, &kv_full[stk], 2 * p.D + it.h * HD, it.kbase, it.b);
          kv_issued = items + 1;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      ++items;
      for (int j = 0; j < it.n; ++j, ++gq) {
        const int st = gq & 1;
        // parity of the previous use of this stage; a fresh barrier passes parity 1 at once
        if (!warp_wait(&qd_empty[st], ((gq >> 1) + 1) & 1, p.err, abort_flag)) {
          ok = false;
          break;
        }
        const int qrow0 = Lk - TILE * (j + 1);  // token row of query column 0
        if (lane == 0) {
          mbar_arrive_expect_tx(&qd_full[st], 2 * TILE_BYTES);
          tma_load_3d(sQ + st * TILE_BYTES, &tm, &qd_full[st], it.h * HD, qrow0, it.b);
          tma_load_3d(sdO + st * TILE_BYTES, &tm_do, &qd_full[st], it.h * HD, qrow0 - (Lk - p.Lq), it.b);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = lane * 4 + e;
          const int qi = qrow0 + c - (Lk - p.Lq);
          const bool real = qi >= 0 && qrow0 + c >= it.qlo;
          const long long off = (static_cast<long long>(it.b) * p.H + it.h) * p.Lq + qi;
          sLse[st * TILE + c] = real ? p.lse[off] : CUDART_INF_F;
          sDs[st * TILE + c] = real ? p.dsum[off] : 0.f;
        }
        mbar_arrive(&qd_full[st]);
      }
    }
    if (lane == 0) {
      for (int j = max(0, kv_issued - 2); j < kv_issued; ++j) mbar_wait(&kv_full[j & 1], (j >> 1) & 1, nullptr, nullptr);
      for (int j = max(0, gq - 2); j < gq; ++j) mbar_wait(&qd_full[j & 1], (j >> 1) & 1, nullptr, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(TILE, TILE, false, false);
      constexpr uint32_t idesc_kv = make_idesc_bf16(TILE, 64, false, true);
      constexpr uint32_t idesc_q = make_idesc_bf16(TILE, 64, true, true);
      const uint32_t pt_base = smem_u32(sPT), ds_base = smem_u32(sdST);
      int items = 0, gq = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < num_items && ok; w += gridDim.x) {
        const BwdItem it = bwd_item(p, w);
        if (it.n == 0) continue;
        const int stk = items & 1;
        const uint32_t k_base = smem_u32(sK + stk * TILE_BYTES), v_base = smem_u32(sV + stk * TILE_BYTES);
        if (!mbar_wait(&kv_full[stk], (items >> 1) & 1, p.err, abort_flag)) break;
        // S^T / dP^T of query tile g, issued as soon as the compute warps hold tile g-1
        auto issue_s = [&](int g) -> bool {
          const int st = g & 1;
          if (!mbar_wait(&qd_full[st], (g >> 1) & 1, p.err, abort_flag) ||
              (g > 0 && !mbar_wait(st_empty, (g - 1) & 1, p.err, abort_flag)))
            return false;
          tc_fence_after();
          const uint32_t q_base = smem_u32(sQ + st * TILE_BYTES);
          const uint32_t do_base = smem_u32(sdO + st * TILE_BYTES);
          for (int ks = 0; ks < 2; ++ks) {
            tc_mma_bf16(tmem, desc_k(k_base, ks * 32), desc_k(q_base, ks * 32), idesc_s, ks);
            tc_mma_bf16(tmem + 128, desc_k(v_base, ks * 32), desc_k(do_base, ks * 32), idesc_s, ks);
          }
          tc_commit(st_full);
          return true;
        };
        if (!issue_s(gq)) break;
        for (int j = 0; j < it.n; ++j) {
          const int g = gq + j;
          const int st = g & 1;
          const uint32_t q_base = smem_u32(sQ + st * TILE_BYTES);
          const uint32_t do_base = smem_u32(sdO + st * TILE_BYTES);
          if ((j + 1 < it.n && !issue_s(g + 1)) || !mbar_wait(pds_full, g & 1, p.err, abort_flag) ||
              (j == 0 && items >= 1 && !mbar_wait(dkv_empty, (items - 1) & 1, p.err, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int ks = 0; ks < 8; ++ks) {
            const uint32_t acc = (j > 0 || ks > 0) ? 1u : 0u;
            tc_mma_bf16(tmem + 256, desc_k128(pt_base, ks), desc_mn(do_base, ks), idesc_kv, acc);
            tc_mma_bf16(tmem + 320, desc_k128(ds_base, ks), desc_mn(q_base, ks), idesc_kv, acc);
          }
          if (g > 0 && !mbar_wait(dq_empty, (g - 1) & 1, p.err, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int ks = 0; ks < 8; ++ks)
            tc_mma_bf16(tmem + 384, desc_mn(ds_base, ks), desc_mn(k_base, ks), idesc_q, ks);
          tc_commit(dq_full);
          tc_commit(pds_empty);
          tc_commit(&qd_empty[st]);
        }
        if (!ok) break;
        tc_commit(dkv_full);
        tc_commit(&kv_empty[stk]);
        gq += it.n;
        ++items;
      }
      tc_commit(done);
      mbar_wait(done, 0, nullptr, nullptr);
    }
  } else {
    // ------------------------------------------------------------ compute
    const int wg = (warp - 2) >> 2;  // query columns [64*wg, 64*wg + 64)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t pt_base = smem_u32(sPT), ds_base = smem_u32(sdST);
    bool ok = true;
    int items = 0, gq = 0;
    for (int w = blockIdx.x; w < num_items && ok; w += gridDim.x) {
      const BwdItem it = bwd_item(p, w);
      const int krow = it.kbase + r;
      const bool key_ok = krow >= it.kst;
      auto drain_dq = [&](int g, int j) -> bool {
        if (!warp_wait(dq_full, g & 1, p.err, abort_flag)) return false;
        tc_fence_after();
        uint32_t gr[16];
        tmem_ld16(t_lane + 384 + wg * 16, gr);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_empty);
        const int qrow = Lk - TILE * (j + 1) + r;  // TMEM lane = query column of tile j
        if (qrow >= it.qlo) {
          float* dst = p.dq_acc + (static_cast<long long>(it.b) * p.Lq + (qrow - (Lk - p.Lq))) * p.D + it.h * HD +
                       wg * 16;
#pragma unroll
          for (int c = 0; c < 4; ++c)
            red_add_v4(dst + c * 4, __uint_as_float(gr[c * 4]), __uint_as_float(gr[c * 4 + 1]),
                       __uint_as_float(gr[c * 4 + 2]), __uint_as_float(gr[c * 4 + 3]));
        }
        return true;
      };
      for (int j = 0; j < it.n; ++j) {
        const int g = gq + j;
        const int st = g & 1;
        const int qrow0 = Lk - TILE * (j + 1);
        if (!warp_wait(&qd_full[st], (g >> 1) & 1, p.err, abort_flag) || !warp_wait(st_full, g & 1, p.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t s[64], dp[64];
        tmem_ld32(t_lane + wg * 64, s);
        tmem_ld32(t_lane + wg * 64 + 32, s + 32);
        tmem_ld32(t_lane + 128 + wg * 64, dp);
        tmem_ld32(t_lane + 128 + wg * 64 + 32, dp + 32);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(st_empty);
        if (g > 0 && !warp_wait(pds_empty, (g - 1) & 1, p.err, abort_flag)) {
          ok = false;
          break;
        }
        const float* lse = sLse + st * TILE + wg * 64;
        const float* dsv = sDs + st * TILE + wg * 64;
        // The query columns this lane's key is visible to are one range qc >= cmin:
        // real queries (row >= qlo) that are not before the key (causal), where a
        // trailing always-visible key or query lifts the causal cut.
        const int qcol0 = qrow0 + wg * 64;
        int cmin = it.qlo - qcol0;
        if (p.causal) {
          const int tail0 = Lk - p.ktail;
          const int causal_min = krow >= tail0 ? INT_MIN / 2 : min(krow, tail0) - qcol0;
          cmin = max(cmin, causal_min);
          // an excluded trailing key is seen only by the queries of the excluded block
          if (krow >= Lk - p.kexcl) cmin = max(cmin, Lk - p.kexcl - qcol0);
        }
        if (!key_ok) cmin = INT_MAX / 2;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          float pe[8], de[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int qc = c * 8 + k;
            const float pv = qc >= cmin ? ex2_mix<EXPV>(fmaf(__uint_as_float(s[qc]), p.scale2, -lse[qc]), k) : 0.f;
            pe[k] = pv;
            de[k] = pv * (__uint_as_float(dp[qc]) - dsv[qc]) * p.scale;
          }
          const uint32_t off = swz_off(r, wg * 8 + c);
          st_smem_v4(pt_base + off, packp<INT_PACK>(pe[0], pe[1]), packp<INT_PACK>(pe[2], pe[3]),
                     packp<INT_PACK>(pe[4], pe[5]), packp<INT_PACK>(pe[6], pe[7]));
          st_smem_v4(ds_base + off, packp<INT_PACK>(de[0], de[1]), packp<INT_PACK>(de[2], de[3]),
                     packp<INT_PACK>(de[4], de[5]), packp<INT_PACK>(de[6], de[7]));
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(pds_full);
        if (j > 0 && !drain_dq(g - 1, j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && it.n > 0) ok = drain_dq(gq + it.n - 1, it.n - 1);
      if (!ok) break;
      // dK (warpgroup 1) and dV (warpgroup 0) of this key tile. The TMEM read is
      // done by whole warps; only the store depends on the lane's key row.
      float gk[HD];
#pragma unroll
      for (int d = 0; d < HD; ++d) gk[d] = 0.f;
      if (it.n > 0) {
        if (!warp_wait(dkv_full, items & 1, p.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t gr[HD];
        tmem_ld32(t_lane + (wg == 0 ? 256 : 320), gr);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dkv_empty);
#pragma unroll
        for (int d = 0; d < HD; ++d) gk[d] = key_ok ? __uint_as_float(gr[d]) : 0.f;
        ++items;
      }
      gq += it.n;
      if (krow >= 0) {
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.dqkv) +
                                              (static_cast<long long>(it.b) * Lk + krow) * 3 * p.D +
                                              (wg == 0 ? 2 * p.D : p.D) + it.h * HD);
#pragma unroll
        for (int c = 0; c < HD / 8; ++c)
          dst[c] = make_uint4(pack2(gk[c * 8], gk[c * 8 + 1]), pack2(gk[c * 8 + 2], gk[c * 8 + 3]),
                              pack2(gk[c * 8 + 4], gk[c * 8 + 5]), pack2(gk[c * 8 + 6], gk[c * 8 + 7]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// dqkv[:, :, 0:D] = bf16(dQ) on query rows, 0 elsewhere (8 elements per thread).
__global__ void __launch_bounds__(256) fmha_bwd_post_kernel(const float* __restrict__ dq_acc,
                                                            __nv_bfloat16* __restrict__ dqkv, int B, int Lk,
                                                            int Lq, int D) {
  const long long idx = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  const long long total = static_cast<long long>(B) * Lk * D;
  if (idx >= total) return;
  const long long row = idx / D;
  const int c = static_cast<int>(idx - row * D);
  const int b = static_cast<int>(row / Lk);
  const int k = static_cast<int>(row - static_cast<long long>(b) * Lk);
  const int qi = k - (Lk - Lq);
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (qi >= 0) {
    const float* src = dq_acc + (static_cast<long long>(b) * Lq + qi) * D + c;
    const float4 a = *reinterpret_cast<const float4*>(src);
    const float4 e = *reinterpret_cast<const float4*>(src + 4);
    v = make_uint4(pack2(a.x, a.y), pack2(a.z, a.w), pack2(e.x, e.y), pack2(e.z, e.w));
  }
  *reinterpret_cast<uint4*>(dqkv + row * 3 * D + c) = v;
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// [B, L, W] bf16 rows (row stride W), box 64 x 128 x 1, 128-byte swizzle.
bool encode_rows(CUtensorMap* map, const void* base, uint64_t W, uint64_t L, uint64_t B) {
  auto fn = encode_fn();
  // The encoder is a driver call: it needs this thread's context current (an
  // autograd worker thread may not have made any runtime call yet).
  bind_context_once();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {W, L, B};
  cuuint64_t strides[2] = {W * 2, L * W * 2};
  cuuint32_t box[3] = {64, TILE, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

Params make_params(const FmhaArgs& a) {
  Params p;
  p.out = a.out;
  p.lse = a.lse;
  p.kstart = a.kstart;
  p.dq_acc = a.dq_acc;
  p.dsum = a.dsum;
  p.dqkv = a.dqkv;
  p.B = a.B;
  p.H = a.H;
  p.Lk = a.Lk;
  p.Lq = a.Lq;
  p.D = a.H * HD;
  p.causal = a.causal ? 1 : 0;
  p.ktail = a.causal ? a.ktail : 0;
  p.kexcl = a.causal ? a.kexcl : 0;
  p.scale = a.scale > 0.f ? a.scale : 1.f / sqrtf(static_cast<float>(HD));
  p.scale2 = p.scale * kLog2e;
  p.err = a.err;
  return p;
}

const char* g_reason = "";

// Kernel variant: bf16 packing of P / dS with integer ops or cvt
// (MDL_B200_FMHA_INT_PACK=1/0) x share of exponentials on the FMA pipes
// (MDL_B200_FMHA_EXP_POLY=0: none, 2: every second, 4: every fourth). Measured on
// the OneTrans layer-0 shape (B=1024, L=544, 8 heads): cvt + all exponentials on
// the special-function unit is fastest (forward 1.48 ms, backward 3.52 ms); every
// variant that moves work to the integer / FMA pipes is slower (up to 2.31 / 4.23
// ms), i.e. the kernels are bound by instruction issue and latency, not by the
// special-function unit. Default: cvt, no polynomial.
int kernel_variant() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("MDL_B200_FMHA_INT_PACK");
    const int ip = (e != nullptr && e[0] == '1') ? 1 : 0;
    const char* x = std::getenv("MDL_B200_FMHA_EXP_POLY");
    const int ev = x == nullptr ? 0 : (x[0] == '2' ? 1 : (x[0] == '4' ? 2 : 0));
    v = ip * 3 + ev;
  }
  return v;
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

// Records why a host call failed (read back by fmha_last_error()).
cudaError_t fail(const char* why, cudaError_t e) {
  if (e != cudaSuccess) g_reason = why;
  return e;
}

bool shapes_ok(const FmhaArgs& a) {
  return a.hd == HD && a.B > 0 && a.H > 0 && a.Lq > 0 && a.Lq <= a.Lk && a.kstart != nullptr && a.ktail >= 0 &&
         a.ktail <= TILE && a.ktail <= a.Lq && a.kexcl >= 0 && a.kexcl <= a.ktail &&
         (reinterpret_cast<uintptr_t>(a.qkv) & 15) == 0;
}

}  // namespace

cudaError_t fmha_fwd(const FmhaArgs& a, cudaStream_t stream) {
  if (!shapes_ok(a) || a.out == nullptr || a.lse == nullptr ||
      (reinterpret_cast<uintptr_t>(a.out) & 15))
    return fail("fmha_fwd: bad shapes or pointers", cudaErrorInvalidValue);
  const Params p = make_params(a);
  CUtensorMap tm;
  if (!encode_rows(&tm, a.qkv, 3ull * p.D, a.Lk, a.B)) return fail("fmha_fwd: qkv tensor map", cudaErrorInvalidValue);
  const int variant = kernel_variant();
  using FwdKern = void (*)(const CUtensorMap, const Params, int);
  static const FwdKern kerns[6] = {fmha_fwd_kernel<false, 0>, fmha_fwd_kernel<false, 2>, fmha_fwd_kernel<false, 4>,
                                   fmha_fwd_kernel<true, 0>,  fmha_fwd_kernel<true, 2>,  fmha_fwd_kernel<true, 4>};
  const FwdKern kern = kerns[variant];
  static bool configured[6] = {false, false, false, false, false, false};
  if (!configured[variant]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, F_SMEM);
    if (e != cudaSuccess) return fail("fmha_fwd: smem attribute", e);
    configured[variant] = true;
  }
  const long long items = static_cast<long long>(a.H) * a.B * ((a.Lq + TILE - 1) / TILE);
  if (items > 0x7fffffffLL) return fail("fmha_fwd: too many work items", cudaErrorInvalidValue);
  const int grid = static_cast<int>(std::min<long long>(items, 2LL * num_sms()));
  kern<<<grid, F_THREADS, F_SMEM, stream>>>(tm, p, static_cast<int>(items));
  return fail("fmha_fwd: launch", cudaGetLastError());
}

cudaError_t fmha_bwd(const FmhaArgs& a, cudaStream_t stream) {
  if (!shapes_ok(a) || a.out == nullptr || a.lse == nullptr || a.dout == nullptr || a.dqkv == nullptr ||
      a.dq_acc == nullptr || a.dsum == nullptr || (reinterpret_cast<uintptr_t>(a.dout) & 15) ||
      (reinterpret_cast<uintptr_t>(a.dqkv) & 15) || (reinterpret_cast<uintptr_t>(a.dq_acc) & 15))
    return fail("fmha_bwd: bad shapes or pointers", cudaErrorInvalidValue);
  const Params p = make_params(a);
  CUtensorMap tm, tm_do;
  if (!encode_rows(&tm, a.qkv, 3ull * p.D, a.Lk, a.B)) return fail("fmha_bwd: qkv tensor map", cudaErrorInvalidValue);
  if (!encode_rows(&tm_do, a.dout, p.D, a.Lq, a.B)) return fail("fmha_bwd: dout tensor map", cudaErrorInvalidValue);
  const int variant = kernel_variant();
  using BwdKern = void (*)(const CUtensorMap, const CUtensorMap, const Params, int);
  static const BwdKern kerns[6] = {fmha_bwd_kernel<false, 0>, fmha_bwd_kernel<false, 2>, fmha_bwd_kernel<false, 4>,
                                   fmha_bwd_kernel<true, 0>,  fmha_bwd_kernel<true, 2>,  fmha_bwd_kernel<true, 4>};
  const BwdKern kern = kerns[variant];
  static bool configured[6] = {false, false, false, false, false, false};
  if (!configured[variant]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, B_SMEM);
    if (e != cudaSuccess) return fail("fmha_bwd: smem attribute", e);
    configured[variant] = true;
  }
  const long long rows = static_cast<long long>(a.B) * a.Lq;
  fmha_bwd_pre_kernel<<<static_cast<unsigned>((rows * 32 + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(a.out), reinterpret_cast<const __nv_bfloat16*>(a.dout), a.dsum,
      a.dq_acc, a.B, a.Lq, a.H, p.D);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail("fmha_bwd: pre-kernel launch", e);
  const long long items = static_cast<long long>(a.H) * a.B * ((a.Lk + TILE - 1) / TILE);
  if (items > 0x7fffffffLL) return fail("fmha_bwd: too many work items", cudaErrorInvalidValue);
  const int grid = static_cast<int>(std::min<long long>(items, num_sms()));
  kern<<<grid, NUM_THREADS, B_SMEM, stream>>>(tm, tm_do, p, static_cast<int>(items));
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail("fmha_bwd: main launch", e);
  const long long vec = static_cast<long long>(a.B) * a.Lk * p.D / 8;
  fmha_bwd_post_kernel<<<static_cast<unsigned>((vec + 255) / 256), 256, 0, stream>>>(
      a.dq_acc, reinterpret_cast<__nv_bfloat16*>(a.dqkv), a.B, a.Lk, a.Lq, p.D);
  return fail("fmha_bwd: post-kernel launch", cudaGetLastError());
}

const char* fmha_last_error() { return g_reason; }

}  // namespace mdl
