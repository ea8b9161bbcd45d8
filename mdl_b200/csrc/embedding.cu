// Fused embedding-bag lookup / gradient push / row-wise Adagrad for sm_100a.
//
// Replaces the reference's owner-routed lookup (src/embeddings.py:476-674,
// 1112-1517: unique -> argsort -> all_to_all of split counts with a host read
// -> all_to_all of ids -> gather -> all_to_all of rows -> index_copy), its
// mean pooling of bags (src/model.py:509-678) and its Triton row-wise Adagrad
// (src/optim.py:31-62).
//
// Every rank's table shards live in one fp32 slab. With one rank a lookup is ONE
// kernel (emb_pool_fwd_kernel): each warp walks its bags, computes the table row
// (the reference's EmbeddingShardSpec owner/local-row mapping, kept
// bit-compatible for checkpoints), pools the rows in registers and stores bf16
// into the tokenizer GEMM's input layout; its backward pushes each id's gradient
// into the grad slab and marks the row in the touched-row byte flags.
//
// With several ranks every random row access stays local (owner-push): random
// peer reads over NVLink are dominated by address translation and latency.
// emb_route_kernel groups this rank's bags into per-(bag, owner) bundles in its
// own peer-visible staging; after a device barrier emb_owner_fwd_kernel (on each
// owner) gathers and pools the rows of the bundles routed to it from local HBM and
// adds one pooled fp32 vector per bundle into the requester's accumulator with
// vector reductions over NVLink; acc_to_bf16_kernel converts the accumulator. In
// the backward emb_owner_bwd_kernel reads each bundle's bf16 output-gradient slice
// from the requester once and adds it into the owner's local gradient rows,
// marking them touched. The owner then compacts its touched rows and applies
// row-wise Adagrad to exactly those rows.
#include "common.cuh"
#include "embedding.h"

namespace mdl {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ long long find_feature(const long long* prefix, int nf, long long w) {
  int lo = 0, hi = nf;  // find f with prefix[f] <= w < prefix[f+1]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(prefix + mid) <= w) lo = mid; else hi = mid;
  }
  return lo;
}

__device__ __forceinline__ long long hash_id(long long v, int mode, long long buckets) {
  if (mode == 1) {
    if (v == 0) return 0;  // null -> padding
    return static_cast<long long>(static_cast<unsigned long long>(v) & static_cast<unsigned long long>(buckets - 1)) + 1;
  }
  return v;
}

__device__ __forceinline__ long long phys_col(int c, int slice, int stride) {
  return slice > 0 ? static_cast<long long>(c / slice) * stride + (c % slice) : c;
}

template <bool SYS>
__device__ __forceinline__ void red_add4(float* dst, const float* v) {
  if (SYS) {
    asm volatile("red.relaxed.sys.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(dst), "f"(v[0]), "f"(v[1]),
                 "f"(v[2]), "f"(v[3])
                 : "memory");
  } else {
    asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(dst), "f"(v[0]), "f"(v[1]),
                 "f"(v[2]), "f"(v[3])
                 : "memory");
  }
}

constexpr int kChunkBags = 32;  // bags per warp work item (all 32 lanes hold one bag's offsets)

// Everything a warp needs about its work item, loaded once per warp.
struct Chunk {
  int f = 0, t = -1, pool = 0, hmode = 0, width = 0, dim = 0, lanes = 1, lg = 0;
  long long buckets = 1, rows = 0;
  long long first = 0;  // first bag (sample row) of the chunk within the feature
  int nb = 0;           // bags in the chunk (<= 32)
  long long g0 = 0;     // CSR index of the chunk's first bag
  // output columns: logical c0 + col -> physical p0 + col (+ delta past `split`)
  long long out_base = 0, out_ld = 0;
  int p0 = 0, split = 1 << 30, delta = 0;
  bool general = false;  // more than one slice boundary inside the feature: per-column mapping
  int c0 = 0, slice = 0, sstride = 0;
  const float* tbl = nullptr;  // this rank's shard of the table (single-rank fast path)
  float* gtbl = nullptr;       // ... and of its gradient
  unsigned char* ftbl = nullptr;  // ... and of its touched flags
};

__device__ __forceinline__ Chunk load_chunk(const EmbPlan& p, long long warp) {
  Chunk c;
  c.f = static_cast<int>(find_feature(p.f_chunk_prefix, p.num_features, warp));
  const int f = c.f;
  c.t = __ldg(p.f_table + f);
  c.pool = __ldg(p.f_pool + f);
  c.hmode = __ldg(p.f_hash + f);
  c.buckets = __ldg(p.f_buckets + f);
  c.width = __ldg(p.f_width + f);
  c.lanes = __ldg(p.f_lanes + f);
  c.lg = __ffs(c.lanes) - 1;
  if (c.t >= 0) {
    c.rows = __ldg(p.t_rows + c.t);
    c.dim = __ldg(p.t_dim + c.t);
    const long long tb = __ldg(p.t_base_all + p.rank * p.num_tables + c.t);
    c.tbl = p.slabs[p.rank] + tb;
    if (p.grad_slabs[p.rank] != nullptr) c.gtbl = p.grad_slabs[p.rank] + tb;
    if (p.flags[p.rank] != nullptr) c.ftbl = p.flags[p.rank] + __ldg(p.t_row_base_all + p.rank * p.num_tables + c.t);
  }
  c.first = (warp - __ldg(p.f_chunk_prefix + f)) * kChunkBags;
  const long long n_bags = __ldg(p.f_bag_prefix + f + 1) - __ldg(p.f_bag_prefix + f);
  const long long left = n_bags - c.first;
  c.nb = static_cast<int>(left < kChunkBags ? (left > 0 ? left : 0) : kChunkBags);
  c.g0 = __ldg(p.f_src_bag + f) + c.first;
  c.out_base = __ldg(p.f_out_base + f);
  c.out_ld = __ldg(p.f_out_ld + f);
  c.c0 = __ldg(p.f_out_col + f);
  c.slice = __ldg(p.f_slice + f);
  c.sstride = __ldg(p.f_slice_stride + f);
  if (c.slice > 0) {
    const int r = c.c0 % c.slice;
    c.p0 = (c.c0 / c.slice) * c.sstride + r;
    c.split = c.slice - r;
    c.delta = c.sstride - c.slice;
    c.general = c.width > c.split + c.slice;
  } else {
    c.p0 = c.c0;
  }
  return c;
}

// Physical output column of feature column `col`.
__device__ __forceinline__ long long out_col(const Chunk& c, int col) {
  if (c.general) return phys_col(c.c0 + col, c.slice, c.sstride);
  return c.p0 + col + (col >= c.split ? c.delta : 0);
}

__device__ __forceinline__ void store4(const Chunk& c, __nv_bfloat16* out, long long row_off, int col, int valid,
                                       const float* v) {
  const long long p0 = out_col(c, col);
  const bool contiguous = !c.general && ((col < c.split) == (col + 3 < c.split));
  if (valid == 4 && contiguous && ((row_off + p0) & 3) == 0) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
    const __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(out + row_off + p0) = u;
  } else {
    for (int j = 0; j < valid; ++j) out[row_off + out_col(c, col + j)] = __float2bfloat16_rn(v[j]);
  }
}

__device__ __forceinline__ void load4(const Chunk& c, const __nv_bfloat16* g, long long row_off, int col, int valid,
                                      float* v) {
  const long long p0 = out_col(c, col);
  const bool contiguous = !c.general && ((col < c.split) == (col + 3 < c.split));
  if (valid == 4 && contiguous && ((row_off + p0) & 3) == 0) {
    const uint2 u = *reinterpret_cast<const uint2*>(g + row_off + p0);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  } else {
    for (int j = 0; j < 4; ++j) v[j] = j < valid ? __bfloat162float(g[row_off + out_col(c, col + j)]) : 0.f;
  }
}

__device__ __forceinline__ void route(const EmbPlan& p, int t, long long id, int& owner, long long& row) {
  if (__ldg(p.t_mode + t) != 0) {
    owner = __ldg(p.t_owner + t);
    row = id;
  } else if (p.world == 1) {
    owner = 0;
    row = id;
  } else {
    const long long cyc = __ldg(p.t_cyc + t);
    if (id < (1LL << 31) && cyc < (1LL << 31)) {  // 32-bit division is several times cheaper
      const unsigned w = static_cast<unsigned>(p.world);
      owner = static_cast<int>((static_cast<unsigned>(id) + static_cast<unsigned>(cyc)) % w);
      row = static_cast<long long>(static_cast<unsigned>(id) / w);
    } else {
      owner = static_cast<int>((id + cyc) % p.world);
      row = id / p.world;
    }
  }
}

// CSR range [beg, end) of bag `lane` of the chunk (lanes >= nb get an empty range).
__device__ __forceinline__ void bag_ranges(const long long* offs, const Chunk& c, int lane, long long& beg,
                                           long long& end) {
  beg = lane < c.nb ? offs[c.g0 + lane] : 0;
  end = __shfl_down_sync(0xffffffffu, beg, 1);
  if (lane == c.nb - 1) end = offs[c.g0 + c.nb];
  if (lane >= c.nb) end = beg;
}

// First valid id of the bag (single-valued features), 0 when none; records bad ids.
__device__ __forceinline__ long long first_valid(const EmbPlan& p, const long long* ids, const Chunk& c,
                                                 long long beg, long long end) {
  for (long long q = beg; q < end; ++q) {
    const long long id = hash_id(ids[q], c.hmode, c.buckets);
    if (id <= 0) continue;  // null / padding
    if (id >= c.rows) {
      record_error(p.err, MDL_ERR_BAD_INDEX);
      continue;
    }
    return id;
  }
  return 0;
}

// Source row of `id`: the local shard directly when this is the only rank
// (64-bit IMAD on an unsigned id), else the owner's slab (peer memory).
template <bool LOCAL>
__device__ __forceinline__ const float* row_src(const EmbPlan& p, const Chunk& c, long long id) {
  if (LOCAL) return c.tbl + static_cast<unsigned long long>(id) * static_cast<unsigned>(c.dim);
  int owner;
  long long row;
  route(p, c.t, id, owner, row);
  return p.slabs[owner] + __ldg(p.t_base_all + owner * p.num_tables + c.t) + row * c.dim;
}

template <int NV, bool LOCAL>  // float4 vectors per lane: width <= 4 * lanes * NV
__global__ void __launch_bounds__(kThreads, NV <= 2 ? 4 : 2) emb_pool_fwd_kernel(const EmbPlan p, long long total_chunks) {
  const long long warp = (static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  if (warp >= total_chunks) return;
  const int lane = threadIdx.x & 31;
  const Chunk c = load_chunk(p, warp);
  if (c.nb <= 0) return;
  const int sub = lane >> c.lg, sl = lane & (c.lanes - 1);
  const int bps = 32 >> c.lg;  // bags per step
  const int stride_cols = 4 * c.lanes;
  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out) + c.out_base;
  if (c.t < 0) {  // dense input columns
    const int dcol = __ldg(p.f_dense_col + c.f);
    for (int s = 0; s * bps < c.nb; ++s) {
      const int bag = s * bps + sub;
      if (bag >= c.nb) continue;
      const long long brow = c.first + bag;
      const float* src = p.dense + brow * p.dense_ld + dcol;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int col = sl * 4 + i * stride_cols;
        if (col < c.width) {
          float v[4];
          for (int j = 0; j < 4; ++j) v[j] = (col + j < c.width) ? __ldg(src + col + j) : 0.f;
          store4(c, out, brow * c.out_ld, col, min(4, c.width - col), v);
        }
      }
    }
    return;
  }
  long long beg, end;
  bag_ranges(p.id_offsets, c, lane, beg, end);
  if (c.pool == 0) {
    // one id per bag, found by the bag's own lane; lane groups then fetch the rows
    const long long my_id = first_valid(p, p.ids, c, beg, end);
    for (int s0 = 0; s0 * bps < c.nb; s0 += 2) {
      float v[2][NV][4];
      long long brow[2];
      bool ok[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int bag = (s0 + u) * bps + sub;
        const long long id = __shfl_sync(0xffffffffu, my_id, bag & 31);
        ok[u] = bag < c.nb;
        brow[u] = c.first + bag;
        const float* src = (ok[u] && id > 0) ? row_src<LOCAL>(p, c, id) : nullptr;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const int col = sl * 4 + i * stride_cols;
          float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
          if (src != nullptr && col < c.dim) x = *reinterpret_cast<const float4*>(src + col);
          v[u][i][0] = x.x; v[u][i][1] = x.y; v[u][i][2] = x.z; v[u][i][3] = x.w;
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (!ok[u]) continue;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const int col = sl * 4 + i * stride_cols;
          if (col < c.width) store4(c, out, brow[u] * c.out_ld, col, min(4, c.width - col), v[u][i]);
        }
      }
    }
    return;
  }
  // bags (sum / mean): each lane group walks its bag four ids at a time
  for (int s = 0; s * bps < c.nb; ++s) {
    const int bag = s * bps + sub;
    const long long qb = __shfl_sync(0xffffffffu, beg, bag & 31);
    const long long qe = __shfl_sync(0xffffffffu, end, bag & 31);
    if (bag >= c.nb) continue;
    float acc[NV][4];
#pragma unroll
    for (int i = 0; i < NV; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    int count = 0;
    for (long long q = qb; q < qe; q += 4) {
      long long id[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) id[u] = q + u < qe ? hash_id(__ldg(p.ids + q + u), c.hmode, c.buckets) : 0;
      float4 x[4][NV];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const bool bad = id[u] >= c.rows;
        if (bad) record_error(p.err, MDL_ERR_BAD_INDEX);
        const float* src = nullptr;
        if (id[u] > 0 && !bad) {
          src = row_src<LOCAL>(p, c, id[u]);
          ++count;
        }
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const int col = sl * 4 + i * stride_cols;
          x[u][i] = (src != nullptr && col < c.dim) ? *reinterpret_cast<const float4*>(src + col)
                                                    : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          acc[i][0] += x[u][i].x; acc[i][1] += x[u][i].y; acc[i][2] += x[u][i].z; acc[i][3] += x[u][i].w;
        }
    }
    if (c.pool == 1 && count > 0) {
      const float inv = 1.f / static_cast<float>(count);
#pragma unroll
      for (int i = 0; i < NV; ++i)
        for (int j = 0; j < 4; ++j) acc[i][j] *= inv;
    }
    const long long brow = c.first + bag;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int col = sl * 4 + i * stride_cols;
      if (col < c.width) store4(c, out, brow * c.out_ld, col, min(4, c.width - col), acc[i]);
    }
  }
}

template <bool SYS, int NV, bool LOCAL>
__global__ void __launch_bounds__(kThreads, NV <= 2 ? 4 : 2)
    emb_pool_bwd_kernel(const EmbPlan p, const __nv_bfloat16* __restrict__ grad_out, long long total_chunks) {
  const long long warp = (static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  if (warp >= total_chunks) return;
  const int lane = threadIdx.x & 31;
  const Chunk c = load_chunk(p, warp);
  if (c.nb <= 0 || c.t < 0) return;  // dense inputs have no trainable table
  const int sub = lane >> c.lg, sl = lane & (c.lanes - 1);
  const int bps = 32 >> c.lg;
  const int stride_cols = 4 * c.lanes;
  const __nv_bfloat16* gbase = grad_out + c.out_base;
  long long beg, end;
  bag_ranges(p.id_offsets, c, lane, beg, end);
  // per bag (own lane): the single id (pool none) or the valid-id count (mean)
  long long my_id = 0;
  int my_count = 0;
  if (c.pool == 0) {
    my_id = first_valid(p, p.ids, c, beg, end);
  } else if (c.pool == 1) {
    for (long long q = beg; q < end; ++q) {
      const long long id = hash_id(__ldg(p.ids + q), c.hmode, c.buckets);
      if (id > 0 && id < c.rows) ++my_count;
    }
  }
  for (int s = 0; s * bps < c.nb; ++s) {
    const int bag = s * bps + sub;
    const long long qb = __shfl_sync(0xffffffffu, beg, bag & 31);
    const long long qe = __shfl_sync(0xffffffffu, end, bag & 31);
    const long long one = __shfl_sync(0xffffffffu, my_id, bag & 31);
    const int cnt = __shfl_sync(0xffffffffu, my_count, bag & 31);
    if (bag >= c.nb) continue;
    if (c.pool == 0 && one <= 0) continue;
    if (c.pool == 1 && cnt == 0) continue;
    const float scale = c.pool == 1 ? 1.f / static_cast<float>(cnt) : 1.f;
    const long long brow = c.first + bag;
    float g[NV][4];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int col = sl * 4 + i * stride_cols;
      if (col < c.dim) {
        load4(c, gbase, brow * c.out_ld, col, min(4, c.dim - col), g[i]);
        for (int j = 0; j < 4; ++j) g[i][j] *= scale;
      }
    }
    auto push = [&](long long id) {
      float* dst;
      unsigned char* flag;
      if (LOCAL) {
        dst = c.gtbl + static_cast<unsigned long long>(id) * static_cast<unsigned>(c.dim);
        flag = c.ftbl + id;
      } else {
        int owner;
        long long row;
        route(p, c.t, id, owner, row);
        dst = p.grad_slabs[owner] + __ldg(p.t_base_all + owner * p.num_tables + c.t) + row * c.dim;
        flag = p.flags[owner] + __ldg(p.t_row_base_all + owner * p.num_tables + c.t) + row;
      }
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int col = sl * 4 + i * stride_cols;
        if (col < c.dim) red_add4<SYS>(dst + col, g[i]);
      }
      // Mark the row touched: an idempotent byte store (no atomic, no shared counter).
      if (sl == 0) *reinterpret_cast<volatile unsigned char*>(flag) = 1;
    };
    if (c.pool == 0) {
      push(one);
      continue;
    }
    for (long long q = qb; q < qe; q += 4) {
      long long id[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) id[u] = q + u < qe ? hash_id(__ldg(p.ids + q + u), c.hmode, c.buckets) : 0;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (id[u] > 0 && id[u] < c.rows) push(id[u]);
    }
  }
}

// ---- owner-push kernels (multi-rank) -----------------------------------------
// Physical output column of column `col` of feature f (host-computed phys0/split;
// split < 0 marks a feature that crosses several token slices).
__device__ __forceinline__ long long feat_col(const EmbPlan& p, int f, int col) {
  const int split = __ldg(p.f_split + f);
  if (split < 0) return phys_col(__ldg(p.f_out_col + f) + col, __ldg(p.f_slice + f), __ldg(p.f_slice_stride + f));
  return __ldg(p.f_phys0 + f) + col + (col >= split ? __ldg(p.f_slice_stride + f) - __ldg(p.f_slice + f) : 0);
}

__device__ __forceinline__ bool feat_vec4(const EmbPlan& p, int f, int col, long long addr) {
  const int split = __ldg(p.f_split + f);
  return split >= 0 && ((col < split) == (col + 3 < split)) && (addr & 3) == 0;
}

// Route pass of this rank: lane = bag. Per (bag, owner) one bundle; rows of
// multi-row bundles go to the owner's row list, contiguous per bundle.
__global__ void __launch_bounds__(kThreads) emb_route_kernel(const EmbPlan p, const OwnerArgs o,
                                                            long long total_chunks) {
  const long long warp = (static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  if (warp >= total_chunks) return;
  const int lane = threadIdx.x & 31;
  const Chunk c = load_chunk(p, warp);
  if (c.nb <= 0) return;
  if (c.t < 0) {  // dense inputs: copied into this rank's own accumulator
    float* acc = o.acc[p.rank] + c.out_base;
    const int dcol = __ldg(p.f_dense_col + c.f);
    const int sub = lane >> c.lg, sl = lane & (c.lanes - 1);
    const int bps = 32 >> c.lg;
    for (int s = 0; s * bps < c.nb; ++s) {
      const int bag = s * bps + sub;
      if (bag >= c.nb) continue;
      const long long brow = c.first + bag;
      const float* src = o.dense + brow * o.dense_ld + dcol;
      for (int col = sl * 4; col < c.width; col += 4 * c.lanes)
        for (int j = 0; j < 4 && col + j < c.width; ++j)
          acc[brow * c.out_ld + out_col(c, col + j)] = __ldg(src + col + j);
    }
    return;
  }
  const int W = p.world;
  long long beg, end;
  bag_ranges(p.id_offsets, c, lane, beg, end);
  // per owner: rows of this lane's bag and the last one seen (registers: the owner
  // index is only ever compared against compile-time constants)
  int cnt[kMaxWorld], last[kMaxWorld];
#pragma unroll
  for (int j = 0; j < kMaxWorld; ++j) cnt[j] = last[j] = 0;
  int valid = 0;
  auto note = [&](long long id) {
    int owner;
    long long row;
    route(p, c.t, id, owner, row);
#pragma unroll
    for (int j = 0; j < kMaxWorld; ++j) {
      if (j == owner) {
        ++cnt[j];
        last[j] = static_cast<int>(row);
      }
    }
    ++valid;
  };
  if (c.pool == 0) {
    const long long id = first_valid(p, p.ids, c, beg, end);
    if (id > 0) note(id);
  } else {
    for (long long q = beg; q < end; ++q) {
      const long long id = hash_id(__ldg(p.ids + q), c.hmode, c.buckets);
      if (id <= 0) continue;
      if (id >= c.rows) {
        record_error(p.err, MDL_ERR_BAD_INDEX);
        continue;
      }
      note(id);
    }
  }
  const float scale = (c.pool == 1 && valid > 0) ? 1.f / static_cast<float>(valid) : 1.f;
  // allocate bundles and row-list slots owner by owner (warp-aggregated atomics)
  int row_start[kMaxWorld];
  bool need_rows = false;
  const unsigned lt = (1u << lane) - 1u;
#pragma unroll
  for (int j = 0; j < kMaxWorld; ++j) {
    row_start[j] = 0;
    if (j >= W) continue;
    const int k = cnt[j];
    const unsigned want = __ballot_sync(0xffffffffu, k > 0);
    if (want == 0) continue;
    const int multi = k > 1 ? k : 0;  // rows that go to the row list
    int incl = multi;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += y;
    }
    const int total_rows = __shfl_sync(0xffffffffu, incl, 31);
    int bbase = 0, rbase = 0;
    if (lane == 0) {
      bbase = atomicAdd(o.counts[p.rank] + 2 * j, __popc(want));
      if (total_rows > 0) rbase = atomicAdd(o.counts[p.rank] + 2 * j + 1, total_rows);
    }
    bbase = __shfl_sync(0xffffffffu, bbase, 0);
    rbase = __shfl_sync(0xffffffffu, rbase, 0);
    if (k > 0) {
      const long long bi = bbase + __popc(want & lt);
      row_start[j] = rbase + incl - multi;
      if (bi < o.cap_bundles && (multi == 0 || row_start[j] + multi <= o.cap_rows)) {
        RouteBundle b;
        b.bag = static_cast<int>(c.first + lane);
        b.f_count = c.f | (k << 16);
        b.row = k == 1 ? last[j] : row_start[j];
        b.scale = scale;
        o.bundles[p.rank][j * o.cap_bundles + bi] = b;
        need_rows |= multi > 0;
      } else {
        record_error(p.err, MDL_ERR_CAPACITY);
        cnt[j] = 0;  // nothing of this bag reaches owner j
      }
    }
  }
  if (!need_rows) return;
  // second pass: rows of multi-row bundles, in bag order
  int fill[kMaxWorld];
#pragma unroll
  for (int j = 0; j < kMaxWorld; ++j) fill[j] = 0;
  for (long long q = beg; q < end; ++q) {
    const long long id = hash_id(__ldg(p.ids + q), c.hmode, c.buckets);
    if (id <= 0 || id >= c.rows) continue;
    int owner;
    long long row;
    route(p, c.t, id, owner, row);
#pragma unroll
    for (int j = 0; j < kMaxWorld; ++j) {
      if (j == owner && cnt[j] > 1) {
        o.rows[p.rank][j * o.cap_rows + row_start[j] + fill[j]] = static_cast<int>(row);
        ++fill[j];
      }
    }
  }
}

// Owner side, forward: one group of 16 lanes per bundle (two in flight): gather and
// sum the bundle's rows from the local shard, scale, add the pooled vector into the
// requester's accumulator.
template <int NV>
__global__ void __launch_bounds__(kThreads) emb_owner_fwd_kernel(const EmbPlan p, const OwnerArgs o) {
  constexpr int G = 16;
  const int sub = threadIdx.x % G;
  const long long gid = (static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x) / G;
  const long long ngroups = static_cast<long long>(gridDim.x) * kThreads / G;
  const float* slab = p.slabs[p.rank];
  for (int r = 0; r < p.world; ++r) {
    const long long n = min(static_cast<long long>(o.counts[r][2 * p.rank]), o.cap_bundles);
    const RouteBundle* seg = o.bundles[r] + p.rank * o.cap_bundles;
    const int* rl = o.rows[r] + p.rank * o.cap_rows;
    float* acc = o.acc[r];
    for (long long e0 = gid; e0 < n; e0 += 2 * ngroups) {
      RouteBundle bd[2];
      bool ok[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const long long e = e0 + u * ngroups;
        ok[u] = e < n;
        if (ok[u]) bd[u] = seg[e];
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (!ok[u]) continue;
        const int f = bd[u].f_count & 0xffff, k = bd[u].f_count >> 16;
        const int t = __ldg(p.f_table + f);
        const int dim = __ldg(p.t_dim + t);
        const float* tbl = slab + __ldg(p.t_base_all + p.rank * p.num_tables + t);
        float sum[NV][4];
#pragma unroll
        for (int i = 0; i < NV; ++i) sum[i][0] = sum[i][1] = sum[i][2] = sum[i][3] = 0.f;
        for (int q = 0; q < k; q += 4) {
          int rows[4];
#pragma unroll
          for (int v = 0; v < 4; ++v) rows[v] = q + v < k ? (k == 1 ? bd[u].row : rl[bd[u].row + q + v]) : -1;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            if (rows[v] < 0) continue;
            const float* src = tbl + static_cast<long long>(rows[v]) * dim;
#pragma unroll
            for (int i = 0; i < NV; ++i) {
              const int col = (sub + i * G) * 4;
              if (col < dim) {
                const float4 x = *reinterpret_cast<const float4*>(src + col);
                sum[i][0] += x.x; sum[i][1] += x.y; sum[i][2] += x.z; sum[i][3] += x.w;
              }
            }
          }
        }
        const long long row_off = __ldg(p.f_out_base + f) + static_cast<long long>(bd[u].bag) * __ldg(p.f_out_ld + f);
        const int width = __ldg(p.f_width + f);
        const float sc = bd[u].scale;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const int col = (sub + i * G) * 4;
          if (col >= width) continue;
          const float v[4] = {sum[i][0] * sc, sum[i][1] * sc, sum[i][2] * sc, sum[i][3] * sc};
          const long long a = row_off + feat_col(p, f, col);
          if (col + 4 <= width && feat_vec4(p, f, col, a)) {
            red_add4<true>(acc + a, v);
          } else {
            for (int j = 0; j < 4 && col + j < width; ++j) atomicAdd(acc + row_off + feat_col(p, f, col + j), v[j]);
          }
        }
      }
    }
  }
}

// Owner side, backward: per bundle read the requester's bf16 gradient slice of the
// bag once and add it into every row of the bundle (local), marking them touched.
template <int NV>
__global__ void __launch_bounds__(kThreads) emb_owner_bwd_kernel(const EmbPlan p, const OwnerArgs o) {
  constexpr int G = 16;
  const int sub = threadIdx.x % G;
  const long long gid = (static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x) / G;
  const long long ngroups = static_cast<long long>(gridDim.x) * kThreads / G;
  float* gslab = p.grad_slabs[p.rank];
  unsigned char* flags = p.flags[p.rank];
  for (int r = 0; r < p.world; ++r) {
    const long long n = min(static_cast<long long>(o.counts[r][2 * p.rank]), o.cap_bundles);
    const RouteBundle* seg = o.bundles[r] + p.rank * o.cap_bundles;
    const int* rl = o.rows[r] + p.rank * o.cap_rows;
    const __nv_bfloat16* grad = reinterpret_cast<const __nv_bfloat16*>(o.grad[r]);
    for (long long e0 = gid; e0 < n; e0 += 2 * ngroups) {
      RouteBundle bd[2];
      bool ok[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const long long e = e0 + u * ngroups;
        ok[u] = e < n;
        if (ok[u]) bd[u] = seg[e];
      }
      float g[2][NV][4];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (!ok[u]) continue;
        const int f = bd[u].f_count & 0xffff;
        const long long row_off = __ldg(p.f_out_base + f) + static_cast<long long>(bd[u].bag) * __ldg(p.f_out_ld + f);
        const int width = __ldg(p.f_width + f);
        const float sc = bd[u].scale;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
          const int col = (sub + i * G) * 4;
          g[u][i][0] = g[u][i][1] = g[u][i][2] = g[u][i][3] = 0.f;
          if (col >= width) continue;
          const long long a = row_off + feat_col(p, f, col);
          if (col + 4 <= width && feat_vec4(p, f, col, a)) {
            const uint2 w = *reinterpret_cast<const uint2*>(grad + a);
            const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.x));
            const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w.y));
            g[u][i][0] = lo.x * sc; g[u][i][1] = lo.y * sc; g[u][i][2] = hi.x * sc; g[u][i][3] = hi.y * sc;
          } else {
            for (int j = 0; j < 4 && col + j < width; ++j)
              g[u][i][j] = __bfloat162float(grad[row_off + feat_col(p, f, col + j)]) * sc;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (!ok[u]) continue;
        const int f = bd[u].f_count & 0xffff, k = bd[u].f_count >> 16;
        const int t = __ldg(p.f_table + f);
        const int dim = __ldg(p.t_dim + t);
        float* tbl = gslab + __ldg(p.t_base_all + p.rank * p.num_tables + t);
        unsigned char* ftbl = flags + __ldg(p.t_row_base_all + p.rank * p.num_tables + t);
        for (int q = 0; q < k; ++q) {
          const long long row = k == 1 ? bd[u].row : rl[bd[u].row + q];
#pragma unroll
          for (int i = 0; i < NV; ++i) {
            const int col = (sub + i * G) * 4;
            if (col < dim) red_add4<false>(tbl + row * dim + col, g[u][i]);
          }
          if (sub == 0) *reinterpret_cast<volatile unsigned char*>(ftbl + row) = 1;
        }
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads) acc_to_bf16_kernel(const float* __restrict__ acc, __nv_bfloat16* out,
                                                               long long n8) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 a = reinterpret_cast<const float4*>(acc)[2 * i];
    const float4 b = reinterpret_cast<const float4*>(acc)[2 * i + 1];
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
    h[0] = __floats2bfloat162_rn(a.x, a.y);
    h[1] = __floats2bfloat162_rn(a.z, a.w);
    h[2] = __floats2bfloat162_rn(b.x, b.y);
    h[3] = __floats2bfloat162_rn(b.z, b.w);
    reinterpret_cast<uint4*>(out)[i] = u;
  }
}

// Walk the touched-row byte flags of this rank in warp-sized chunks of 512 rows
// (each lane tests 16 flags with one 16-byte load) and call `fn(rs)` with the
// whole warp for every touched row-space index, in ballot order.
template <typename F>
__device__ __forceinline__ void for_each_touched(const AdagradArgs& a, F&& fn) {
  const int lane = threadIdx.x & 31;
  const long long nwarps = static_cast<long long>(gridDim.x) * (blockDim.x / 32);
  const long long nchunks = (a.total_rows + 511) / 512;
  for (long long chunk = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; chunk < nchunks;
       chunk += nwarps) {
    const uint4 f = *reinterpret_cast<const uint4*>(a.flags + chunk * 512 + lane * 16);
    unsigned mask = 0;
    const unsigned words[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
    for (int w = 0; w < 4; ++w)
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if ((words[w] >> (8 * k)) & 0xffu) mask |= 1u << (4 * w + k);
    while (true) {
      const unsigned ballot = __ballot_sync(0xffffffffu, mask != 0);
      if (ballot == 0) break;
      const int src = __ffs(ballot) - 1;
      const unsigned m = __shfl_sync(0xffffffffu, mask, src);
      const int bit = __ffs(m) - 1;
      if (lane == src) mask &= ~(1u << bit);
      fn(chunk * 512 + src * 16 + bit);
    }
  }
}

// Table of a row-space index (warp-uniform binary search over t_row_base).
__device__ __forceinline__ int table_of_row(const AdagradArgs& a, long long rs) {
  int lo = 0, hi = a.num_tables;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(a.t_row_base + mid) <= rs) lo = mid; else hi = mid;
  }
  return lo;
}

template <int NV>  // dim <= 128 * NV
__global__ void __launch_bounds__(kThreads) rowwise_adagrad_kernel(const AdagradArgs a) {
  const int lane = threadIdx.x & 31;
  const float clip = a.clip_scale != nullptr ? *a.clip_scale : 1.f;
  const float gscale = a.grad_scale * clip;
  for_each_touched(a, [&](long long rs) {
    const int t = table_of_row(a, rs);
    const long long row = rs - __ldg(a.t_row_base + t);
    const int dim = __ldg(a.t_dim + t);
    const long long base = __ldg(a.t_base + t) + row * dim;
    float g[NV][4];
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int col = lane * 4 + i * 128;
      if (col < dim) {
        const float4 v = *reinterpret_cast<const float4*>(a.grad_slab + base + col);
        g[i][0] = v.x * gscale; g[i][1] = v.y * gscale; g[i][2] = v.z * gscale; g[i][3] = v.w * gscale;
        sq += g[i][0] * g[i][0] + g[i][1] * g[i][1] + g[i][2] * g[i][2] + g[i][3] * g[i][3];
      }
    }
    sq = warp_sum(sq);
    float acc = 0.f;
    if (lane == 0) {
      acc = a.acc[rs] + sq / static_cast<float>(dim);
      a.acc[rs] = acc;
      a.flags[rs] = 0;
    }
    acc = __shfl_sync(0xffffffffu, acc, 0);
    const float step = a.lr / (sqrtf(acc) + a.eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int col = lane * 4 + i * 128;
      if (col < dim) {
        float4* w = reinterpret_cast<float4*>(a.slab + base + col);
        float4 v = *w;
        v.x -= step * g[i][0]; v.y -= step * g[i][1]; v.z -= step * g[i][2]; v.w -= step * g[i][3];
        *w = v;
        *reinterpret_cast<float4*>(a.grad_slab + base + col) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  });
}

// Thread-per-row variant for narrow tables (dim <= 128): each thread tests 16
// flags with one coalesced 16-byte load and updates its own touched rows, so
// all touched rows of a warp are in flight at once. Table row bases are staged
// in shared memory for the row -> table search.
__global__ void __launch_bounds__(kThreads) rowwise_adagrad_thread_kernel(const AdagradArgs a) {
  extern __shared__ long long s_rb[];
  const bool staged = a.num_tables <= 4096;
  if (staged)
    for (int i = threadIdx.x; i < a.num_tables; i += blockDim.x) s_rb[i] = __ldg(a.t_row_base + i);
  __syncthreads();
  const float clip = a.clip_scale != nullptr ? *a.clip_scale : 1.f;
  const float gscale = a.grad_scale * clip;
  const long long n16 = (a.total_rows + 15) / 16;
  uint4* flags16 = reinterpret_cast<uint4*>(a.flags);
  for (long long c = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; c < n16;
       c += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint4 f = flags16[c];
    if ((f.x | f.y | f.z | f.w) == 0u) continue;
    const unsigned words[4] = {f.x, f.y, f.z, f.w};
    for (int k = 0; k < 16; ++k) {
      if (((words[k >> 2] >> (8 * (k & 3))) & 0xffu) == 0u) continue;
      const long long rs = c * 16 + k;
      int lo = 0, hi = a.num_tables;
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        const long long v = staged ? s_rb[mid] : __ldg(a.t_row_base + mid);
        if (v <= rs) lo = mid; else hi = mid;
      }
      const int t = lo;
      const long long row = rs - (staged ? s_rb[t] : __ldg(a.t_row_base + t));
      const int dim = __ldg(a.t_dim + t);
      const long long base = __ldg(a.t_base + t) + row * dim;
      float sq = 0.f;
      for (int col = 0; col < dim; col += 4) {
        const float4 v = *reinterpret_cast<const float4*>(a.grad_slab + base + col);
        sq += (v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w) * gscale * gscale;
      }
      const float acc = a.acc[rs] + sq / static_cast<float>(dim);
      a.acc[rs] = acc;
      const float step = a.lr / (sqrtf(acc) + a.eps);
      for (int col = 0; col < dim; col += 4) {
        float4* gp = reinterpret_cast<float4*>(a.grad_slab + base + col);
        const float4 g = *gp;
        float4* w = reinterpret_cast<float4*>(a.slab + base + col);
        float4 v = *w;
        v.x -= step * g.x * gscale; v.y -= step * g.y * gscale; v.z -= step * g.z * gscale; v.w -= step * g.w * gscale;
        *w = v;
        *gp = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    flags16[c] = make_uint4(0u, 0u, 0u, 0u);
  }
}

// ---- touched-row list: compaction, then a coalesced update per row ----------
__global__ void __launch_bounds__(kThreads) compact_touched_kernel(const AdagradArgs a) {
  __shared__ unsigned s_warp[kThreads / 32];
  __shared__ unsigned s_base;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long n16 = (a.total_rows + 15) / 16;
  uint4* flags16 = reinterpret_cast<uint4*>(a.flags);
  for (long long base = static_cast<long long>(blockIdx.x) * blockDim.x; base < n16;
       base += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long c = base + threadIdx.x;
    uint4 f = make_uint4(0u, 0u, 0u, 0u);
    if (c < n16) f = flags16[c];
    // one bit per touched row of this thread's 16
    unsigned bits = 0;
    const unsigned words[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
    for (int w = 0; w < 4; ++w)
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if ((words[w] >> (8 * k)) & 0xffu) bits |= 1u << (4 * w + k);
    const unsigned n = __popc(bits);
    // block-wide exclusive prefix sum of n
    unsigned incl = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned tot = 0;
      for (int w = 0; w < kThreads / 32; ++w) {
        const unsigned x = s_warp[w];
        s_warp[w] = tot;
        tot += x;
      }
      s_base = tot ? atomicAdd(a.count, tot) : 0u;
    }
    __syncthreads();
    unsigned pos = s_base + s_warp[warp] + incl - n;
    while (bits) {
      const int k = __ffs(bits) - 1;
      bits &= bits - 1;
      a.list[pos++] = static_cast<unsigned>(c * 16 + k);
    }
    if (n) flags16[c] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();  // s_warp / s_base are rewritten by the next iteration
  }
}

// Row of table t for a row-space index: binary search over the table row bases
// (staged in shared memory when they fit).
__device__ __forceinline__ int table_of(const long long* rb, int num_tables, long long rs) {
  int lo = 0, hi = num_tables;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (rb[mid] <= rs) lo = mid; else hi = mid;
  }
  return lo;
}

// G lanes per row (G in {8, 16, 32}), NV float4 per lane: dim <= 4 * G * NV.
template <int G, int NV, bool NORM>
__global__ void __launch_bounds__(kThreads) adagrad_list_kernel(const AdagradArgs a, float* out_sq) {
  extern __shared__ long long s_rb[];
  const bool staged = a.num_tables <= 4096;
  if (staged)
    for (int i = threadIdx.x; i < a.num_tables; i += blockDim.x) s_rb[i] = __ldg(a.t_row_base + i);
  __syncthreads();
  const long long* rb = staged ? s_rb : a.t_row_base;
  const float clip = (!NORM && a.clip_scale != nullptr) ? *a.clip_scale : 1.f;
  const float gscale = a.grad_scale * clip;
  const unsigned n = *a.count;
  const int sub = threadIdx.x % G;
  constexpr int RPW = 32 / G;  // rows per warp per iteration
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x / 32);
  float sq_total = 0.f;
  // Warp-uniform trip count: every lane reaches the group shuffles.
  for (long long i0 = ((static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * RPW; i0 < n;
       i0 += warps * RPW) {
    const long long i = i0 + (threadIdx.x & 31) / G;
    const bool valid = i < n;
    long long rs = 0, base = 0;
    int dim = 0;
    if (valid) {
      rs = a.list[i];
      const int t = table_of(rb, a.num_tables, rs);
      dim = __ldg(a.t_dim + t);
      base = __ldg(a.t_base + t) + (rs - rb[t]) * dim;
    }
    float4 g[NV];
    float sq = 0.f;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int col = (sub + v * G) * 4;
      g[v] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (col < dim) {
        const float4 x = *reinterpret_cast<const float4*>(a.grad_slab + base + col);
        g[v] = make_float4(x.x * gscale, x.y * gscale, x.z * gscale, x.w * gscale);
        sq += g[v].x * g[v].x + g[v].y * g[v].y + g[v].z * g[v].z + g[v].w * g[v].w;
      }
    }
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o, G);
    if (!valid) continue;
    if (NORM) {
      if (sub == 0) sq_total += sq;
      continue;
    }
    if (a.full) {  // per-element sums live at the weight's offsets
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const int col = (sub + v * G) * 4;
        if (col < dim) {
          float4* s4 = reinterpret_cast<float4*>(a.acc + base + col);
          float4* w = reinterpret_cast<float4*>(a.slab + base + col);
          float4 sacc = *s4, x = *w;
          sacc.x += g[v].x * g[v].x; sacc.y += g[v].y * g[v].y;
          sacc.z += g[v].z * g[v].z; sacc.w += g[v].w * g[v].w;
          x.x -= a.lr * g[v].x / (sqrtf(sacc.x) + a.eps);
          x.y -= a.lr * g[v].y / (sqrtf(sacc.y) + a.eps);
          x.z -= a.lr * g[v].z / (sqrtf(sacc.z) + a.eps);
          x.w -= a.lr * g[v].w / (sqrtf(sacc.w) + a.eps);
          *s4 = sacc;
          *w = x;
          *reinterpret_cast<float4*>(a.grad_slab + base + col) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      continue;
    }
    const float acc = a.acc[rs] + sq / static_cast<float>(dim);
    const float step = a.lr / (sqrtf(acc) + a.eps);
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int col = (sub + v * G) * 4;
      if (col < dim) {
        float4* w = reinterpret_cast<float4*>(a.slab + base + col);
        float4 x = *w;
        x.x -= step * g[v].x; x.y -= step * g[v].y; x.z -= step * g[v].z; x.w -= step * g[v].w;
        *w = x;
        *reinterpret_cast<float4*>(a.grad_slab + base + col) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    if (sub == 0) a.acc[rs] = acc;
  }
  if (NORM) {
    sq_total = warp_sum(sq_total);
    if ((threadIdx.x & 31) == 0 && sq_total != 0.f) atomicAdd(out_sq, sq_total);
  }
}

template <bool NORM>
cudaError_t launch_list(const AdagradArgs& a, float* out_sq, cudaStream_t stream) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = sms * 8;
  const size_t smem = a.num_tables <= 4096 ? static_cast<size_t>(a.num_tables) * sizeof(long long) : 0;
  if (a.max_dim <= 32) adagrad_list_kernel<8, 1, NORM><<<grid, kThreads, smem, stream>>>(a, out_sq);
  else if (a.max_dim <= 64) adagrad_list_kernel<16, 1, NORM><<<grid, kThreads, smem, stream>>>(a, out_sq);
  else if (a.max_dim <= 128) adagrad_list_kernel<32, 1, NORM><<<grid, kThreads, smem, stream>>>(a, out_sq);
  else if (a.max_dim <= 256) adagrad_list_kernel<32, 2, NORM><<<grid, kThreads, smem, stream>>>(a, out_sq);
  else if (a.max_dim <= 512) adagrad_list_kernel<32, 4, NORM><<<grid, kThreads, smem, stream>>>(a, out_sq);
  else if (a.max_dim <= 1024) adagrad_list_kernel<32, 8, NORM><<<grid, kThreads, smem, stream>>>(a, out_sq);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

__global__ void __launch_bounds__(kThreads) touched_sqnorm_kernel(const AdagradArgs a, float* out_sq) {
  const int lane = threadIdx.x & 31;
  float sq = 0.f;
  for_each_touched(a, [&](long long rs) {
    const int t = table_of_row(a, rs);
    const long long row = rs - __ldg(a.t_row_base + t);
    const int dim = __ldg(a.t_dim + t);
    const long long base = __ldg(a.t_base + t) + row * dim;
    for (int col = lane * 4; col < dim; col += 128) {
      const float4 v = *reinterpret_cast<const float4*>(a.grad_slab + base + col);
      sq += (v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w) * a.grad_scale * a.grad_scale;
    }
  });
  sq = warp_sum(sq);
  if (lane == 0) atomicAdd(out_sq, sq);
}

int blocks_for(long long warps) { return static_cast<int>((warps * 32 + kThreads - 1) / kThreads); }

int scan_grid(long long total_rows) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long want = blocks_for((total_rows + 511) / 512);
  return static_cast<int>(want < sms * 8 ? (want > 0 ? want : 1) : sms * 8);
}

}  // namespace

cudaError_t emb_pool_forward(const EmbPlan& plan, long long total_chunks, cudaStream_t stream) {
  if (total_chunks <= 0) return cudaSuccess;
  const int grid = blocks_for(total_chunks);
  const bool local = plan.world == 1;
#define MDL_FWD(NV)                                                                        \
  if (local) emb_pool_fwd_kernel<NV, true><<<grid, kThreads, 0, stream>>>(plan, total_chunks); \
  else emb_pool_fwd_kernel<NV, false><<<grid, kThreads, 0, stream>>>(plan, total_chunks);
  if (plan.max_vec <= 1) { MDL_FWD(1) } else if (plan.max_vec <= 2) { MDL_FWD(2) }
  else if (plan.max_vec <= 4) { MDL_FWD(4) } else { MDL_FWD(8) }
#undef MDL_FWD
  return cudaGetLastError();
}

cudaError_t emb_pool_backward(const EmbPlan& plan, const void* grad_out, long long total_chunks,
                              cudaStream_t stream) {
  if (total_chunks <= 0) return cudaSuccess;
  const auto* g = reinterpret_cast<const __nv_bfloat16*>(grad_out);
  const int grid = blocks_for(total_chunks);
#define MDL_BWD(SYS, NV, L) emb_pool_bwd_kernel<SYS, NV, L><<<grid, kThreads, 0, stream>>>(plan, g, total_chunks)
  const int nv = plan.max_vec <= 1 ? 1 : plan.max_vec <= 2 ? 2 : plan.max_vec <= 4 ? 4 : 8;
  if (plan.world > 1) {
    if (nv == 1) MDL_BWD(true, 1, false); else if (nv == 2) MDL_BWD(true, 2, false);
    else if (nv == 4) MDL_BWD(true, 4, false); else MDL_BWD(true, 8, false);
  } else {
    if (nv == 1) MDL_BWD(false, 1, true); else if (nv == 2) MDL_BWD(false, 2, true);
    else if (nv == 4) MDL_BWD(false, 4, true); else MDL_BWD(false, 8, true);
  }
#undef MDL_BWD
  return cudaGetLastError();
}

int owner_grid() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms * 8;
}

bool owner_args_ok(const EmbPlan& plan, const OwnerArgs& o) {
  if (o.cap_bundles <= 0 || o.cap_rows <= 0) return false;
  for (int r = 0; r < plan.world; ++r)
    if (o.bundles[r] == nullptr || o.rows[r] == nullptr || o.counts[r] == nullptr) return false;
  return true;
}

cudaError_t emb_route(const EmbPlan& plan, const OwnerArgs& o, long long total_chunks, cudaStream_t stream) {
  if (total_chunks <= 0) return cudaSuccess;
  if (!owner_args_ok(plan, o) || o.acc[plan.rank] == nullptr) return cudaErrorInvalidValue;
  emb_route_kernel<<<blocks_for(total_chunks), kThreads, 0, stream>>>(plan, o, total_chunks);
  return cudaGetLastError();
}

cudaError_t emb_owner_forward(const EmbPlan& plan, const OwnerArgs& o, cudaStream_t stream) {
  if (!owner_args_ok(plan, o)) return cudaErrorInvalidValue;
  for (int r = 0; r < plan.world; ++r)
    if (o.acc[r] == nullptr) return cudaErrorInvalidValue;
  const int grid = owner_grid();
  // NV float4 per lane of a 16-lane group: table dims <= 64 * NV
  if (plan.max_dim <= 64) emb_owner_fwd_kernel<1><<<grid, kThreads, 0, stream>>>(plan, o);
  else if (plan.max_dim <= 128) emb_owner_fwd_kernel<2><<<grid, kThreads, 0, stream>>>(plan, o);
  else if (plan.max_dim <= 256) emb_owner_fwd_kernel<4><<<grid, kThreads, 0, stream>>>(plan, o);
  else if (plan.max_dim <= 512) emb_owner_fwd_kernel<8><<<grid, kThreads, 0, stream>>>(plan, o);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t emb_owner_backward(const EmbPlan& plan, const OwnerArgs& o, cudaStream_t stream) {
  if (!owner_args_ok(plan, o)) return cudaErrorInvalidValue;
  for (int r = 0; r < plan.world; ++r)
    if (o.grad[r] == nullptr) return cudaErrorInvalidValue;
  if (plan.grad_slabs[plan.rank] == nullptr || plan.flags[plan.rank] == nullptr) return cudaErrorInvalidValue;
  const int grid = owner_grid();
  if (plan.max_dim <= 64) emb_owner_bwd_kernel<1><<<grid, kThreads, 0, stream>>>(plan, o);
  else if (plan.max_dim <= 128) emb_owner_bwd_kernel<2><<<grid, kThreads, 0, stream>>>(plan, o);
  else if (plan.max_dim <= 256) emb_owner_bwd_kernel<4><<<grid, kThreads, 0, stream>>>(plan, o);
  else if (plan.max_dim <= 512) emb_owner_bwd_kernel<8><<<grid, kThreads, 0, stream>>>(plan, o);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t emb_acc_to_bf16(const float* acc, void* out, long long n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  if ((n % 8) || (reinterpret_cast<uintptr_t>(acc) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long n8 = n / 8;
  const long long want = (n8 + kThreads - 1) / kThreads;
  const int grid = static_cast<int>(want < sms * 16 ? want : sms * 16);
  acc_to_bf16_kernel<<<grid, kThreads, 0, stream>>>(acc, reinterpret_cast<__nv_bfloat16*>(out), n8);
  return cudaGetLastError();
}

cudaError_t compact_touched(const AdagradArgs& a, cudaStream_t stream) {
  if (a.list == nullptr || a.count == nullptr) return cudaErrorInvalidValue;
  if (a.total_rows >= (1LL << 32)) return cudaErrorInvalidValue;  // list entries are 32-bit
  cudaError_t e = cudaMemsetAsync(a.count, 0, sizeof(unsigned), stream);
  if (e != cudaSuccess) return e;
  if (a.total_rows <= 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long want = ((a.total_rows + 15) / 16 + kThreads - 1) / kThreads;
  const int grid = static_cast<int>(want < sms * 8 ? (want > 0 ? want : 1) : sms * 8);
  compact_touched_kernel<<<grid, kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t rowwise_adagrad_apply(const AdagradArgs& a, cudaStream_t stream) {
  if (a.total_rows <= 0) return cudaSuccess;
  if (a.list != nullptr) return launch_list<false>(a, nullptr, stream);
  if (a.full) return cudaErrorInvalidValue;  // the per-element update walks the touched list
  const int grid = scan_grid(a.total_rows);
  if (a.max_dim <= 128) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long want = ((a.total_rows + 15) / 16 + kThreads - 1) / kThreads;
    const int tgrid = static_cast<int>(want < sms * 8 ? (want > 0 ? want : 1) : sms * 8);
    const size_t smem = a.num_tables <= 4096 ? static_cast<size_t>(a.num_tables) * sizeof(long long) : 0;
    rowwise_adagrad_thread_kernel<<<tgrid, kThreads, smem, stream>>>(a);
    return cudaGetLastError();
  }
  if (a.max_dim <= 128) rowwise_adagrad_kernel<1><<<grid, kThreads, 0, stream>>>(a);
  else if (a.max_dim <= 256) rowwise_adagrad_kernel<2><<<grid, kThreads, 0, stream>>>(a);
  else if (a.max_dim <= 512) rowwise_adagrad_kernel<4><<<grid, kThreads, 0, stream>>>(a);
  else rowwise_adagrad_kernel<8><<<grid, kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t touched_grad_sqnorm(const AdagradArgs& a, float* out_sq, cudaStream_t stream) {
  if (a.total_rows <= 0) return cudaSuccess;
  if (a.list != nullptr) return launch_list<true>(a, out_sq, stream);
  touched_sqnorm_kernel<<<scan_grid(a.total_rows), kThreads, 0, stream>>>(a, out_sq);
  return cudaGetLastError();
}

}  // namespace mdl
