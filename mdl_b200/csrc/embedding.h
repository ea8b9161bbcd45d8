// Host interface of the fused embedding-bag kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mdl {

constexpr int kMaxWorld = 8;

// Everything a lookup/update launch needs. Arrays are device pointers.
// "Slab": one fp32 buffer per rank holding the local shard of every table;
// table t occupies elements [t_base[t], t_base[t] + local_rows_t * dim_t).
// The "row space" numbers the local rows of all tables: row r of table t has
// row-space index t_row_base[t] + r (used by the Adagrad accumulator and the
// touched-row flags).
struct EmbPlan {
  int num_features = 0;
  int world = 1;
  int rank = 0;
  int max_vec = 8;  // max over features of ceil(width / (4 * lanes)) (selects the kernel variant)
  // work list: feature f owns warp-chunks [f_chunk_prefix[f], f_chunk_prefix[f+1])
  const long long* f_chunk_prefix = nullptr;  // [F+1]
  const long long* f_bag_prefix = nullptr;    // [F+1] prefix of bag counts (work split)
  const long long* f_src_bag = nullptr;       // [F] first CSR bag of feature f's ids in the batch (several plan
                                              // features may read one batch feature)
  const long long* id_offsets = nullptr;      // [total_bags+1] CSR offsets into ids
  const long long* ids = nullptr;             // raw ids (int64)
  // per feature
  const int* f_table = nullptr;        // table index, -1 for a dense feature
  const int* f_pool = nullptr;         // 0 none (first id), 1 mean, 2 sum
  const int* f_hash = nullptr;         // 0 ids used as-is, 1 pre_hashed low bits (+1)
  const long long* f_buckets = nullptr;// pre_hashed bucket count (power of two)
  const int* f_width = nullptr;        // output width (embedding dim or dense width)
  const int* f_lanes = nullptr;        // lanes per bag (power of two)
  const long long* f_out_base = nullptr;  // element offset of the feature's output matrix
  const long long* f_out_ld = nullptr;    // row stride of that matrix (elements)
  const int* f_out_col = nullptr;      // first logical column of the feature
  const int* f_slice = nullptr;        // per-feature column map: phys = (c/slice)*stride + c%slice (0 = identity)
  const int* f_slice_stride = nullptr;
  const int* f_dense_col = nullptr;    // dense features: first column in `dense`
  const int* f_phys0 = nullptr;        // physical column of the feature's first column
  const int* f_split = nullptr;        // columns before the next slice boundary (-1: several boundaries)
  int max_dim = 0;                     // widest table of the plan (owner-push kernels)
  // per table
  const long long* t_base = nullptr;
  const long long* t_row_base = nullptr;
  const int* t_dim = nullptr;
  const int* t_mode = nullptr;         // 0 row-wise cyclic, 1 table-wise
  const int* t_cyc = nullptr;          // row-wise cyclic offset
  const int* t_owner = nullptr;        // table-wise owner rank
  const long long* t_rows = nullptr;   // global row count (bounds check)
  // layouts of EVERY rank (local row counts differ per rank): [world * num_tables]
  int num_tables = 0;
  const long long* t_base_all = nullptr;      // t_base_all[r * T + t]: element base of table t in rank r's slab
  const long long* t_row_base_all = nullptr;  // t_row_base_all[r * T + t]: its row-space base on rank r
  // peer-visible buffers, one pointer per rank (index = rank)
  float* slabs[kMaxWorld] = {};
  float* grad_slabs[kMaxWorld] = {};
  unsigned char* flags[kMaxWorld] = {};  // touched-row byte flags, indexed by row space
  // dense inputs (fp32 [rows, dense_ld]) and the pooled output (bf16)
  const float* dense = nullptr;
  long long dense_ld = 0;
  void* out = nullptr;   // bf16
  int* err = nullptr;
};

// Forward: pool every bag of every feature into `out` (bf16).
cudaError_t emb_pool_forward(const EmbPlan& plan, long long total_chunks, cudaStream_t stream);

// Backward: push d(out) of every id to its owner's grad slab and mark the
// touched rows. `grad_out` has the same layout as `out`.
cudaError_t emb_pool_backward(const EmbPlan& plan, const void* grad_out, long long total_chunks,
                              cudaStream_t stream);

// ---- multi-rank lookup ("owner-push") ----------------------------------------
// With several ranks the random row traffic stays in each owner's local HBM and
// only contiguous staging buffers are read or written over NVLink:
//   route   : each rank walks its own bags once. For every (bag, owner) pair
//             with contributing ids it appends a bundle {bag, feature, count,
//             scale} to the owner's segment and the ids' owner-local rows to the
//             owner's row list (a single row is kept in the bundle itself).
//             Dense inputs go straight into the rank's own accumulator.
//   forward : owner o reads its bundles from every rank r, gathers and sums the
//             bundle's rows from its local shard, scales, and adds ONE pooled
//             vector per bundle into r's fp32 accumulator [rows, out_ld] (vector
//             reductions over NVLink); r then converts it to the bf16 output.
//   backward: r stages d(out) in peer-visible memory; owner o reads the bf16
//             gradient slice of each bundle's bag once and adds it into the
//             bundle's LOCAL grad rows, marking them touched.
// An owner's work is the ids it owns, whatever the number of ranks; NVLink
// carries one vector per (bag, owner) in each direction.
struct RouteBundle {
  int bag;        // sample row within the batch
  int f_count;    // plan feature | (number of rows << 16)
  int row;        // the row itself when count == 1, else the first index in the row list
  float scale;    // 1 (sum / single id) or 1 / valid ids of the bag (mean)
};
struct OwnerArgs {
  RouteBundle* bundles[kMaxWorld] = {};  // rank r's bundles: [world][cap_bundles]
  int* rows[kMaxWorld] = {};             // rank r's row lists: [world][cap_rows]
  int* counts[kMaxWorld] = {};           // rank r's [world][2]: bundles, rows per owner
  long long cap_bundles = 0, cap_rows = 0;
  float* acc[kMaxWorld] = {};            // forward: each rank's fp32 accumulator
  const void* grad[kMaxWorld] = {};      // backward: each rank's bf16 d(out)
  const float* dense = nullptr;          // this rank's dense inputs (route pass)
  long long dense_ld = 0;
};
// route pass of this rank (its counts and accumulator zeroed beforehand)
cudaError_t emb_route(const EmbPlan& plan, const OwnerArgs& o, long long total_chunks, cudaStream_t stream);
cudaError_t emb_owner_forward(const EmbPlan& plan, const OwnerArgs& o, cudaStream_t stream);
cudaError_t emb_owner_backward(const EmbPlan& plan, const OwnerArgs& o, cudaStream_t stream);
// out[i] = bf16(acc[i]) for i < n (n a multiple of 8, 16-byte aligned buffers)
cudaError_t emb_acc_to_bf16(const float* acc, void* out, long long n, cudaStream_t stream);

// Row-wise Adagrad over this rank's touched rows (reference optim.py:31-62):
//   g = grad * grad_scale * clip_scale[0]; acc += mean(g^2); w -= lr * g / (sqrt(acc) + eps)
// then zero the grad rows and clear the flags. Touched rows are found by a
// scan of the byte flags (16 per lane per load), so the backward needs no
// shared counter and there is no capacity limit.
struct AdagradArgs {
  float* slab = nullptr;
  float* grad_slab = nullptr;
  float* acc = nullptr;              // fp32 [row space]
  unsigned char* flags = nullptr;    // [row space, padded to a multiple of 512]
  long long total_rows = 0;
  int num_tables = 0;
  const long long* t_base = nullptr;
  const long long* t_row_base = nullptr;
  const int* t_dim = nullptr;
  float lr = 0.f, eps = 1e-10f, grad_scale = 1.f;
  const float* clip_scale = nullptr;  // optional device scalar (nullptr = 1)
  int max_dim = 1024;                 // widest table (selects the kernel variant)
  int* err = nullptr;
  // Touched-row list (row-space indices, capacity total_rows) written by
  // compact_touched. When set, the update and the norm walk the list instead of
  // scanning the flags.
  unsigned* list = nullptr;
  unsigned* count = nullptr;
  // Full (per-element) Adagrad: acc holds one fp32 sum per weight element at the
  // weight's slab offset (torch.optim.Adagrad / ShardedAdagrad semantics); needs the list.
  bool full = false;
};
cudaError_t rowwise_adagrad_apply(const AdagradArgs& a, cudaStream_t stream);

// Collect the touched rows into a.list / a.count (any order) and clear their
// flags. One 16-byte flag load per thread, a block-wide prefix sum and one
// atomic per block.
cudaError_t compact_touched(const AdagradArgs& a, cudaStream_t stream);

// Sum of squared (scaled) gradients over the touched rows (for global sparse clipping).
cudaError_t touched_grad_sqnorm(const AdagradArgs& a, float* out_sq, cudaStream_t stream);

}  // namespace mdl
