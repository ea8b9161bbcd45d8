// Python bindings of the mdl_b200 native kernels. This is the only
// translation unit that includes torch headers; the kernels themselves live in
// the .cu files and take raw pointers plus a cudaStream_t.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cmath>
#include <optional>
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace {

// Number of kernels launched through these bindings (benchmarks report it).
long long g_launches = 0;
int64_t launch_count() { return g_launches; }

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <typename T = void>
T* ptr(const at::Tensor& t) {
  return t.defined() ? reinterpret_cast<T*>(t.data_ptr()) : nullptr;
}
template <typename T = void>
T* optr(const std::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

cudaStream_t stream_of(const at::Tensor& t) { return at::cuda::getCurrentCUDAStream(t.device().index()).stream(); }

void require_cuda(const at::Tensor& t, const char* name) {
  if (!t.is_cuda()) throw std::invalid_argument(std::string(name) + " must be a CUDA tensor");
}

// ------------------------------------------------------------------ GEMM
void gemm(const at::Tensor& A, int64_t lda, int64_t gsA, bool a_mn, const at::Tensor& B, int64_t ldb,
          int64_t gsB, bool b_mn, int64_t M, int64_t N, int64_t K, int64_t G, const at::Tensor& out,
          int64_t ldc, int64_t gsC, const std::optional<at::Tensor>& out2,
          const std::optional<at::Tensor>& bias, int64_t gs_bias, const std::optional<at::Tensor>& aux,
          int64_t ld_aux, int64_t gs_aux, const std::optional<at::Tensor>& colsum, int64_t gs_colsum,
          int64_t act, double alpha, bool accumulate, const std::optional<at::Tensor>& err,
          int64_t max_ctas, int64_t KG, int64_t ksA, int64_t ksB) {
  require_cuda(A, "A");
  require_cuda(B, "B");
  require_cuda(out, "out");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm operands must be bf16");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kFloat, "gemm out must be bf16/fp32");
  if (bias) TORCH_CHECK(bias->scalar_type() == at::kFloat, "bias must be fp32");
  if (colsum) TORCH_CHECK(colsum->scalar_type() == at::kFloat, "colsum must be fp32");
  if (aux) TORCH_CHECK(aux->scalar_type() == at::kBFloat16, "aux must be bf16");
  if (out2) TORCH_CHECK(out2->scalar_type() == at::kBFloat16, "out2 must be bf16");
  c10::cuda::CUDAGuard guard(A.device());
  mdl::GemmArgs a;
  a.A = A.data_ptr();
  a.lda = lda;
  a.gsA = gsA;
  a.a_mn_major = a_mn;
  a.B = B.data_ptr();
  a.ldb = ldb;
  a.gsB = gsB;
  a.b_mn_major = b_mn;
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  a.G = static_cast<int>(G);
  a.KG = static_cast<int>(KG);
  a.ksA = ksA;
  a.ksB = ksB;
  a.out = out.data_ptr();
  a.ldc = ldc;
  a.gsC = gsC;
  a.out_fp32 = out.scalar_type() == at::kFloat;
  a.accumulate = accumulate;
  a.out2 = optr(out2);
  a.bias = optr<const float>(bias);
  a.gs_bias = gs_bias;
  a.aux = optr(aux);
  a.ld_aux = ld_aux;
  a.gs_aux = gs_aux;
  a.colsum = optr<float>(colsum);
  a.gs_colsum = gs_colsum;
  a.act = static_cast<int>(act);
  a.alpha = static_cast<float>(alpha);
  a.err = optr<int>(err);
  a.max_ctas = static_cast<int>(max_ctas);
  check(mdl::gemm_bf16_tcgen05(a, stream_of(A)), "gemm_bf16_tcgen05");
  g_launches += 1;
}


// ------------------------------------------------------------------ embedding
template <typename T>
const T* dptr(const at::Tensor& t) { return t.defined() && t.numel() ? reinterpret_cast<const T*>(t.data_ptr()) : nullptr; }

mdl::EmbPlan make_plan(const std::vector<at::Tensor>& meta, const std::vector<int64_t>& slabs,
                       const std::vector<int64_t>& grad_slabs, const std::vector<int64_t>& flags, int64_t rank,
                       const at::Tensor& ids, const at::Tensor& id_offsets, const std::optional<at::Tensor>& dense,
                       int64_t dense_ld, const std::optional<at::Tensor>& err, int64_t max_vec) {
  // meta order (all device tensors):
  //  0 f_chunk_prefix(i64) 1 f_bag_prefix(i64) 2 f_table(i32) 3 f_pool(i32) 4 f_hash(i32) 5 f_buckets(i64)
  //  6 f_width(i32) 7 f_lanes(i32) 8 f_out_base(i64) 9 f_out_ld(i64) 10 f_out_col(i32) 11 f_slice(i32)
  //  12 f_slice_stride(i32) 13 f_dense_col(i32) 14 t_base(i64) 15 t_row_base(i64) 16 t_dim(i32) 17 t_mode(i32)
  //  18 t_cyc(i32) 19 t_owner(i32) 20 t_rows(i64) 21 t_base_all(i64 [W*T]) 22 t_row_base_all(i64 [W*T])
  //  23 f_src_bag(i64) 24 f_phys0(i32) 25 f_split(i32)
  TORCH_CHECK(meta.size() == 26, "embedding plan needs 26 metadata tensors");
  mdl::EmbPlan p;
  p.num_features = static_cast<int>(meta[2].numel());
  p.world = static_cast<int>(slabs.size());
  TORCH_CHECK(p.world >= 1 && p.world <= mdl::kMaxWorld, "world size out of range");
  p.rank = static_cast<int>(rank);
  p.max_vec = static_cast<int>(max_vec);
  p.f_chunk_prefix = dptr<long long>(meta[0]);
  p.f_bag_prefix = dptr<long long>(meta[1]);
  p.f_table = dptr<int>(meta[2]);
  p.f_pool = dptr<int>(meta[3]);
  p.f_hash = dptr<int>(meta[4]);
  p.f_buckets = dptr<long long>(meta[5]);
  p.f_width = dptr<int>(meta[6]);
  p.f_lanes = dptr<int>(meta[7]);
  p.f_out_base = dptr<long long>(meta[8]);
  p.f_out_ld = dptr<long long>(meta[9]);
  p.f_out_col = dptr<int>(meta[10]);
  p.f_slice = dptr<int>(meta[11]);
  p.f_slice_stride = dptr<int>(meta[12]);
  p.f_dense_col = dptr<int>(meta[13]);
  p.t_base = dptr<long long>(meta[14]);
  p.t_row_base = dptr<long long>(meta[15]);
  p.t_dim = dptr<int>(meta[16]);
  p.t_mode = dptr<int>(meta[17]);
  p.t_cyc = dptr<int>(meta[18]);
  p.t_owner = dptr<int>(meta[19]);
  p.t_rows = dptr<long long>(meta[20]);
  p.num_tables = static_cast<int>(meta[14].numel());
  p.t_base_all = dptr<long long>(meta[21]);
  p.t_row_base_all = dptr<long long>(meta[22]);
  p.f_src_bag = dptr<long long>(meta[23]);
  p.f_phys0 = dptr<int>(meta[24]);
  p.f_split = dptr<int>(meta[25]);
  TORCH_CHECK(meta[23].numel() == p.num_features, "f_src_bag must have one entry per feature");
  TORCH_CHECK(meta[21].numel() == static_cast<int64_t>(p.num_tables) * p.world, "t_base_all must be [world * T]");
  for (int r = 0; r < p.world; ++r) {
    p.slabs[r] = reinterpret_cast<float*>(slabs[r]);
    if (r < static_cast<int>(grad_slabs.size())) p.grad_slabs[r] = reinterpret_cast<float*>(grad_slabs[r]);
    if (r < static_cast<int>(flags.size())) p.flags[r] = reinterpret_cast<unsigned char*>(flags[r]);
  }
  p.ids = dptr<long long>(ids);
  p.id_offsets = dptr<long long>(id_offsets);
  p.dense = dense.has_value() ? dptr<float>(*dense) : nullptr;
  p.dense_ld = dense_ld;
  p.err = optr<int>(err);
  return p;
}

void emb_forward(const std::vector<at::Tensor>& meta, const std::vector<int64_t>& slabs, int64_t rank,
                 const at::Tensor& ids, const at::Tensor& id_offsets, const std::optional<at::Tensor>& dense,
                 int64_t dense_ld, const at::Tensor& out, int64_t total_chunks, const std::optional<at::Tensor>& err,
                 int64_t max_vec) {
  c10::cuda::CUDAGuard guard(out.device());
  TORCH_CHECK(out.scalar_type() == at::kBFloat16, "embedding output must be bf16");
  mdl::EmbPlan p = make_plan(meta, slabs, {}, {}, rank, ids, id_offsets, dense, dense_ld, err, max_vec);
  p.out = out.data_ptr();
  check(mdl::emb_pool_forward(p, total_chunks, stream_of(out)), "emb_pool_forward");
  g_launches += 1;
}

void emb_backward(const std::vector<at::Tensor>& meta, const std::vector<int64_t>& slabs,
                  const std::vector<int64_t>& grad_slabs, const std::vector<int64_t>& flags, int64_t rank,
                  const at::Tensor& ids, const at::Tensor& id_offsets, const at::Tensor& grad_out,
                  int64_t total_chunks, const std::optional<at::Tensor>& err, int64_t max_vec) {
  c10::cuda::CUDAGuard guard(grad_out.device());
  TORCH_CHECK(grad_out.scalar_type() == at::kBFloat16, "embedding grad must be bf16");
  mdl::EmbPlan p = make_plan(meta, slabs, grad_slabs, flags, rank, ids, id_offsets, std::nullopt, 0, err, max_vec);
  check(mdl::emb_pool_backward(p, grad_out.data_ptr(), total_chunks, stream_of(grad_out)), "emb_pool_backward");
  g_launches += 1;
}

mdl::OwnerArgs owner_args(const std::vector<int64_t>& bundles, const std::vector<int64_t>& rows,
                          const std::vector<int64_t>& counts, int64_t cap_bundles, int64_t cap_rows, int world) {
  TORCH_CHECK(static_cast<int>(bundles.size()) == world && static_cast<int>(rows.size()) == world &&
                  static_cast<int>(counts.size()) == world,
              "one bundle, row-list and count pointer per rank");
  mdl::OwnerArgs o;
  for (int r = 0; r < world; ++r) {
    o.bundles[r] = reinterpret_cast<mdl::RouteBundle*>(bundles[r]);
    o.rows[r] = reinterpret_cast<int*>(rows[r]);
    o.counts[r] = reinterpret_cast<int*>(counts[r]);
  }
  o.cap_bundles = cap_bundles;
  o.cap_rows = cap_rows;
  return o;
}

// Route pass: this rank's contributing ids -> entries in their owners' segments;
// dense inputs -> this rank's accumulator.
void emb_route(const std::vector<at::Tensor>& meta, const std::vector<int64_t>& slabs, int64_t rank,
               const at::Tensor& ids, const at::Tensor& id_offsets, const std::vector<int64_t>& bundles,
               const std::vector<int64_t>& rows, const std::vector<int64_t>& counts, int64_t cap_bundles,
               int64_t cap_rows, const at::Tensor& acc,
               const std::optional<at::Tensor>& dense, int64_t dense_ld, int64_t total_chunks,
               const std::optional<at::Tensor>& err, int64_t max_vec) {
  c10::cuda::CUDAGuard guard(ids.device());
  mdl::EmbPlan p = make_plan(meta, slabs, {}, {}, rank, ids, id_offsets, std::nullopt, 0, err, max_vec);
  mdl::OwnerArgs o = owner_args(bundles, rows, counts, cap_bundles, cap_rows, p.world);
  TORCH_CHECK(acc.scalar_type() == at::kFloat, "accumulator must be fp32");
  o.acc[p.rank] = acc.data_ptr<float>();
  if (dense.has_value()) {
    TORCH_CHECK(dense->scalar_type() == at::kFloat, "dense inputs must be fp32");
    o.dense = dense->data_ptr<float>();
    o.dense_ld = dense_ld;
  }
  check(mdl::emb_route(p, o, total_chunks, stream_of(ids)), "emb_route");
  g_launches += 1;
}

void emb_owner_forward(const std::vector<at::Tensor>& meta, const std::vector<int64_t>& slabs, int64_t rank,
                       const at::Tensor& ids, const at::Tensor& id_offsets, const std::vector<int64_t>& bundles,
                       const std::vector<int64_t>& rows, const std::vector<int64_t>& counts, int64_t cap_bundles,
                       int64_t cap_rows, const std::vector<int64_t>& accs,
                       int64_t max_dim, const std::optional<at::Tensor>& err) {
  c10::cuda::CUDAGuard guard(ids.device());
  mdl::EmbPlan p = make_plan(meta, slabs, {}, {}, rank, ids, id_offsets, std::nullopt, 0, err, 1);
  p.max_dim = static_cast<int>(max_dim);
  mdl::OwnerArgs o = owner_args(bundles, rows, counts, cap_bundles, cap_rows, p.world);
  TORCH_CHECK(static_cast<int>(accs.size()) == p.world, "one accumulator pointer per rank");
  for (int r = 0; r < p.world; ++r) o.acc[r] = reinterpret_cast<float*>(accs[r]);
  check(mdl::emb_owner_forward(p, o, stream_of(ids)), "emb_owner_forward");
  g_launches += 1;
}

void emb_owner_backward(const std::vector<at::Tensor>& meta, const std::vector<int64_t>& slabs,
                        const std::vector<int64_t>& grad_slabs, const std::vector<int64_t>& flags, int64_t rank,
                        const at::Tensor& ids, const at::Tensor& id_offsets, const std::vector<int64_t>& bundles,
                        const std::vector<int64_t>& rows, const std::vector<int64_t>& counts, int64_t cap_bundles,
                        int64_t cap_rows, const std::vector<int64_t>& grads,
                        int64_t max_dim, const std::optional<at::Tensor>& err) {
  c10::cuda::CUDAGuard guard(ids.device());
  mdl::EmbPlan p = make_plan(meta, slabs, grad_slabs, flags, rank, ids, id_offsets, std::nullopt, 0, err, 1);
  p.max_dim = static_cast<int>(max_dim);
  mdl::OwnerArgs o = owner_args(bundles, rows, counts, cap_bundles, cap_rows, p.world);
  TORCH_CHECK(static_cast<int>(grads.size()) == p.world, "one staged gradient pointer per rank");
  for (int r = 0; r < p.world; ++r) o.grad[r] = reinterpret_cast<const void*>(grads[r]);
  check(mdl::emb_owner_backward(p, o, stream_of(ids)), "emb_owner_backward");
  g_launches += 1;
}

void emb_acc_to_bf16(const at::Tensor& acc, const at::Tensor& out) {
  c10::cuda::CUDAGuard guard(acc.device());
  TORCH_CHECK(acc.scalar_type() == at::kFloat && out.scalar_type() == at::kBFloat16, "fp32 -> bf16");
  TORCH_CHECK(acc.numel() >= out.numel() && out.is_contiguous(), "accumulator smaller than the output");
  check(mdl::emb_acc_to_bf16(acc.data_ptr<float>(), out.data_ptr(), out.numel(), stream_of(out)), "emb_acc_to_bf16");
  g_launches += 1;
}

mdl::AdagradArgs adagrad_args(const at::Tensor& slab, const at::Tensor& grad_slab, const at::Tensor& acc,
                              const at::Tensor& flags, int64_t total_rows, const at::Tensor& t_base,
                              const at::Tensor& t_row_base, const at::Tensor& t_dim, double lr, double eps,
                              double grad_scale, const std::optional<at::Tensor>& clip,
                              const std::optional<at::Tensor>& err, int64_t max_dim) {
  TORCH_CHECK(flags.scalar_type() == at::kByte && flags.numel() >= (total_rows + 511) / 512 * 512,
              "flags must be uint8 padded to a multiple of 512 rows");
  mdl::AdagradArgs a;
  a.slab = ptr<float>(slab);
  a.grad_slab = ptr<float>(grad_slab);
  a.acc = ptr<float>(acc);
  a.flags = ptr<unsigned char>(flags);
  a.total_rows = total_rows;
  a.num_tables = static_cast<int>(t_base.numel());
  a.t_base = ptr<const long long>(t_base);
  a.t_row_base = ptr<const long long>(t_row_base);
  a.t_dim = ptr<const int>(t_dim);
  a.lr = static_cast<float>(lr);
  a.eps = static_cast<float>(eps);
  a.grad_scale = static_cast<float>(grad_scale);
  a.clip_scale = optr<const float>(clip);
  a.max_dim = static_cast<int>(max_dim);
  a.err = optr<int>(err);
  return a;
}

void set_list(mdl::AdagradArgs& a, const std::optional<at::Tensor>& list, const std::optional<at::Tensor>& count) {
  if (list.has_value() != count.has_value()) TORCH_CHECK(false, "touched list and count go together");
  if (!list.has_value()) return;
  TORCH_CHECK(list->scalar_type() == at::kInt && list->numel() >= a.total_rows, "touched list: int32 [total_rows]");
  TORCH_CHECK(count->scalar_type() == at::kInt && count->numel() >= 1, "touched count: int32 [1]");
  a.list = reinterpret_cast<unsigned*>(list->data_ptr());
  a.count = reinterpret_cast<unsigned*>(count->data_ptr());
}

void adagrad_apply(const at::Tensor& slab, const at::Tensor& grad_slab, const at::Tensor& acc, const at::Tensor& flags,
                   int64_t total_rows, const at::Tensor& t_base, const at::Tensor& t_row_base,
                   const at::Tensor& t_dim, double lr, double eps, double grad_scale,
                   const std::optional<at::Tensor>& clip, const std::optional<at::Tensor>& err, int64_t max_dim,
                   const std::optional<at::Tensor>& list, const std::optional<at::Tensor>& count, bool full) {
  c10::cuda::CUDAGuard guard(slab.device());
  auto a = adagrad_args(slab, grad_slab, acc, flags, total_rows, t_base, t_row_base, t_dim, lr, eps, grad_scale,
                        clip, err, max_dim);
  set_list(a, list, count);
  a.full = full;
  TORCH_CHECK(!full || acc.numel() >= slab.numel(), "full Adagrad: one accumulator per weight element");
  check(mdl::rowwise_adagrad_apply(a, stream_of(slab)), "rowwise_adagrad_apply");
  g_launches += 1;
}

void compact_touched(const at::Tensor& flags, int64_t total_rows, const at::Tensor& list, const at::Tensor& count) {
  c10::cuda::CUDAGuard guard(flags.device());
  TORCH_CHECK(flags.scalar_type() == at::kByte && flags.numel() >= (total_rows + 511) / 512 * 512,
              "flags must be uint8 padded to a multiple of 512 rows");
  mdl::AdagradArgs a;
  a.flags = ptr<unsigned char>(flags);
  a.total_rows = total_rows;
  set_list(a, list, count);
  check(mdl::compact_touched(a, stream_of(flags)), "compact_touched");
  g_launches += 1;
}

void touched_sqnorm(const at::Tensor& grad_slab, const at::Tensor& flags, int64_t total_rows,
                    const at::Tensor& t_base, const at::Tensor& t_row_base, const at::Tensor& t_dim, double grad_scale,
                    const at::Tensor& out, const std::optional<at::Tensor>& list,
                    const std::optional<at::Tensor>& count, int64_t max_dim) {
  c10::cuda::CUDAGuard guard(grad_slab.device());
  mdl::AdagradArgs a = adagrad_args(grad_slab, grad_slab, grad_slab, flags, total_rows, t_base, t_row_base, t_dim,
                                    0.0, 1.0, grad_scale, std::nullopt, std::nullopt, max_dim);
  set_list(a, list, count);
  check(mdl::touched_grad_sqnorm(a, ptr<float>(out), stream_of(grad_slab)), "touched_grad_sqnorm");
  g_launches += 1;
}

// ------------------------------------------------------------------ norms
void ln_fwd(const at::Tensor& a, const std::optional<at::Tensor>& b, const std::optional<at::Tensor>& gamma,
            const std::optional<at::Tensor>& beta, const at::Tensor& out, const at::Tensor& mean,
            const at::Tensor& rstd, int64_t B, int64_t T, int64_t D, bool mix, double eps) {
  c10::cuda::CUDAGuard guard(a.device());
  mdl::LNFwdArgs p;
  p.a = a.data_ptr();
  p.b = optr(b);
  p.gamma = optr<const float>(gamma);
  p.beta = optr<const float>(beta);
  p.out = out.data_ptr();
  p.mean = ptr<float>(mean);
  p.rstd = ptr<float>(rstd);
  p.B = static_cast<int>(B);
  p.T = static_cast<int>(T);
  p.D = static_cast<int>(D);
  p.mix = mix ? 1 : 0;
  p.eps = static_cast<float>(eps);
  check(mdl::layernorm_fwd(p, stream_of(a)), "layernorm_fwd");
  g_launches += 1;
}

int64_t ln_bwd_grid(int64_t B) { return mdl::layernorm_bwd_grid(static_cast<int>(B)); }

void ln_bwd(const std::optional<at::Tensor>& dy, const std::optional<at::Tensor>& dy_bcast, double bcast_scale,
            const at::Tensor& a, const std::optional<at::Tensor>& b, const at::Tensor& mean, const at::Tensor& rstd,
            const std::optional<at::Tensor>& gamma, const at::Tensor& dx, const std::optional<at::Tensor>& dx2,
            const at::Tensor& partials, const std::optional<at::Tensor>& dgamma, const std::optional<at::Tensor>& dbeta,
            int64_t B, int64_t T, int64_t D, bool mix, int64_t grid, const std::optional<at::Tensor>& res) {
  c10::cuda::CUDAGuard guard(a.device());
  mdl::LNBwdArgs p;
  p.dy = optr(dy);
  p.dy_bcast = optr(dy_bcast);
  p.bcast_scale = static_cast<float>(bcast_scale);
  p.a = a.data_ptr();
  p.b = optr(b);
  p.mean = ptr<float>(mean);
  p.rstd = ptr<float>(rstd);
  p.gamma = optr<const float>(gamma);
  p.dx = dx.data_ptr();
  p.dx2 = optr(dx2);
  p.res = optr(res);
  p.partials = ptr<float>(partials);
  p.dgamma = optr<float>(dgamma);
  p.dbeta = optr<float>(dbeta);
  p.B = static_cast<int>(B);
  p.T = static_cast<int>(T);
  p.D = static_cast<int>(D);
  p.mix = mix ? 1 : 0;
  p.grid = static_cast<int>(grid);
  check(mdl::layernorm_bwd(p, stream_of(a)), "layernorm_bwd");
  g_launches += 2;
}

void rms_fwd(const at::Tensor& x, const std::optional<at::Tensor>& w, const at::Tensor& out, const at::Tensor& rstd,
             int64_t rows, int64_t D, double eps) {
  c10::cuda::CUDAGuard guard(x.device());
  mdl::RMSArgs p;
  p.x = x.data_ptr();
  p.weight = optr<const float>(w);
  p.out = out.data_ptr();
  p.rstd = ptr<float>(rstd);
  p.rows = rows;
  p.D = static_cast<int>(D);
  p.eps = static_cast<float>(eps);
  check(mdl::rmsnorm_fwd(p, stream_of(x)), "rmsnorm_fwd");
  g_launches += 1;
}

void rms_bwd(const at::Tensor& x, const std::optional<at::Tensor>& w, const at::Tensor& rstd, const at::Tensor& dy,
             const at::Tensor& dx, const std::optional<at::Tensor>& dw, int64_t rows, int64_t D,
             const std::optional<at::Tensor>& dres, int64_t res_period, int64_t res_tail) {
  c10::cuda::CUDAGuard guard(x.device());
  mdl::RMSArgs p;
  p.x = x.data_ptr();
  p.weight = optr<const float>(w);
  p.rstd = ptr<float>(rstd);
  p.dy = dy.data_ptr();
  p.dx = dx.data_ptr();
  p.dweight = optr<float>(dw);
  p.rows = rows;
  p.D = static_cast<int>(D);
  p.dres = optr(dres);
  p.res_period = static_cast<int>(res_period);
  p.res_tail = static_cast<int>(res_tail);
  check(mdl::rmsnorm_bwd(p, stream_of(x)), "rmsnorm_bwd");
  g_launches += 1;
}

// ------------------------------------------------------------------ misc
void token_mean(const at::Tensor& x, const at::Tensor& out, int64_t B, int64_t T, int64_t D) {
  c10::cuda::CUDAGuard guard(x.device());
  check(mdl::token_mean_fwd(x.data_ptr(), out.data_ptr(), static_cast<int>(B), static_cast<int>(T),
                            static_cast<int>(D), stream_of(x)),
        "token_mean_fwd");
  g_launches += 1;
}

void colsum(const at::Tensor& x, const at::Tensor& out, int64_t G, int64_t M, int64_t N, int64_t ld, int64_t gs,
            double scale, int64_t gs_out) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kFloat, "colsum: bf16 in, fp32 out");
  check(mdl::colsum_bf16(x.data_ptr(), ptr<float>(out), static_cast<int>(G), M, static_cast<int>(N), ld, gs,
                         static_cast<float>(scale), stream_of(x), gs_out),
        "colsum_bf16");
  g_launches += 1;
}

void head_bce(const at::Tensor& act, const at::Tensor& pre, const at::Tensor& w2, const std::optional<at::Tensor>& b2,
              const std::optional<at::Tensor>& labels, const std::optional<at::Tensor>& mask,
              const std::optional<at::Tensor>& task_scale, const std::optional<at::Tensor>& logits,
              const std::optional<at::Tensor>& loss, const std::optional<at::Tensor>& dpre,
              const std::optional<at::Tensor>& dw2, const std::optional<at::Tensor>& db2, int64_t B, int64_t ntask,
              int64_t H, bool relu) {
  c10::cuda::CUDAGuard guard(act.device());
  mdl::HeadArgs p;
  p.act = act.data_ptr();
  p.pre = pre.data_ptr();
  p.w2 = ptr<const float>(w2);
  p.b2 = optr<const float>(b2);
  p.labels = optr<const float>(labels);
  p.mask = optr<const float>(mask);
  p.task_scale = optr<const float>(task_scale);
  p.logits = optr<float>(logits);
  p.loss = optr<float>(loss);
  p.dpre = optr(dpre);
  p.dw2 = optr<float>(dw2);
  p.db2 = optr<float>(db2);
  p.B = static_cast<int>(B);
  p.ntask = static_cast<int>(ntask);
  p.H = static_cast<int>(H);
  p.relu = relu ? 1 : 0;
  check(mdl::head_bce(p, stream_of(act)), "head_bce");
  g_launches += 1;
}

mdl::OptimArgs optim_args(const at::Tensor& param, const at::Tensor& grad, const at::Tensor& s1,
                          const std::optional<at::Tensor>& s2, const std::optional<at::Tensor>& shadow, double lr,
                          double beta1, double beta2, double eps, double wd, double bc1, double bc2, double alpha,
                          double grad_scale, const std::optional<at::Tensor>& clip) {
  mdl::OptimArgs a;
  a.param = ptr<float>(param);
  a.grad = ptr<const float>(grad);
  a.state1 = ptr<float>(s1);
  a.state2 = optr<float>(s2);
  a.shadow = optr(shadow);
  a.n = param.numel();
  a.lr = static_cast<float>(lr);
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.eps = static_cast<float>(eps);
  a.weight_decay = static_cast<float>(wd);
  a.bias_correction1 = static_cast<float>(bc1);
  a.bias_correction2 = static_cast<float>(bc2);
  a.alpha = static_cast<float>(alpha);
  a.grad_scale = static_cast<float>(grad_scale);
  a.clip = optr<const float>(clip);
  return a;
}

void adam(const at::Tensor& param, const at::Tensor& grad, const at::Tensor& m, const at::Tensor& v,
          const std::optional<at::Tensor>& shadow, double lr, double beta1, double beta2, double eps, double wd,
          double bc1, double bc2, double grad_scale, const std::optional<at::Tensor>& clip, bool zero_grad,
          int64_t max_blocks) {
  c10::cuda::CUDAGuard guard(param.device());
  auto a = optim_args(param, grad, m, v, shadow, lr, beta1, beta2, eps, wd, bc1, bc2, 0.0, grad_scale, clip);
  a.zero_grad = zero_grad;
  a.max_blocks = static_cast<int>(max_blocks);
  check(mdl::adam_step(a, stream_of(param)), "adam_step");
  g_launches += 1;
}

void rmsprop(const at::Tensor& param, const at::Tensor& grad, const at::Tensor& sq,
             const std::optional<at::Tensor>& shadow, double lr, double alpha, double eps, double wd,
             double grad_scale, const std::optional<at::Tensor>& clip, bool zero_grad, int64_t max_blocks) {
  c10::cuda::CUDAGuard guard(param.device());
  auto a = optim_args(param, grad, sq, std::nullopt, shadow, lr, 0.0, 0.0, eps, wd, 1.0, 1.0, alpha, grad_scale, clip);
  a.zero_grad = zero_grad;
  a.max_blocks = static_cast<int>(max_blocks);
  check(mdl::rmsprop_step(a, stream_of(param)), "rmsprop_step");
  g_launches += 1;
}

void sqnorm(const at::Tensor& grad, double grad_scale, const at::Tensor& out) {
  c10::cuda::CUDAGuard guard(grad.device());
  check(mdl::grad_sqnorm(ptr<const float>(grad), grad.numel(), static_cast<float>(grad_scale), ptr<float>(out),
                         stream_of(grad)),
        "grad_sqnorm");
  g_launches += 1;
}

void clip_factor(const at::Tensor& sum_sq, double max_norm, const at::Tensor& clip) {
  c10::cuda::CUDAGuard guard(sum_sq.device());
  check(mdl::clip_factor(ptr<const float>(sum_sq), static_cast<float>(max_norm), ptr<float>(clip), stream_of(sum_sq)),
        "clip_factor");
  g_launches += 1;
}

void cast_bf16(const at::Tensor& src, const at::Tensor& dst) {
  c10::cuda::CUDAGuard guard(src.device());
  check(mdl::cast_f32_bf16(ptr<const float>(src), dst.data_ptr(), src.numel(), stream_of(src)), "cast_f32_bf16");
  g_launches += 1;
}


// ------------------------------------------------------------------ symmetric memory
py::tuple ipc_alloc(int64_t bytes, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  void* p = nullptr;
  cudaIpcMemHandle_t h;
  check(mdl::ipc_alloc(static_cast<size_t>(bytes), &p, &h), "ipc_alloc");
  return py::make_tuple(reinterpret_cast<int64_t>(p), py::bytes(reinterpret_cast<const char*>(&h), sizeof(h)));
}

int64_t ipc_open(const py::bytes& handle, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, s.data(), sizeof(h));
  void* p = nullptr;
  check(mdl::ipc_open(h, &p), "ipc_open");
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr_, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  check(mdl::ipc_close(reinterpret_cast<void*>(ptr_)), "ipc_close");
}

void ipc_free(int64_t ptr_, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  check(mdl::ipc_free(reinterpret_cast<void*>(ptr_)), "ipc_free");
}

at::Tensor tensor_from_ptr(int64_t ptr_, int64_t numel, at::ScalarType dtype, int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::Device(at::kCUDA, static_cast<c10::DeviceIndex>(device)));
  return torch::from_blob(reinterpret_cast<void*>(ptr_), {numel}, opts);
}

void mbar_timeout_selftest(const at::Tensor& err, const at::Tensor& returned) {
  c10::cuda::CUDAGuard guard(err.device());
  TORCH_CHECK(err.scalar_type() == at::kInt && returned.scalar_type() == at::kInt, "int32 words");
  check(mdl::mbar_timeout_selftest(err.data_ptr<int>(), returned.data_ptr<int>(), stream_of(err)),
        "mbar_timeout_selftest");
  g_launches += 1;
}

void set_barrier_limit(double seconds) { mdl::set_barrier_limit_ns(static_cast<uint64_t>(seconds * 1e9)); }

void barrier(const std::vector<int64_t>& signals, const at::Tensor& counter, int64_t rank,
             const std::optional<at::Tensor>& err) {
  c10::cuda::CUDAGuard guard(counter.device());
  unsigned* s[mdl::kMaxWorld] = {};
  for (size_t r = 0; r < signals.size() && r < mdl::kMaxWorld; ++r) s[r] = reinterpret_cast<unsigned*>(signals[r]);
  check(mdl::symm_barrier(s, ptr<unsigned>(counter), static_cast<int>(rank), static_cast<int>(signals.size()),
                          optr<int>(err), stream_of(counter)),
        "symm_barrier");
  g_launches += 1;
}

void dense_sync(const std::vector<int64_t>& grads, const std::vector<int64_t>& params,
                const std::vector<int64_t>& shadows, const at::Tensor& state1, const std::optional<at::Tensor>& state2,
                int64_t begin, int64_t end, int64_t fp32_from, int64_t rank, int64_t optimizer, double lr,
                double beta1, double beta2, double eps, double wd, double bc1, double bc2, double alpha,
                double grad_scale, const std::optional<at::Tensor>& clip, const std::optional<at::Tensor>& sqnorm_out,
                int64_t phase, int64_t max_blocks, const std::vector<int64_t>& multicast) {
  c10::cuda::CUDAGuard guard(state1.device());
  mdl::DenseSyncArgs a;
  TORCH_CHECK(multicast.empty() || multicast.size() == 3, "multicast: [] or [grad, master, shadow] addresses");
  if (!multicast.empty()) {
    a.mc_grad = reinterpret_cast<float*>(multicast[0]);
    a.mc_master = reinterpret_cast<float*>(multicast[1]);
    a.mc_shadow = reinterpret_cast<void*>(multicast[2]);
  }
  a.world = static_cast<int>(grads.size());
  TORCH_CHECK(a.world >= 1 && a.world <= mdl::kMaxWorld, "world out of range");
  for (int r = 0; r < a.world; ++r) {
    a.grads[r] = reinterpret_cast<float*>(grads[r]);
    a.params[r] = reinterpret_cast<float*>(params[r]);
    a.shadows[r] = r < static_cast<int>(shadows.size()) ? reinterpret_cast<void*>(shadows[r]) : nullptr;
  }
  a.state1 = ptr<float>(state1);
  a.state2 = optr<float>(state2);
  a.begin = begin;
  a.end = end;
  a.fp32_from = fp32_from;
  a.rank = static_cast<int>(rank);
  a.optimizer = static_cast<int>(optimizer);
  a.lr = static_cast<float>(lr);
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.eps = static_cast<float>(eps);
  a.weight_decay = static_cast<float>(wd);
  a.bias_correction1 = static_cast<float>(bc1);
  a.bias_correction2 = static_cast<float>(bc2);
  a.alpha = static_cast<float>(alpha);
  a.grad_scale = static_cast<float>(grad_scale);
  a.clip = optr<const float>(clip);
  a.sqnorm_out = optr<float>(sqnorm_out);
  a.phase = static_cast<int>(phase);
  a.max_blocks = static_cast<int>(max_blocks);
  check(mdl::dense_sync_update(a, stream_of(state1)), "dense_sync_update");
  g_launches += 1;
}

void small_allreduce(const std::vector<int64_t>& bufs, const at::Tensor& out, int64_t n) {
  c10::cuda::CUDAGuard guard(out.device());
  float* b[mdl::kMaxWorld] = {};
  for (size_t r = 0; r < bufs.size() && r < mdl::kMaxWorld; ++r) b[r] = reinterpret_cast<float*>(bufs[r]);
  check(mdl::small_allreduce(b, ptr<float>(out), static_cast<int>(n), static_cast<int>(bufs.size()), stream_of(out)),
        "small_allreduce");
  g_launches += 1;
}


// ------------------------------------------------------------------ attention
mdl::SmallAttnArgs small_attn_args(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                                   const at::Tensor& lse, const std::optional<at::Tensor>& key_valid, int64_t B,
                                   int64_t Nq, int64_t Nk, int64_t H, int64_t hd, double scale) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
              "attention operands must be bf16");
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.dim() == 3 && o.dim() == 3, "attention tensors are [B, N, D]");
  TORCH_CHECK(q.stride(2) == 1 && k.stride(2) == 1 && v.stride(2) == 1 && o.stride(2) == 1, "last dim contiguous");
  TORCH_CHECK(k.stride(0) == v.stride(0) && k.stride(1) == v.stride(1), "K and V must share strides");
  mdl::SmallAttnArgs a;
  a.q = q.data_ptr();
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.o = o.data_ptr();
  a.lse = ptr<float>(lse);
  a.key_valid = optr<const int>(key_valid);
  a.ldq = q.stride(1);
  a.ldk = k.stride(1);
  a.ldo = o.stride(1);
  a.bsq = q.stride(0);
  a.bsk = k.stride(0);
  a.bso = o.stride(0);
  a.B = static_cast<int>(B);
  a.Nq = static_cast<int>(Nq);
  a.Nk = static_cast<int>(Nk);
  a.H = static_cast<int>(H);
  a.hd = static_cast<int>(hd);
  a.scale = static_cast<float>(scale);
  return a;
}

void small_attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                    const at::Tensor& lse, const std::optional<at::Tensor>& key_valid, int64_t H, double scale) {
  c10::cuda::CUDAGuard guard(q.device());
  auto a = small_attn_args(q, k, v, o, lse, key_valid, q.size(0), q.size(1), k.size(1), H, q.size(2) / H, scale);
  check(mdl::small_attention_fwd(a, stream_of(q)), "small_attention_fwd");
  g_launches += 1;
}

void small_attn_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
                    const at::Tensor& lse, const std::optional<at::Tensor>& key_valid, const at::Tensor& dout,
                    const at::Tensor& dq, const at::Tensor& dk, const at::Tensor& dv, int64_t H, double scale) {
  c10::cuda::CUDAGuard guard(q.device());
  auto a = small_attn_args(q, k, v, o, lse, key_valid, q.size(0), q.size(1), k.size(1), H, q.size(2) / H, scale);
  TORCH_CHECK(dout.stride(1) == o.stride(1) && dout.stride(0) == o.stride(0), "dO must share O's strides");
  TORCH_CHECK(dq.stride(1) == q.stride(1) && dk.stride(1) == k.stride(1) && dv.stride(1) == k.stride(1),
              "gradients must share their input's strides");
  a.dout = dout.data_ptr();
  a.dq = dq.data_ptr();
  a.dk = dk.data_ptr();
  a.dv = dv.data_ptr();
  check(mdl::small_attention_bwd(a, stream_of(q)), "small_attention_bwd");
  g_launches += 1;
}

void position_add(const at::Tensor& x, const at::Tensor& pos, const at::Tensor& kstart, int64_t B, int64_t L,
                  int64_t D) {
  c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && pos.scalar_type() == at::kFloat && kstart.scalar_type() == at::kInt,
              "position_add: bf16 x, fp32 pos, int32 kstart");
  TORCH_CHECK(x.numel() >= B * L * D && kstart.numel() >= B, "position_add: sizes");
  check(mdl::position_add(x.data_ptr(), pos.data_ptr<float>(), kstart.data_ptr<int>(), static_cast<int>(B),
                          static_cast<int>(L), static_cast<int>(D), stream_of(x)),
        "position_add");
  g_launches += 1;
}

void sqa_fwd(const at::Tensor& q, const at::Tensor& hist, const at::Tensor& kstart, const at::Tensor& ctx,
             const at::Tensor& lse, double scale) {
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(q.scalar_type() == at::kFloat && hist.scalar_type() == at::kBFloat16 &&
                  kstart.scalar_type() == at::kInt && ctx.scalar_type() == at::kFloat && lse.scalar_type() == at::kFloat,
              "sqa_fwd: fp32 q / ctx / lse, bf16 history, int32 kstart");
  TORCH_CHECK(hist.dim() == 4 && hist.is_contiguous() && q.is_contiguous() && ctx.is_contiguous(),
              "sqa_fwd: contiguous q [B, N, D] and history [B, L, N, D]");
  mdl::SqaArgs a;
  a.B = static_cast<int>(hist.size(0)); a.L = static_cast<int>(hist.size(1));
  a.N = static_cast<int>(hist.size(2)); a.D = static_cast<int>(hist.size(3));
  TORCH_CHECK(q.numel() == static_cast<int64_t>(a.B) * a.N * a.D && ctx.numel() == q.numel() &&
                  lse.numel() == static_cast<int64_t>(a.B) * a.N && kstart.numel() >= a.B,
              "sqa_fwd: sizes");
  a.q = q.data_ptr<float>();
  a.hist = reinterpret_cast<const __nv_bfloat16*>(hist.data_ptr());
  a.kstart = kstart.data_ptr<int>();
  a.ctx = ctx.data_ptr<float>();
  a.lse = lse.data_ptr<float>();
  a.scale = static_cast<float>(scale);
  check(mdl::sqa_fwd(a, stream_of(q)), "sqa_fwd");
  g_launches += 1;
}

void sqa_bwd(const at::Tensor& q, const at::Tensor& hist, const at::Tensor& kstart, const at::Tensor& ctx,
             const at::Tensor& lse, const at::Tensor& dctx, const at::Tensor& dq, const at::Tensor& dhist,
             double scale) {
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(dctx.scalar_type() == at::kFloat && dq.scalar_type() == at::kFloat &&
                  dhist.scalar_type() == at::kBFloat16 && dctx.is_contiguous() && dq.is_contiguous() &&
                  dhist.is_contiguous() && dhist.sizes() == hist.sizes() && hist.is_contiguous(),
              "sqa_bwd: fp32 dctx / dq, bf16 dhist shaped like the history");
  mdl::SqaArgs a;
  a.B = static_cast<int>(hist.size(0)); a.L = static_cast<int>(hist.size(1));
  a.N = static_cast<int>(hist.size(2)); a.D = static_cast<int>(hist.size(3));
  TORCH_CHECK(q.numel() == static_cast<int64_t>(a.B) * a.N * a.D && dctx.numel() == q.numel() &&
                  dq.numel() == q.numel() && ctx.numel() == q.numel() && kstart.numel() >= a.B,
              "sqa_bwd: sizes");
  a.q = q.data_ptr<float>();
  a.hist = reinterpret_cast<const __nv_bfloat16*>(hist.data_ptr());
  a.kstart = kstart.data_ptr<int>();
  a.ctx = ctx.data_ptr<float>();
  a.lse = lse.data_ptr<float>();
  a.dctx = dctx.data_ptr<float>();
  a.dq = dq.data_ptr<float>();
  a.dhist = reinterpret_cast<__nv_bfloat16*>(dhist.data_ptr());
  a.scale = static_cast<float>(scale);
  check(mdl::sqa_bwd(a, stream_of(q)), "sqa_bwd");
  g_launches += 1;
}

void sqa_shared_fwd(const at::Tensor& q, const at::Tensor& hist, const at::Tensor& kstart, const at::Tensor& ctx,
                    const at::Tensor& lse, double scale) {
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(q.scalar_type() == at::kFloat && hist.scalar_type() == at::kBFloat16 &&
                  kstart.scalar_type() == at::kInt && ctx.scalar_type() == at::kFloat && lse.scalar_type() == at::kFloat,
              "sqa_shared_fwd: fp32 q / ctx / lse, bf16 history, int32 kstart");
  TORCH_CHECK(hist.dim() == 3 && q.dim() == 3 && hist.is_contiguous() && q.is_contiguous() && ctx.is_contiguous() &&
                  lse.is_contiguous(),
              "sqa_shared_fwd: contiguous q [B, G, D] and history [B, L, D]");
  mdl::SqaSharedArgs a;
  a.B = static_cast<int>(hist.size(0)); a.L = static_cast<int>(hist.size(1)); a.D = static_cast<int>(hist.size(2));
  a.G = static_cast<int>(q.size(1));
  TORCH_CHECK(q.size(0) == a.B && q.size(2) == a.D && ctx.sizes() == q.sizes() &&
                  lse.numel() == static_cast<int64_t>(a.B) * a.G && kstart.numel() >= a.B,
              "sqa_shared_fwd: sizes");
  TORCH_CHECK(mdl::sqa_shared_supported(a.G, a.D), "sqa_shared_fwd: unsupported G / D");
  a.q = q.data_ptr<float>();
  a.hist = reinterpret_cast<const __nv_bfloat16*>(hist.data_ptr());
  a.kstart = kstart.data_ptr<int>();
  a.ctx = ctx.data_ptr<float>();
  a.lse = lse.data_ptr<float>();
  a.scale = static_cast<float>(scale);
  check(mdl::sqa_shared_fwd(a, stream_of(q)), "sqa_shared_fwd");
  g_launches += 1;
}

void sqa_shared_bwd(const at::Tensor& q, const at::Tensor& hist, const at::Tensor& kstart, const at::Tensor& ctx,
                    const at::Tensor& lse, const at::Tensor& dctx, const at::Tensor& dq, const at::Tensor& dhist,
                    double scale) {
  c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(dctx.scalar_type() == at::kFloat && dq.scalar_type() == at::kFloat &&
                  dhist.scalar_type() == at::kBFloat16 && dctx.is_contiguous() && dq.is_contiguous() &&
                  dhist.is_contiguous() && dhist.sizes() == hist.sizes() && hist.is_contiguous() && hist.dim() == 3,
              "sqa_shared_bwd: fp32 dctx / dq, bf16 dhist shaped like the history [B, L, D]");
  mdl::SqaSharedArgs a;
  a.B = static_cast<int>(hist.size(0)); a.L = static_cast<int>(hist.size(1)); a.D = static_cast<int>(hist.size(2));
  a.G = static_cast<int>(q.size(1));
  TORCH_CHECK(q.dim() == 3 && q.size(0) == a.B && q.size(2) == a.D && dctx.sizes() == q.sizes() &&
                  dq.sizes() == q.sizes() && ctx.sizes() == q.sizes() &&
                  lse.numel() == static_cast<int64_t>(a.B) * a.G && kstart.numel() >= a.B,
              "sqa_shared_bwd: sizes");
  TORCH_CHECK(mdl::sqa_shared_supported(a.G, a.D), "sqa_shared_bwd: unsupported G / D");
  a.q = q.data_ptr<float>();
  a.hist = reinterpret_cast<const __nv_bfloat16*>(hist.data_ptr());
  a.kstart = kstart.data_ptr<int>();
  a.ctx = ctx.data_ptr<float>();
  a.lse = lse.data_ptr<float>();
  a.dctx = dctx.data_ptr<float>();
  a.dq = dq.data_ptr<float>();
  a.dhist = reinterpret_cast<__nv_bfloat16*>(dhist.data_ptr());
  a.scale = static_cast<float>(scale);
  check(mdl::sqa_shared_bwd(a, stream_of(q)), "sqa_shared_bwd");
  g_launches += 1;
}

void position_grad(const at::Tensor& dx, const at::Tensor& dpos, const at::Tensor& kstart, int64_t B, int64_t L,
                   int64_t D) {
  c10::cuda::CUDAGuard guard(dx.device());
  TORCH_CHECK(dx.scalar_type() == at::kBFloat16 && dpos.scalar_type() == at::kFloat && kstart.scalar_type() == at::kInt,
              "position_grad: bf16 dx, fp32 dpos, int32 kstart");
  TORCH_CHECK(dpos.numel() >= L * D, "position_grad: dpos holds fewer than L positions");
  check(mdl::position_grad(dx.data_ptr(), dpos.data_ptr<float>(), kstart.data_ptr<int>(), static_cast<int>(B),
                           static_cast<int>(L), static_cast<int>(D), stream_of(dx)),
        "position_grad");
  g_launches += 1;
}

// ------------------------------------------------------------------ flash attention
mdl::FmhaArgs fmha_args(const at::Tensor& qkv, const at::Tensor& kstart, const at::Tensor& out, const at::Tensor& lse,
                        int64_t H, int64_t Lq, bool causal, double scale, const std::optional<at::Tensor>& err,
                        int64_t ktail, int64_t kexcl) {
  require_cuda(qkv, "qkv");
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 3 && qkv.is_contiguous(), "qkv must be [B, Lk, 3D] bf16");
  TORCH_CHECK(kstart.scalar_type() == at::kInt && kstart.numel() == qkv.size(0), "kstart must be int32 [B]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous(), "out must be contiguous bf16");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous(), "lse must be contiguous fp32");
  mdl::FmhaArgs a;
  a.qkv = qkv.data_ptr();
  a.kstart = kstart.data_ptr<int>();
  a.out = out.data_ptr();
  a.lse = lse.data_ptr<float>();
  a.B = static_cast<int>(qkv.size(0));
  a.Lk = static_cast<int>(qkv.size(1));
  a.H = static_cast<int>(H);
  a.hd = static_cast<int>(qkv.size(2) / 3 / H);
  a.Lq = static_cast<int>(Lq);
  a.causal = causal;
  a.ktail = static_cast<int>(ktail);
  a.kexcl = static_cast<int>(kexcl);
  a.scale = static_cast<float>(scale);
  a.err = optr<int>(err);
  TORCH_CHECK(qkv.size(2) == 3 * H * a.hd, "qkv width must be 3 * H * head_dim");
  TORCH_CHECK(out.numel() == static_cast<int64_t>(a.B) * Lq * H * a.hd, "out must be [B, Lq, D]");
  TORCH_CHECK(lse.numel() == static_cast<int64_t>(a.B) * H * Lq, "lse must be [B, H, Lq]");
  return a;
}

void fmha_fwd(const at::Tensor& qkv, const at::Tensor& kstart, const at::Tensor& out, const at::Tensor& lse, int64_t H,
              int64_t Lq, bool causal, double scale, const std::optional<at::Tensor>& err, int64_t ktail,
              int64_t kexcl) {
  c10::cuda::CUDAGuard guard(qkv.device());
  auto a = fmha_args(qkv, kstart, out, lse, H, Lq, causal, scale, err, ktail, kexcl);
  cudaError_t e = mdl::fmha_fwd(a, stream_of(qkv));
  if (e != cudaSuccess) throw std::runtime_error(std::string(mdl::fmha_last_error()) + ": " + cudaGetErrorString(e));
  g_launches += 1;
}

void fmha_bwd(const at::Tensor& qkv, const at::Tensor& kstart, const at::Tensor& out, const at::Tensor& lse,
              const at::Tensor& dout, const at::Tensor& dqkv, const at::Tensor& dq_acc, const at::Tensor& dsum,
              int64_t H, int64_t Lq, bool causal, double scale, const std::optional<at::Tensor>& err,
              int64_t ktail, int64_t kexcl) {
  c10::cuda::CUDAGuard guard(qkv.device());
  auto a = fmha_args(qkv, kstart, out, lse, H, Lq, causal, scale, err, ktail, kexcl);
  TORCH_CHECK(dout.scalar_type() == at::kBFloat16 && dout.is_contiguous() && dout.numel() == out.numel(),
              "dout must be contiguous bf16 like out");
  TORCH_CHECK(dqkv.scalar_type() == at::kBFloat16 && dqkv.is_contiguous() && dqkv.numel() == qkv.numel(),
              "dqkv must be contiguous bf16 like qkv");
  TORCH_CHECK(dq_acc.scalar_type() == at::kFloat && dq_acc.numel() >= out.numel(), "dq_acc must be fp32 [B, Lq, D]");
  TORCH_CHECK(dsum.scalar_type() == at::kFloat && dsum.numel() >= lse.numel(), "dsum must be fp32 [B, H, Lq]");
  a.dout = dout.data_ptr();
  a.dqkv = dqkv.data_ptr();
  a.dq_acc = dq_acc.data_ptr<float>();
  a.dsum = dsum.data_ptr<float>();
  cudaError_t e = mdl::fmha_bwd(a, stream_of(qkv));
  if (e != cudaSuccess) throw std::runtime_error(std::string(mdl::fmha_last_error()) + ": " + cudaGetErrorString(e));
  g_launches += 3;
}

// ------------------------------------------------------------------ CUDA-core attention (small heads)
mdl::AttnSimtArgs simt_args(const at::Tensor& qkv, const at::Tensor& kstart, const at::Tensor& out,
                            const at::Tensor& lse, int64_t H, int64_t Lq, bool causal, double scale, int64_t ktail,
                            int64_t kexcl) {
  require_cuda(qkv, "qkv");
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 3 && qkv.is_contiguous(), "qkv must be [B, Lk, 3D] bf16");
  TORCH_CHECK(kstart.scalar_type() == at::kInt && kstart.is_contiguous() && kstart.numel() == qkv.size(0),
              "kstart must be int32 [B]");
  TORCH_CHECK(qkv.size(2) % (3 * H) == 0, "qkv width must be 3 * H * head_dim");
  mdl::AttnSimtArgs a;
  a.B = static_cast<int>(qkv.size(0));
  a.Lk = static_cast<int>(qkv.size(1));
  a.H = static_cast<int>(H);
  a.hd = static_cast<int>(qkv.size(2) / 3 / H);
  a.Lq = static_cast<int>(Lq);
  TORCH_CHECK(mdl::attn_simt_supported(a.hd), "CUDA-core attention takes head widths 8, 16 and 64");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() &&
                  out.numel() == static_cast<int64_t>(a.B) * Lq * H * a.hd, "out must be bf16 [B, Lq, D]");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.numel() == static_cast<int64_t>(a.B) * H * Lq,
              "lse must be fp32 [B, H, Lq]");
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  a.kstart = kstart.data_ptr<int>();
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.causal = causal ? 1 : 0;
  a.ktail = static_cast<int>(ktail);
  a.kexcl = static_cast<int>(kexcl);
  a.scale = scale > 0 ? static_cast<float>(scale) : 1.f / std::sqrt(static_cast<float>(a.hd));
  return a;
}

void attn_simt_fwd(const at::Tensor& qkv, const at::Tensor& kstart, const at::Tensor& out, const at::Tensor& lse,
                   int64_t H, int64_t Lq, bool causal, double scale, int64_t ktail, int64_t kexcl) {
  c10::cuda::CUDAGuard guard(qkv.device());
  auto a = simt_args(qkv, kstart, out, lse, H, Lq, causal, scale, ktail, kexcl);
  check(mdl::attn_simt_fwd(a, stream_of(qkv)), "attn_simt_fwd");
  g_launches += 1;
}

void attn_simt_bwd(const at::Tensor& qkv, const at::Tensor& kstart, const at::Tensor& out, const at::Tensor& lse,
                   const at::Tensor& dout, const at::Tensor& dqkv, const at::Tensor& dsum, int64_t H, int64_t Lq,
                   bool causal, double scale, int64_t ktail, int64_t kexcl) {
  c10::cuda::CUDAGuard guard(qkv.device());
  auto a = simt_args(qkv, kstart, out, lse, H, Lq, causal, scale, ktail, kexcl);
  TORCH_CHECK(dout.scalar_type() == at::kBFloat16 && dout.is_contiguous() && dout.numel() == out.numel(),
              "dout must be contiguous bf16 like out");
  TORCH_CHECK(dqkv.scalar_type() == at::kBFloat16 && dqkv.is_contiguous() && dqkv.numel() == qkv.numel(),
              "dqkv must be contiguous bf16 like qkv");
  TORCH_CHECK(dsum.scalar_type() == at::kFloat && dsum.numel() >= lse.numel(), "dsum must be fp32 [B, H, Lq]");
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  a.dsum = dsum.data_ptr<float>();
  check(mdl::attn_simt_bwd(a, stream_of(qkv)), "attn_simt_bwd");
  g_launches += 3;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "mdl_b200 native sm_100a kernels";
  m.def("gemm_pair_mode", &mdl::gemm_pair_mode, "set the CTA-pair GEMM mode (-1 auto, 0 off, 1 on); returns the previous",
        py::arg("mode"));
  m.def("gemm", &gemm, "tcgen05 batched GEMM with fused epilogue", py::arg("A"), py::arg("lda"), py::arg("gsA"),
        py::arg("a_mn"), py::arg("B"), py::arg("ldb"), py::arg("gsB"), py::arg("b_mn"), py::arg("M"), py::arg("N"),
        py::arg("K"), py::arg("G"), py::arg("out"), py::arg("ldc"), py::arg("gsC"), py::arg("out2") = py::none(),
        py::arg("bias") = py::none(), py::arg("gs_bias") = 0, py::arg("aux") = py::none(), py::arg("ld_aux") = 0,
        py::arg("gs_aux") = 0, py::arg("colsum") = py::none(), py::arg("gs_colsum") = 0, py::arg("act") = 0,
        py::arg("alpha") = 1.0, py::arg("accumulate") = false, py::arg("err") = py::none(),
        py::arg("max_ctas") = 0, py::arg("KG") = 1, py::arg("ksA") = 0, py::arg("ksB") = 0);

  m.def("emb_forward", &emb_forward);
  m.def("emb_backward", &emb_backward);
  m.def("emb_route", &emb_route);
  m.def("emb_owner_forward", &emb_owner_forward);
  m.def("emb_owner_backward", &emb_owner_backward);
  m.def("emb_acc_to_bf16", &emb_acc_to_bf16);
  m.def("adagrad_apply", &adagrad_apply);
  m.def("touched_sqnorm", &touched_sqnorm);
  m.def("compact_touched", &compact_touched);
  m.def("ln_fwd", &ln_fwd);
  m.def("ln_bwd_grid", &ln_bwd_grid);
  m.def("ln_bwd", &ln_bwd, py::arg("dy"), py::arg("dy_bcast"), py::arg("bcast_scale"), py::arg("a"), py::arg("b"),
        py::arg("mean"), py::arg("rstd"), py::arg("gamma"), py::arg("dx"), py::arg("dx2"), py::arg("partials"),
        py::arg("dgamma"), py::arg("dbeta"), py::arg("B"), py::arg("T"), py::arg("D"), py::arg("mix"), py::arg("grid"),
        py::arg("res") = py::none());
  m.def("rms_fwd", &rms_fwd);
  m.def("rms_bwd", &rms_bwd, py::arg("x"), py::arg("w"), py::arg("rstd"), py::arg("dy"), py::arg("dx"), py::arg("dw"),
        py::arg("rows"), py::arg("D"), py::arg("dres") = py::none(), py::arg("res_period") = 0,
        py::arg("res_tail") = 0);
  m.def("token_mean", &token_mean);
  m.def("colsum", &colsum, py::arg("x"), py::arg("out"), py::arg("G"), py::arg("M"), py::arg("N"), py::arg("ld"),
        py::arg("gs"), py::arg("scale"), py::arg("gs_out") = -1);
  m.def("head_bce", &head_bce);
  m.def("adam", &adam);
  m.def("rmsprop", &rmsprop);
  m.def("sqnorm", &sqnorm);
  m.def("clip_factor", &clip_factor);
  m.def("cast_bf16", &cast_bf16);
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("ipc_free", &ipc_free);
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.def("set_barrier_limit", &set_barrier_limit);
  m.def("mbar_timeout_selftest", &mbar_timeout_selftest);
  m.def("barrier", &barrier);
  m.def("dense_sync", &dense_sync);
  m.def("small_allreduce", &small_allreduce);
  m.def("launch_count", &launch_count);
  m.def("small_attn_fwd", &small_attn_fwd);
  m.def("small_attn_bwd", &small_attn_bwd);
  m.def("attn_simt_fwd", &attn_simt_fwd, "suffix attention on CUDA cores (head widths 8, 16, 64)", py::arg("qkv"),
        py::arg("kstart"), py::arg("out"), py::arg("lse"), py::arg("H"), py::arg("Lq"), py::arg("causal"),
        py::arg("scale"), py::arg("ktail") = 0, py::arg("kexcl") = 0);
  m.def("attn_simt_bwd", &attn_simt_bwd, py::arg("qkv"), py::arg("kstart"), py::arg("out"), py::arg("lse"),
        py::arg("dout"), py::arg("dqkv"), py::arg("dsum"), py::arg("H"), py::arg("Lq"), py::arg("causal"),
        py::arg("scale"), py::arg("ktail") = 0, py::arg("kexcl") = 0);
  m.def("fmha_fwd", &fmha_fwd, py::arg("qkv"), py::arg("kstart"), py::arg("out"), py::arg("lse"), py::arg("H"),
        py::arg("Lq"), py::arg("causal"), py::arg("scale"), py::arg("err") = py::none(), py::arg("ktail") = 0,
        py::arg("kexcl") = 0);
  m.def("position_add", &position_add);
  m.def("position_grad", &position_grad);
  m.def("sqa_fwd", &sqa_fwd);
  m.def("sqa_shared_fwd", &sqa_shared_fwd);
  m.def("sqa_shared_bwd", &sqa_shared_bwd);
  m.def("sqa_shared_supported", [](int G, int D) { return mdl::sqa_shared_supported(G, D); });
  m.def("sqa_bwd", &sqa_bwd);
  m.def("fmha_bwd", &fmha_bwd, py::arg("qkv"), py::arg("kstart"), py::arg("out"), py::arg("lse"), py::arg("dout"),
        py::arg("dqkv"), py::arg("dq_acc"), py::arg("dsum"), py::arg("H"), py::arg("Lq"), py::arg("causal"),
        py::arg("scale"), py::arg("err") = py::none(), py::arg("ktail") = 0,
        py::arg("kexcl") = 0);
}
