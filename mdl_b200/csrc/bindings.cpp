// Python bindings of the mdl_b200 native kernels. This is the only
// translation unit that includes torch headers; the kernels themselves live in
// the .cu files and take raw pointers plus a cudaStream_t.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <optional>
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace {

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
          int64_t max_ctas) {
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
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "mdl_b200 native sm_100a kernels";
  m.def("gemm", &gemm, "tcgen05 batched GEMM with fused epilogue", py::arg("A"), py::arg("lda"), py::arg("gsA"),
        py::arg("a_mn"), py::arg("B"), py::arg("ldb"), py::arg("gsB"), py::arg("b_mn"), py::arg("M"), py::arg("N"),
        py::arg("K"), py::arg("G"), py::arg("out"), py::arg("ldc"), py::arg("gsC"), py::arg("out2") = py::none(),
        py::arg("bias") = py::none(), py::arg("gs_bias") = 0, py::arg("aux") = py::none(), py::arg("ld_aux") = 0,
        py::arg("gs_aux") = 0, py::arg("colsum") = py::none(), py::arg("gs_colsum") = 0, py::arg("act") = 0,
        py::arg("alpha") = 1.0, py::arg("accumulate") = false, py::arg("err") = py::none(),
        py::arg("max_ctas") = 0);
}
