// torch-tensor entry points of the tensor-core GEMM and the LLM kernels.
#include <pybind11/pybind11.h>
#include <torch/extension.h>

#include "kernels.h"
#include "turbol/common.hpp"

namespace py = pybind11;

namespace {

void chk(bool c, const std::string& m) {
  if (!c) throw std::invalid_argument(m);
}
void cuda_ok(int e, const char* what) {
  if (e != 0) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(static_cast<cudaError_t>(e)));
}

// C = epi(A . B^T) with A [M,K] (a_mn=0) or [K,M] (a_mn=1), B [N,K] (b_mn=0) or [K,N] (b_mn=1).
void gemm(const at::Tensor& A, const at::Tensor& B, at::Tensor C, bool a_mn, bool b_mn, py::object bias,
          py::object aux, int epi, bool accumulate, float alpha, int split_k, int bn, py::object err,
          py::object workspace, py::object colsum) {
  chk(A.is_cuda() && B.is_cuda() && C.is_cuda(), "gemm: CUDA tensors required");
  chk(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm: A and B must be bfloat16");
  chk(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "gemm: 2-D operands");
  chk(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "gemm: last dim must be contiguous");
  const int64_t M = a_mn ? A.size(1) : A.size(0);
  const int64_t K = a_mn ? A.size(0) : A.size(1);
  const int64_t N = b_mn ? B.size(1) : B.size(0);
  const int64_t Kb = b_mn ? B.size(0) : B.size(1);
  chk(K == Kb, "gemm: K mismatch");
  chk(C.size(0) == M && C.size(1) == (epi == TB_EPI_SWIGLU ? N / 2 : N), "gemm: C shape mismatch");
  chk(C.scalar_type() == at::kFloat || C.scalar_type() == at::kBFloat16, "gemm: C must be fp32 or bf16");
  TbGemmArgs a{};
  a.A = A.data_ptr();
  a.lda = A.stride(0);
  a.a_mn = a_mn;
  a.B = B.data_ptr();
  a.ldb = B.stride(0);
  a.b_mn = b_mn;
  a.C = C.data_ptr();
  a.ldc = C.stride(0);
  a.c_fp32 = C.scalar_type() == at::kFloat;
  a.c_accumulate = accumulate;
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.K = static_cast<int>(K);
  at::Tensor b, x;
  if (!bias.is_none()) {
    b = bias.cast<at::Tensor>();
    chk(b.scalar_type() == at::kFloat && b.is_contiguous() && b.numel() == N, "gemm: bias must be fp32 [N]");
    a.bias = b.data_ptr<float>();
  }
  if (!aux.is_none()) {
    x = aux.cast<at::Tensor>();
    chk(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1 && x.size(0) == M && x.size(1) == N,
        "gemm: aux must be bf16 [M, N]");
    a.aux = x.data_ptr();
    a.ld_aux = x.stride(0);
  }
  a.epi = epi;
  a.alpha = alpha;
  a.split_k = split_k;
  a.bn_hint = bn;
  if (!err.is_none()) a.error = err.cast<at::Tensor>().data_ptr<int>();
  at::Tensor ws, cs;
  if (!workspace.is_none()) {
    ws = workspace.cast<at::Tensor>();
    chk(ws.is_cuda() && ws.is_contiguous(), "gemm: workspace must be a contiguous CUDA tensor");
    a.workspace = ws.data_ptr();
    a.workspace_bytes = ws.nbytes();
  }
  if (!colsum.is_none()) {
    cs = colsum.cast<at::Tensor>();
    chk(cs.scalar_type() == at::kFloat && cs.is_contiguous() && cs.numel() == N, "gemm: colsum must be fp32 [N]");
    a.colsum = cs.data_ptr<float>();
  }
  cuda_ok(tb_gemm_bf16(&a, turbol::StreamFor(C)), "gemm_bf16");
}

}  // namespace

void register_llm_ops(py::module_& m) {
  m.def("gemm", &gemm, py::arg("A"), py::arg("B"), py::arg("C"), py::arg("a_mn") = false, py::arg("b_mn") = false,
        py::arg("bias") = py::none(), py::arg("aux") = py::none(), py::arg("epi") = 0, py::arg("accumulate") = false,
        py::arg("alpha") = 1.0f, py::arg("split_k") = 0, py::arg("bn") = 0, py::arg("error") = py::none(),
        py::arg("workspace") = py::none(), py::arg("colsum") = py::none());
  m.def("gemm_workspace_numel", [](int M, int N, int K) {
    return static_cast<int64_t>(tb_gemm_workspace_bytes(M, N, K) / 4);
  });
  m.attr("EPI_NONE") = static_cast<int>(TB_EPI_NONE);
  m.attr("EPI_BIAS") = static_cast<int>(TB_EPI_BIAS);
  m.attr("EPI_BIAS_TANH") = static_cast<int>(TB_EPI_BIAS_TANH);
  m.attr("EPI_BIAS_SILU") = static_cast<int>(TB_EPI_BIAS_SILU);
  m.attr("EPI_TANH_BWD") = static_cast<int>(TB_EPI_TANH_BWD);
  m.attr("EPI_RESIDUAL") = static_cast<int>(TB_EPI_RESIDUAL);
  m.attr("EPI_SWIGLU") = static_cast<int>(TB_EPI_SWIGLU);
}
