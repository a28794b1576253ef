// Python bindings of PeerMemory and the NVLink peer-memory collectives.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include "kernels.h"
#include "turbol/common.hpp"
#include "turbol/peer.hpp"

namespace py = pybind11;
using turbol::PeerMemory;

namespace {
void cuda_ok(int e, const char* what) {
  if (e != 0) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(static_cast<cudaError_t>(e)));
}
cudaStream_t cur_stream(int dev) { return c10::cuda::getCurrentCUDAStream(dev).stream(); }

// Counters of one tensor-parallel communicator (int32 CUDA tensor [8]):
// [0] all-gather epoch, [1] all-gather CTA counter, [2] reduce-scatter epoch,
// [3] reduce-scatter CTA counter, [4..5] reduce-scatter arrival targets,
// [6] error word.
extern "C" void tb_tp_set_trace(void* p);
TbTpComm tp_comm(const PeerMemory& p, int64_t hdr_off, int64_t data_off, int64_t parity_bytes, int rows_per_rank,
                 const at::Tensor& ctr, bool rs) {
  if (!ctr.is_cuda() || ctr.scalar_type() != at::kInt || ctr.numel() < 8 || !ctr.is_contiguous())
    throw std::invalid_argument("tp: counters must be a contiguous int32 CUDA tensor [8]");
  const TbPeerTable t = p.Table();
  TbTpComm c{};
  c.rank = t.rank;
  c.world = t.world;
  c.rows_per_rank = rows_per_rank;
  auto* u = reinterpret_cast<unsigned*>(ctr.data_ptr<int>());
  c.epoch_ctr = rs ? u + 2 : u;
  c.done_ctr = rs ? u + 3 : u + 1;
  c.rs_target = u + 4;
  c.err = ctr.data_ptr<int>() + 6;
  for (int r = 0; r < t.world; ++r) {
    c.hdr[r] = static_cast<char*>(t.base[r]) + hdr_off;
    c.data[r] = static_cast<char*>(t.base[r]) + data_off;
  }
  c.parity_bytes = parity_bytes;
  return c;
}

TbGemmArgs tp_gemm_args(const at::Tensor& A, const at::Tensor& B, bool b_mn, int bn) {
  if (!A.is_cuda() || !B.is_cuda() || A.scalar_type() != at::kBFloat16 || B.scalar_type() != at::kBFloat16 ||
      A.dim() != 2 || B.dim() != 2 || A.stride(1) != 1 || B.stride(1) != 1)
    throw std::invalid_argument("tp gemm: A and B must be 2-D bf16 CUDA tensors with a contiguous last dim");
  TbGemmArgs a{};
  a.A = A.data_ptr();
  a.lda = A.stride(0);
  a.B = B.data_ptr();
  a.ldb = B.stride(0);
  a.b_mn = b_mn;
  a.K = static_cast<int>(A.size(1));
  a.N = static_cast<int>(b_mn ? B.size(1) : B.size(0));
  if ((b_mn ? B.size(0) : B.size(1)) != A.size(1)) throw std::invalid_argument("tp gemm: K mismatch");
  a.bn_hint = bn;
  return a;
}
}  // namespace

void register_comm_ops(py::module_& m) {
  m.def("peer_owned_slice", [](int64_t n, int rank, int world) {
    long long lo = 0, hi = 0;
    tb_peer_owned_slice(n, rank, world, &lo, &hi);
    return py::make_tuple(static_cast<int64_t>(lo), static_cast<int64_t>(hi));
  });
  m.def("tp_header_bytes", []() { return static_cast<int64_t>(tb_tp_header_bytes()); });
  m.def("bounded_wait_probe", [](at::Tensor flags, int64_t expect, double budget_s, at::Tensor err) {
    if (!flags.is_cuda() || flags.scalar_type() != at::kInt || !err.is_cuda() || err.scalar_type() != at::kInt)
      throw std::invalid_argument("bounded_wait_probe: int32 CUDA tensors");
    cuda_ok(tb_bounded_wait_probe(reinterpret_cast<const unsigned*>(flags.data_ptr<int>()),
                                  static_cast<int>(flags.numel()), static_cast<unsigned>(expect),
                                  static_cast<unsigned long long>(budget_s * 1e9), err.data_ptr<int>(),
                                  cur_stream(flags.device().index())),
            "bounded_wait_probe");
  }, py::arg("flags"), py::arg("expect"), py::arg("budget_s"), py::arg("err"));
  m.def("tp_set_trace", [](py::object t) {
    tb_tp_set_trace(t.is_none() ? nullptr : t.cast<at::Tensor>().data_ptr());
  });
  py::class_<PeerMemory>(m, "PeerMemory")
      .def(py::init<size_t, int>(), py::arg("payload_bytes"), py::arg("device"))
      .def("handle", [](const PeerMemory& p) { return py::bytes(p.Handle()); })
      .def("open",
           [](PeerMemory& p, const std::vector<py::bytes>& hs, int rank) {
             std::vector<std::string> v;
             for (auto& h : hs) v.push_back(h);
             p.Open(v, rank);
           },
           py::arg("handles"), py::arg("rank"))
      .def("payload_bytes", &PeerMemory::PayloadBytes)
      .def("rank", &PeerMemory::rank)
      .def("world", &PeerMemory::world)
      // zero-copy view of this rank's payload [offset, offset + numel * itemsize)
      .def("tensor",
           [](PeerMemory& p, int64_t offset, int64_t numel, py::object dtype) {
             const at::ScalarType st = torch::python::detail::py_object_to_dtype(dtype);
             const int64_t item = static_cast<int64_t>(c10::elementSize(st));
             if (offset < 0 || offset % 16 || static_cast<size_t>(offset + numel * item) > p.PayloadBytes())
               throw std::invalid_argument("PeerMemory.tensor: out of range or misaligned");
             void* ptr = static_cast<char*>(p.Payload()) + offset;
             return at::from_blob(ptr, {numel}, at::TensorOptions().dtype(st).device(at::kCUDA, p.device()));
           },
           py::arg("offset"), py::arg("numel"), py::arg("dtype"), py::keep_alive<0, 1>())
      .def("error", [](const PeerMemory& p) {
        int e = 0;
        cudaMemcpy(&e, p.ErrorWord(), sizeof(int), cudaMemcpyDeviceToHost);
        return e;
      })
      .def("clear_error", [](const PeerMemory& p) { cudaMemset(p.ErrorWord(), 0, sizeof(int)); })
      .def("allreduce",
           [](PeerMemory& p, int64_t in_off, int64_t out_off, int64_t n, float scale) {
             cuda_ok(tb_peer_allreduce(p.Table(), in_off, out_off, n, scale, p.DoneCounter(), p.ErrorWord(),
                                       cur_stream(p.device())),
                     "peer_allreduce");
           },
           py::arg("in_offset"), py::arg("out_offset"), py::arg("numel"), py::arg("scale") = 1.0f)
      .def("scatter_copy",
           [](PeerMemory& p, at::Tensor src0, at::Tensor src1, at::Tensor segs, int64_t total_vecs, int64_t dst_base) {
             static_assert(sizeof(TbCopySeg) == 8 * sizeof(int64_t), "TbCopySeg layout");
             if (!src0.is_cuda() || !src1.is_cuda() || !segs.is_cuda() || segs.scalar_type() != at::kLong ||
                 segs.dim() != 2 || segs.size(1) != 8 || !segs.is_contiguous())
               throw std::invalid_argument("scatter_copy: CUDA sources and int64 segments [n, 8] on the device");
             cuda_ok(tb_peer_scatter_copy(p.Table(), src0.data_ptr(), src1.data_ptr(),
                                          reinterpret_cast<const TbCopySeg*>(segs.data_ptr<int64_t>()),
                                          static_cast<int>(segs.size(0)), total_vecs, dst_base, p.DoneCounter(),
                                          p.ErrorWord(), cur_stream(p.device())),
                     "peer_scatter_copy");
           },
           py::arg("src0"), py::arg("src1"), py::arg("segs"), py::arg("total_vecs"), py::arg("dst_base") = 0)
      .def("payload_ptrs",
           [](const PeerMemory& p) {
             const TbPeerTable t = p.Table();
             std::vector<int64_t> v;
             for (int r = 0; r < t.world; ++r) v.push_back(reinterpret_cast<int64_t>(t.base[r]));
             return v;
           })
      // all-gather -> GEMM: out[M, N] = gather_rows(shard) . W^T  (+ epilogue)
      .def("tp_ag_gemm",
           [](PeerMemory& p, int64_t hdr_off, int64_t data_off, int64_t parity_bytes, at::Tensor ctr,
              at::Tensor shard, at::Tensor W, at::Tensor out, bool b_mn, py::object bias, py::object aux, int epi,
              int bn, py::object gather_out, py::object c2) {
             TbGemmArgs a = tp_gemm_args(shard, W, b_mn, bn);
             const int rows = static_cast<int>(shard.size(0));
             a.M = rows * p.world();
             if (!out.is_cuda() || out.dim() != 2 || out.stride(1) != 1 || out.size(0) != a.M ||
                 out.size(1) != (epi == TB_EPI_SWIGLU ? a.N / 2 : a.N))
               throw std::invalid_argument("tp_ag_gemm: out must be [world * rows, N]");
             a.C = out.data_ptr();
             a.ldc = out.stride(0);
             a.c_fp32 = out.scalar_type() == at::kFloat;
             a.epi = epi;
             at::Tensor b, x;
             if (!bias.is_none()) {
               b = bias.cast<at::Tensor>();
               a.bias = b.data_ptr<float>();
             }
             if (!aux.is_none()) {
               x = aux.cast<at::Tensor>();
               a.aux = x.data_ptr();
               a.ld_aux = x.stride(0);
             }
             TbTpComm c = tp_comm(p, hdr_off, data_off, parity_bytes, rows, ctr, false);
             at::Tensor g;
             if (!gather_out.is_none()) {
               g = gather_out.cast<at::Tensor>();
               if (!g.is_cuda() || g.scalar_type() != at::kBFloat16 || g.dim() != 2 || g.stride(1) != 1 ||
                   g.size(0) != a.M || g.size(1) != a.K)
                 throw std::invalid_argument("tp_ag_gemm: gather_out must be bf16 [world * rows, K]");
               c.gather_out = g.data_ptr();
               c.ld_gather = g.stride(0);
             }
             at::Tensor raw;
             if (!c2.is_none()) {
               raw = c2.cast<at::Tensor>();
               if (epi != TB_EPI_SWIGLU || !raw.is_cuda() || raw.scalar_type() != at::kBFloat16 || raw.dim() != 2 ||
                   raw.stride(1) != 1 || raw.size(0) != a.M || raw.size(1) != a.N)
                 throw std::invalid_argument("tp_ag_gemm: c2 (EPI_SWIGLU only) must be bf16 [world * rows, N]");
               a.C2 = raw.data_ptr();
               a.ldc2 = raw.stride(0);
             }
             a.error = c.err;
             cuda_ok(tb_tp_ag_gemm(&c, &a, cur_stream(p.device())), "tp_ag_gemm");
           },
           py::arg("hdr_off"), py::arg("data_off"), py::arg("parity_bytes"), py::arg("ctr"), py::arg("shard"),
           py::arg("W"), py::arg("out"), py::arg("b_mn") = false, py::arg("bias") = py::none(),
           py::arg("aux") = py::none(), py::arg("epi") = 0, py::arg("bn") = 0, py::arg("gather_out") = py::none(),
           py::arg("c2") = py::none())
      // GEMM -> reduce-scatter: out[M / world, N] = rows of sum_r(A_r . W_r^T) (+ bias) (+ residual)
      .def("tp_gemm_rs",
           [](PeerMemory& p, int64_t hdr_off, int64_t data_off, int64_t parity_bytes, at::Tensor ctr, at::Tensor A,
              at::Tensor W, at::Tensor out, bool b_mn, py::object bias, py::object residual, int bn) {
             TbGemmArgs a = tp_gemm_args(A, W, b_mn, bn);
             a.M = static_cast<int>(A.size(0));
             if (a.M % p.world()) throw std::invalid_argument("tp_gemm_rs: rows must divide by the world size");
             const int rows = a.M / p.world();
             if (!out.is_cuda() || out.scalar_type() != at::kBFloat16 || out.dim() != 2 || out.stride(1) != 1 ||
                 out.size(0) != rows || out.size(1) != a.N)
               throw std::invalid_argument("tp_gemm_rs: out must be bf16 [M / world, N]");
             a.epi = TB_EPI_NONE;
             at::Tensor b, r;
             const float* bp = nullptr;
             const void* rp = nullptr;
             int64_t ldr = 0;
             if (!bias.is_none()) {
               b = bias.cast<at::Tensor>();
               bp = b.data_ptr<float>();
             }
             if (!residual.is_none()) {
               r = residual.cast<at::Tensor>();
               if (r.scalar_type() != at::kBFloat16 || r.size(0) != rows || r.size(1) != a.N || r.stride(1) != 1)
                 throw std::invalid_argument("tp_gemm_rs: residual must be bf16 [M / world, N]");
               rp = r.data_ptr();
               ldr = r.stride(0);
             }
             TbTpComm c = tp_comm(p, hdr_off, data_off, parity_bytes, rows, ctr, true);
             a.error = c.err;
             cuda_ok(tb_tp_gemm_rs(&c, &a, out.data_ptr(), out.stride(0), bp, rp, ldr, cur_stream(p.device())),
                     "tp_gemm_rs");
           },
           py::arg("hdr_off"), py::arg("data_off"), py::arg("parity_bytes"), py::arg("ctr"), py::arg("A"),
           py::arg("W"), py::arg("out"), py::arg("b_mn") = false, py::arg("bias") = py::none(),
           py::arg("residual") = py::none(), py::arg("bn") = 0)
      .def("allreduce_adam",
           [](PeerMemory& p, int64_t grad_off, int64_t param_off, int64_t shadow_off, int64_t n, at::Tensor m1,
              at::Tensor m2, float lr, float b1, float b2, float eps, float wd, float grad_scale, at::Tensor step) {
             long long lo = 0, hi = 0;
             tb_peer_owned_slice(n, p.rank(), p.world(), &lo, &hi);
             if (!m1.is_cuda() || m1.scalar_type() != at::kFloat || m1.numel() < hi - lo || !m2.is_cuda() ||
                 m2.scalar_type() != at::kFloat || m2.numel() < hi - lo || step.scalar_type() != at::kLong)
               throw std::invalid_argument("allreduce_adam: m and v must be fp32 CUDA tensors of the owned shard");
             TbAdamParams hp{lr, b1, b2, eps, wd, grad_scale, 0.f, 0};
             cuda_ok(tb_peer_allreduce_adam(p.Table(), grad_off, param_off, shadow_off, n, m1.data_ptr<float>(),
                                            m2.data_ptr<float>(), hp,
                                            reinterpret_cast<const long long*>(step.data_ptr<int64_t>()),
                                            p.DoneCounter(), p.ErrorWord(), cur_stream(p.device())),
                     "peer_allreduce_adam");
           })
      .def("allreduce_adam_rep",
           [](PeerMemory& p, int64_t grad_off, int64_t send_off, int64_t param_off, int64_t shadow_off, int64_t n,
              at::Tensor m1, at::Tensor m2, float lr, float b1, float b2, float eps, float wd, float grad_scale,
              at::Tensor step) {
             if (!m1.is_cuda() || m1.scalar_type() != at::kFloat || m1.numel() < n || !m2.is_cuda() ||
                 m2.scalar_type() != at::kFloat || m2.numel() < n || step.scalar_type() != at::kLong)
               throw std::invalid_argument("allreduce_adam_rep: m and v must be fp32 CUDA tensors of the whole vector");
             TbAdamParams hp{lr, b1, b2, eps, wd, grad_scale, 0.f, 0};
             cuda_ok(tb_peer_allreduce_adam_rep(p.Table(), grad_off, send_off, param_off, shadow_off, n,
                                                m1.data_ptr<float>(), m2.data_ptr<float>(), hp,
                                                reinterpret_cast<const long long*>(step.data_ptr<int64_t>()),
                                                p.RepEpoch(), p.DoneCounter(), p.ErrorWord(), cur_stream(p.device())),
                     "peer_allreduce_adam_rep");
           });
}
