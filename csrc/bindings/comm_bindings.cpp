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
}  // namespace

void register_comm_ops(py::module_& m) {
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
      .def("allreduce_adam",
           [](PeerMemory& p, int64_t grad_off, int64_t param_off, int64_t shadow_off, int64_t n, at::Tensor m1,
              at::Tensor m2, float lr, float b1, float b2, float eps, float wd, float grad_scale, at::Tensor step) {
             if (!m1.is_cuda() || m1.scalar_type() != at::kFloat || m1.numel() < n || !m2.is_cuda() ||
                 m2.numel() < n || step.scalar_type() != at::kLong)
               throw std::invalid_argument("allreduce_adam: bad state tensors");
             TbAdamParams hp{lr, b1, b2, eps, wd, grad_scale, 0.f, 0};
             cuda_ok(tb_peer_allreduce_adam(p.Table(), grad_off, param_off, shadow_off, n, m1.data_ptr<float>(),
                                            m2.data_ptr<float>(), hp,
                                            reinterpret_cast<const long long*>(step.data_ptr<int64_t>()),
                                            p.DoneCounter(), p.ErrorWord(), cur_stream(p.device())),
                     "peer_allreduce_adam");
           });
}
