// Python bindings of the C++ distributed runtime (turbol/distributed.hpp):
// submodule `turbol_core.dist` with NcclCommunicator, DistributedConfig,
// DistributedTrainer, PipelineConfig and PipelineTrainer.  Tensors are torch
// CUDA tensors (shared zero-copy with the C++ Tensor); pipeline stage
// functions are Python callables, invoked with the GIL held.
#include <pybind11/functional.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include "turbol/distributed.hpp"

namespace py = pybind11;
using namespace turbol;
using namespace turbol::distributed;

namespace {

Status need_cuda(const at::Tensor& t, const char* what) {
  if (!t.is_cuda() || !t.is_contiguous())
    return Status::InvalidArgument(std::string(what) + ": a contiguous CUDA tensor is required");
  return Status::Ok();
}

bool mean_op(const std::string& op, Status* st) {
  if (op != "sum" && op != "mean") *st = Status::InvalidArgument("op must be \"sum\" or \"mean\"");
  return op == "mean";
}

}  // namespace

void register_dist(py::module_& m) {
  py::enum_<ParallelStrategy>(m, "ParallelStrategy")
      .value("kDataParallel", ParallelStrategy::kDataParallel)
      .value("kModelParallel", ParallelStrategy::kModelParallel)
      .value("kPipelineParallel", ParallelStrategy::kPipelineParallel);

  py::class_<NcclCommunicator>(m, "NcclCommunicator")
      .def(py::init<>())
      .def_static("instance", &NcclCommunicator::Instance, py::return_value_policy::reference)
      .def("initialize", &NcclCommunicator::Initialize, py::arg("rank"), py::arg("world_size"), py::arg("device_id") = 0,
           py::arg("master_addr") = "127.0.0.1", py::arg("master_port") = 29500, py::arg("timeout_s") = 120.0,
           py::arg("key") = "turbol/nccl_id", py::call_guard<py::gil_scoped_release>())
      .def("shutdown", &NcclCommunicator::Shutdown)
      .def("abort", &NcclCommunicator::Abort)
      .def("all_reduce",
           [](NcclCommunicator& c, at::Tensor t, const std::string& op) {
             Status st = need_cuda(t, "all_reduce");
             const bool mean = mean_op(op, &st);
             if (!st.ok()) return st;
             return c.AllReduce(t.data_ptr(), t.data_ptr(), static_cast<size_t>(t.numel()), mean,
                                FromTorch(t.scalar_type()));
           },
           py::arg("tensor"), py::arg("op") = "sum")
      .def("reduce_scatter",
           [](NcclCommunicator& c, at::Tensor in, at::Tensor out, const std::string& op) {
             Status st = need_cuda(in, "reduce_scatter");
             if (st.ok()) st = need_cuda(out, "reduce_scatter");
             const bool mean = mean_op(op, &st);
             if (st.ok() && in.numel() != out.numel() * c.world_size())
               st = Status::InvalidArgument("reduce_scatter: in must hold world_size x out elements");
             if (!st.ok()) return st;
             return c.ReduceScatter(in.data_ptr(), out.data_ptr(), static_cast<size_t>(out.numel()), mean,
                                    FromTorch(in.scalar_type()));
           },
           py::arg("input"), py::arg("output"), py::arg("op") = "sum")
      .def("all_gather",
           [](NcclCommunicator& c, at::Tensor in, at::Tensor out) {
             Status st = need_cuda(in, "all_gather");
             if (st.ok()) st = need_cuda(out, "all_gather");
             if (st.ok() && out.numel() != in.numel() * c.world_size())
               st = Status::InvalidArgument("all_gather: out must hold world_size x in elements");
             if (!st.ok()) return st;
             return c.AllGather(in.data_ptr(), out.data_ptr(), static_cast<size_t>(in.numel()),
                                FromTorch(in.scalar_type()));
           },
           py::arg("input"), py::arg("output"))
      .def("broadcast",
           [](NcclCommunicator& c, at::Tensor t, int root) {
             Status st = need_cuda(t, "broadcast");
             if (!st.ok()) return st;
             return c.Broadcast(t.data_ptr(), t.data_ptr(), static_cast<size_t>(t.numel()), root,
                                FromTorch(t.scalar_type()));
           },
           py::arg("tensor"), py::arg("root") = 0)
      .def("send",
           [](NcclCommunicator& c, at::Tensor t, int peer) {
             Status st = need_cuda(t, "send");
             if (!st.ok()) return st;
             return c.Send(t.data_ptr(), static_cast<size_t>(t.numel()), peer, FromTorch(t.scalar_type()));
           },
           py::arg("tensor"), py::arg("peer"))
      .def("recv",
           [](NcclCommunicator& c, at::Tensor t, int peer) {
             Status st = need_cuda(t, "recv");
             if (!st.ok()) return st;
             return c.Recv(t.data_ptr(), static_cast<size_t>(t.numel()), peer, FromTorch(t.scalar_type()));
           },
           py::arg("tensor"), py::arg("peer"))
      .def("group_start", &NcclCommunicator::GroupStart)
      .def("group_end", &NcclCommunicator::GroupEnd)
      .def("barrier", &NcclCommunicator::Barrier, py::call_guard<py::gil_scoped_release>())
      .def_property_readonly("rank", &NcclCommunicator::rank)
      .def_property_readonly("world_size", &NcclCommunicator::world_size)
      .def_property_readonly("device", &NcclCommunicator::device)
      .def("is_initialized", &NcclCommunicator::is_initialized);

  py::class_<DistributedConfig>(m, "DistributedConfig")
      .def(py::init<>())
      .def_readwrite("strategy", &DistributedConfig::strategy)
      .def_readwrite("world_size", &DistributedConfig::world_size)
      .def_readwrite("rank", &DistributedConfig::rank)
      .def_readwrite("master_addr", &DistributedConfig::master_addr)
      .def_readwrite("master_port", &DistributedConfig::master_port)
      .def_readwrite("use_nccl", &DistributedConfig::use_nccl)
      .def_readwrite("device_id", &DistributedConfig::device_id)
      .def_readwrite("timeout_s", &DistributedConfig::timeout_s);

  py::class_<DistributedTrainer>(m, "DistributedTrainer")
      .def(py::init<const DistributedConfig&>(), py::arg("config") = DistributedConfig())
      .def("initialize", &DistributedTrainer::Initialize, py::call_guard<py::gil_scoped_release>())
      .def("shutdown", &DistributedTrainer::Shutdown)
      .def("all_reduce",
           [](DistributedTrainer& d, at::Tensor t, const std::string& op) {
             Tensor tt(t);  // shares t's storage
             return d.AllReduce(&tt, op);
           },
           py::arg("tensor"), py::arg("op") = "sum")
      .def("broadcast",
           [](DistributedTrainer& d, at::Tensor t, int root) {
             Tensor tt(t);
             return d.Broadcast(&tt, root);
           },
           py::arg("tensor"), py::arg("root_rank") = 0)
      .def("barrier", &DistributedTrainer::Barrier, py::call_guard<py::gil_scoped_release>())
      .def("get_rank", &DistributedTrainer::GetRank)
      .def("get_world_size", &DistributedTrainer::GetWorldSize)
      .def("communicator", &DistributedTrainer::communicator, py::return_value_policy::reference_internal);

  py::class_<PipelineConfig>(m, "PipelineConfig")
      .def(py::init<>())
      .def_readwrite("num_pipeline_stages", &PipelineConfig::num_pipeline_stages)
      .def_readwrite("num_microbatches", &PipelineConfig::num_microbatches)
      .def_readwrite("stage_id", &PipelineConfig::stage_id)
      .def_readwrite("num_warmup_microbatches", &PipelineConfig::num_warmup_microbatches)
      .def_readwrite("microbatch_seq_len", &PipelineConfig::microbatch_seq_len)
      .def_readwrite("microbatch_batch_sz", &PipelineConfig::microbatch_batch_sz)
      .def_readwrite("hidden_size", &PipelineConfig::hidden_size)
      .def_readwrite("max_cache_seq_len", &PipelineConfig::max_cache_seq_len)
      .def_readwrite("activation_checkpointing", &PipelineConfig::activation_checkpointing)
      .def_readwrite("checkpoint_every_n_layers", &PipelineConfig::checkpoint_every_n_layers);

  py::class_<PipelineTrainer>(m, "PipelineTrainer")
      .def(py::init<const PipelineConfig&>(), py::arg("config"))
      .def("initialize",
           [](PipelineTrainer& p, NcclCommunicator* comm, py::object input, py::object forward, py::object loss,
              py::object backward, py::object recompute, const std::string& dtype) {
             StageFunctions f;
             if (!input.is_none()) {
               auto fn = input.cast<py::function>();
               f.input = [fn](int i) { return fn(i).cast<at::Tensor>(); };
             }
             auto fw = forward.cast<py::function>();
             f.forward = [fw](int i, const at::Tensor& x) { return fw(i, x).cast<at::Tensor>(); };
             if (!loss.is_none()) {
               auto fn = loss.cast<py::function>();
               f.loss = [fn](int i, const at::Tensor& x) {
                 py::tuple r = fn(i, x);
                 return std::make_pair(r[0].cast<float>(), r[1].cast<at::Tensor>());
               };
             }
             auto bw = backward.cast<py::function>();
             f.backward = [bw](int i, const at::Tensor& d) { return bw(i, d).cast<at::Tensor>(); };
             if (!recompute.is_none()) {
               auto fn = recompute.cast<py::function>();
               f.recompute = [fn](int i, const at::Tensor& x) { fn(i, x); };
             }
             const at::ScalarType dt = dtype == "float32" ? at::kFloat : at::kBFloat16;
             return p.Initialize(comm, std::move(f), dt);
           },
           py::arg("comm"), py::arg("input") = py::none(), py::arg("forward"), py::arg("loss") = py::none(),
           py::arg("backward"), py::arg("recompute") = py::none(), py::arg("dtype") = "bfloat16")
      .def("shutdown", &PipelineTrainer::Shutdown)
      .def("training_step",
           [](PipelineTrainer& p) {
             float loss = 0.f;
             Status st = p.TrainingStep(&loss);
             return py::make_tuple(st, loss);
           })
      .def("forward",
           [](PipelineTrainer& p) {
             std::vector<at::Tensor> outs;
             Status st = p.Forward(&outs);
             return py::make_tuple(st, outs);
           })
      .def("last_order", &PipelineTrainer::LastOrder)
      .def("current_step", &PipelineTrainer::CurrentStep);
}
