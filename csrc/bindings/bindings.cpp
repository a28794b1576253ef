// pybind11 module turbol_b200.turbol_core: the host runtime classes and the
// raw kernel ops (submodule `ops`).
//
// Parity: the class and method names follow the reference's
// turbol_vllm/python/turbol/pybind11_bindings.cpp:114-510 (Status, Shape,
// Tensor, GPUEnvironment, RingBuffer, Config, RewardConfig/Result/Engine,
// SpanID, ProfilerGuard, ProfilerConfig, Profiler, AggregatedStats,
// TensorBoardWriter, Labels, PrometheusWriter, get_version,
// get_device_count, get_memory_info).  Additions: zero-copy torch/DLPack
// exchange on Tensor, CartPole and prioritized replay, Dataset/ByteTokenizer,
// TcpStore, PipelineSchedule, KVBlockManager, CoreEngine, TensorUtils.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

#include <sstream>

#include "turbol/common.hpp"
#include "turbol/config.hpp"
#include "turbol/engines.hpp"
#include "turbol/observability.hpp"
#include "turbol/runtime.hpp"

namespace py = pybind11;
using namespace turbol;

void register_kernel_ops(py::module_& ops);  // ops_bindings.cpp
void register_llm_ops(py::module_& ops);      // llm_bindings.cpp
void register_comm_ops(py::module_& ops);     // comm_bindings.cpp
void register_dist(py::module_& m);           // dist_bindings.cpp

namespace {

void throw_if(const Status& s) {
  if (!s.ok()) {
    if (s.code() == StatusCode::kInvalidArgument) throw std::invalid_argument(s.message());
    if (s.code() == StatusCode::kTimeout) throw std::runtime_error("Timeout: " + s.message());
    throw std::runtime_error(s.ToString());
  }
}

py::object tensor_to_numpy(const Tensor& t) {
  if (!t.defined()) return py::none();
  py::object tt = py::cast(t.torch());
  if (t.is_cuda()) return tt.attr("cpu")().attr("numpy")();
  return tt.attr("numpy")();  // zero-copy, writable view on CPU
}

Tensor make_tensor(py::object shape, const std::string& dtype, const std::string& device) {
  std::vector<int64_t> dims;
  for (auto h : shape) dims.push_back(h.cast<int64_t>());
  return Tensor(Shape(dims), ParseDataType(dtype), Device::Parse(device));
}

EnvType parse_env(const std::string& s) {
  if (s == "linear" || s == "LinearEnv" || s == "Linear") return EnvType::kLinear;
  if (s == "cartpole" || s == "CartPole" || s == "CartPole-v1") return EnvType::kCartPole;
  throw std::invalid_argument("unknown env_type: " + s);
}

}  // namespace

PYBIND11_MODULE(turbol_core, m) {
  m.doc() = "turbol_b200 native core (B200 / sm_100a)";

  py::enum_<StatusCode>(m, "StatusCode")
      .value("kOk", StatusCode::kOk)
      .value("kInvalidArgument", StatusCode::kInvalidArgument)
      .value("kNotFound", StatusCode::kNotFound)
      .value("kAlreadyExists", StatusCode::kAlreadyExists)
      .value("kResourceExhausted", StatusCode::kResourceExhausted)
      .value("kUnimplemented", StatusCode::kUnimplemented)
      .value("kInternalError", StatusCode::kInternalError)
      .value("kUnavailable", StatusCode::kUnavailable)
      .value("kTimeout", StatusCode::kTimeout)
      .value("kCudaError", StatusCode::kCudaError);
  // this library's earlier names for codes 4 and 5
  m.attr("StatusCode").attr("kOutOfMemory") = StatusCode::kResourceExhausted;
  m.attr("StatusCode").attr("kNotImplemented") = StatusCode::kUnimplemented;

  py::class_<Status>(m, "Status")
      .def(py::init<>())
      .def(py::init<StatusCode, std::string>(), py::arg("code"), py::arg("message") = "")
      .def("ok", &Status::ok)
      .def("code", [](const Status& s) { return static_cast<int>(s.code()); })
      .def("message", &Status::message)
      .def("__bool__", &Status::ok)
      .def("__repr__", &Status::ToString);

  py::class_<Shape>(m, "Shape")
      .def(py::init<>())
      .def(py::init<std::vector<int64_t>>())
      .def("__len__", &Shape::size)
      .def("__getitem__",
           [](const Shape& s, py::ssize_t i) {
             if (i < 0) i += static_cast<py::ssize_t>(s.size());
             if (i < 0 || static_cast<size_t>(i) >= s.size()) throw py::index_error();
             return s.dims[static_cast<size_t>(i)];
           })
      .def("__eq__", [](const Shape& a, const Shape& b) { return a == b; })
      .def("numel", &Shape::numel)
      .def("to_list", [](const Shape& s) { return s.dims; })
      .def("__repr__", &Shape::ToString);

  py::class_<Tensor>(m, "Tensor")
      .def(py::init<>())
      .def(py::init(&make_tensor), py::arg("shape"), py::arg("dtype") = "float32", py::arg("device") = "cpu")
      .def_static("from_torch", [](const at::Tensor& t) { return Tensor(t); }, py::arg("tensor"),
                  "Adopts a torch tensor's storage (zero-copy when contiguous).")
      .def("numel", &Tensor::numel)
      .def("shape", &Tensor::shape)
      .def("dtype", [](const Tensor& t) { return DataTypeName(t.dtype()); })
      .def("device", [](const Tensor& t) { return t.device().ToString(); })
      .def("is_cuda", &Tensor::is_cuda)
      .def("size_bytes", &Tensor::size_bytes)
      .def("clone", &Tensor::Clone)
      .def("to_numpy", &tensor_to_numpy)
      .def("to_device", [](Tensor& t, const std::string& d) { return t.ToDevice(Device::Parse(d)); }, py::arg("device"))
      .def("copy_from", [](Tensor& t, const Tensor& s) { throw_if(t.CopyFrom(s)); })
      .def("set_", [](Tensor& t, const at::Tensor& x) { t = Tensor(x); }, py::arg("tensor"),
           "Rebinds this Tensor to `tensor`'s storage (out-parameter helper).")
      .def("torch", [](Tensor& t) { return t.torch(); }, "Zero-copy torch view of the storage.")
      .def("__dlpack__",
           [](Tensor& t, py::args args, py::kwargs kw) { return py::cast(t.torch()).attr("__dlpack__")(*args, **kw); })
      .def("__dlpack_device__", [](Tensor& t) { return py::cast(t.torch()).attr("__dlpack_device__")(); })
      .def_property_readonly("__cuda_array_interface__",
                             [](Tensor& t) { return py::cast(t.torch()).attr("__cuda_array_interface__"); })
      .def("__repr__", [](const Tensor& t) {
        std::ostringstream o;
        o << "turbol.Tensor(" << t.shape().ToString() << ", " << DataTypeName(t.dtype()) << ", "
          << t.device().ToString() << ")";
        return o.str();
      });

  // ---------------- environments ----------------
  py::class_<CartPoleConfig>(m, "CartPoleConfig")
      .def(py::init<>())
      .def_readwrite("gravity", &CartPoleConfig::gravity)
      .def_readwrite("masscart", &CartPoleConfig::masscart)
      .def_readwrite("masspole", &CartPoleConfig::masspole)
      .def_readwrite("length", &CartPoleConfig::length)
      .def_readwrite("force_mag", &CartPoleConfig::force_mag)
      .def_readwrite("tau", &CartPoleConfig::tau)
      .def_readwrite("x_threshold", &CartPoleConfig::x_threshold)
      .def_readwrite("theta_threshold", &CartPoleConfig::theta_threshold)
      .def_readwrite("init_range", &CartPoleConfig::init_range)
      .def_readwrite("max_steps", &CartPoleConfig::max_steps);

  py::class_<GPUEnvironment>(m, "GPUEnvironment")
      .def(py::init([](int n, int od, int ad, const std::string& dev, const std::string& type, uint64_t seed) {
             return new GPUEnvironment(n, od, ad, Device::Parse(dev), parse_env(type), seed);
           }),
           py::arg("num_envs") = 1, py::arg("obs_dim") = 4, py::arg("act_dim") = 2, py::arg("device") = "cpu",
           py::arg("env_type") = "linear", py::arg("seed") = 42)
      .def("reset", &GPUEnvironment::Reset)
      .def("step",
           [](GPUEnvironment& e, py::object action) {
             Tensor o, r, d;
             if (py::isinstance<Tensor>(action)) {
               throw_if(e.Step(action.cast<Tensor&>(), &o, &r, &d));  // by reference: no copy
             } else {
               throw_if(e.Step(Tensor(action.cast<at::Tensor>()), &o, &r, &d));
             }
             return py::make_tuple(std::move(o), std::move(r), std::move(d));
           },
           py::arg("action"))
      .def("step_into",
           [](GPUEnvironment& e, const at::Tensor& a, at::Tensor o, at::Tensor r, at::Tensor d) {
             throw_if(e.StepInto(a, o, r, d));
           },
           py::arg("action"), py::arg("obs"), py::arg("reward"), py::arg("done"))
      .def("observe", &GPUEnvironment::Observe)
      .def("state", [](GPUEnvironment& e) { return e.StateTensor(); }, "Live state tensor (no copy).")
      .def("episode_buffers",
           [](GPUEnvironment& e) { return py::make_tuple(e.EpLen(), e.EpRet(), e.EpCount(), e.StatsTensor()); })
      .def("take_episode_stats", &GPUEnvironment::TakeEpisodeStats)
      .def("num_envs", &GPUEnvironment::NumEnvs)
      .def("obs_dim", &GPUEnvironment::ObsDim)
      .def("act_dim", &GPUEnvironment::ActDim)
      .def("obs_shape", &GPUEnvironment::ObsShape)
      .def("act_shape", &GPUEnvironment::ActionShape)
      .def("env_type", [](const GPUEnvironment& e) { return e.type() == EnvType::kCartPole ? "cartpole" : "linear"; })
      .def("seed", &GPUEnvironment::seed)
      .def("decay", &GPUEnvironment::decay)
      .def("force", &GPUEnvironment::force)
      .def("done_threshold", &GPUEnvironment::done_threshold)
      .def("cartpole_config", &GPUEnvironment::cartpole, py::return_value_policy::reference_internal);

  // ---------------- replay ----------------
  py::class_<RingBuffer>(m, "RingBuffer")
      .def(py::init([](int64_t cap, int od, int ad, const std::string& dev, uint64_t seed) {
             return new RingBuffer(cap, od, ad, Device::Parse(dev), seed);
           }),
           py::arg("capacity"), py::arg("obs_dim"), py::arg("act_dim"), py::arg("device") = "cpu",
           py::arg("seed") = 0)
      .def("push",
           [](RingBuffer& b, const Tensor& o, const Tensor& a, const Tensor& r, bool d) { return b.Push(o, a, r, d); },
           py::arg("obs"), py::arg("act"), py::arg("reward"), py::arg("done"))
      .def("push_batch", &RingBuffer::PushBatch, py::arg("obs"), py::arg("act"), py::arg("reward"), py::arg("done"))
      .def("sample",
           [](RingBuffer& b, int bs, Tensor* o, Tensor* a, Tensor* r, Tensor* d) { return b.Sample(bs, o, a, r, d); },
           py::arg("batch_size"), py::arg("obs"), py::arg("act"), py::arg("reward"), py::arg("done"))
      .def("sample_batch",
           [](RingBuffer& b, int bs) {
             Tensor o, a, r, d;
             throw_if(b.Sample(bs, &o, &a, &r, &d));
             return py::make_tuple(o.torch(), a.torch(), r.torch(), d.torch());
           },
           py::arg("batch_size"), "Pythonic form: returns (obs, act, reward, done) torch tensors.")
      .def("sample_indices", &RingBuffer::SampleIndices)
      .def("gather",
           [](RingBuffer& b, const at::Tensor& idx) {
             Tensor o, a, r, d;
             throw_if(b.Gather(idx, &o, &a, &r, &d));
             return py::make_tuple(o.torch(), a.torch(), r.torch(), d.torch());
           })
      .def("size", &RingBuffer::Size)
      .def("capacity", &RingBuffer::Capacity)
      .def("head", &RingBuffer::Head)
      .def("clear", &RingBuffer::Clear)
      .def("storage", [](RingBuffer& b) {
        return py::make_tuple(b.Observations(), b.Actions(), b.Rewards(), b.Dones());
      });

  py::class_<PrioritizedReplayBuffer, RingBuffer>(m, "PrioritizedReplayBuffer")
      .def(py::init([](int64_t cap, int od, int ad, float alpha, float beta, float eps, const std::string& dev,
                       uint64_t seed) {
             return new PrioritizedReplayBuffer(cap, od, ad, alpha, beta, eps, Device::Parse(dev), seed);
           }),
           py::arg("capacity"), py::arg("obs_dim"), py::arg("act_dim"), py::arg("alpha") = 0.6f,
           py::arg("beta") = 0.4f, py::arg("eps") = 1e-6f, py::arg("device") = "cpu", py::arg("seed") = 0)
      .def("sample_prioritized",
           [](PrioritizedReplayBuffer& b, int bs, py::object beta) {
             Tensor o, a, r, d;
             at::Tensor idx, w;
             const float be = beta.is_none() ? b.beta() : beta.cast<float>();
             throw_if(b.SamplePrioritized(bs, be, &o, &a, &r, &d, &idx, &w));
             return py::make_tuple(o.torch(), a.torch(), r.torch(), d.torch(), idx, w);
           },
           py::arg("batch_size"), py::arg("beta") = py::none())
      .def("update_priorities",
           [](PrioritizedReplayBuffer& b, const at::Tensor& i, const at::Tensor& p) {
             throw_if(b.UpdatePriorities(i, p));
           })
      .def("total_priority", &PrioritizedReplayBuffer::TotalPriority)
      .def("tree", [](PrioritizedReplayBuffer& b) { return b.Tree(); })
      .def("leaves", &PrioritizedReplayBuffer::Leaves)
      .def("alpha", &PrioritizedReplayBuffer::alpha)
      .def("beta", &PrioritizedReplayBuffer::beta);

  // ---------------- config ----------------
  py::class_<Config>(m, "Config")
      .def(py::init<>())
      .def("load", &Config::Load)
      .def("save", &Config::Save)
      .def("get_float", [](const Config& c, const std::string& k, double d) { return c.GetFloat(k, d); },
           py::arg("key"), py::arg("default"))
      .def("get_int", [](const Config& c, const std::string& k, long long d) { return c.GetInt(k, d); },
           py::arg("key"), py::arg("default"))
      .def("get_bool", [](const Config& c, const std::string& k, bool d) { return c.GetBool(k, d); },
           py::arg("key"), py::arg("default"))
      .def("get_str", [](const Config& c, const std::string& k, const std::string& d) { return c.GetString(k, d); },
           py::arg("key"), py::arg("default"))
      // bool must be tried before int (Python bool is an int subclass)
      .def("set", [](Config& c, const std::string& k, bool v) { c.SetBool(k, v); }, py::arg("key"), py::arg("value"))
      .def("set", [](Config& c, const std::string& k, long long v) { c.SetInt(k, v); }, py::arg("key"),
           py::arg("value"))
      .def("set", [](Config& c, const std::string& k, double v) { c.SetFloat(k, v); }, py::arg("key"),
           py::arg("value"))
      .def("set", [](Config& c, const std::string& k, const std::string& v) { c.SetString(k, v); }, py::arg("key"),
           py::arg("value"))
      .def("has", &Config::Has)
      .def("erase", &Config::Erase)
      .def("keys", &Config::Keys)
      .def("__len__", &Config::size);

  // ---------------- rewards ----------------
  py::class_<RewardConfig>(m, "RewardConfig")
      .def(py::init<>())
      .def_readwrite("kl_coef", &RewardConfig::kl_coef)
      .def_readwrite("kl_target", &RewardConfig::kl_target)
      .def_readwrite("adaptive_kl", &RewardConfig::adaptive_kl)
      .def_readwrite("kl_adapt_rate", &RewardConfig::kl_adapt_rate)
      .def_readwrite("normalize", &RewardConfig::normalize)
      .def_readwrite("whiten", &RewardConfig::whiten)
      .def_readwrite("reward_clip", &RewardConfig::reward_clip)
      .def_readwrite("gamma", &RewardConfig::gamma)
      .def_readwrite("format_bonus", &RewardConfig::format_bonus)
      .def_readwrite("length_penalty", &RewardConfig::length_penalty)
      .def_readwrite("target_length", &RewardConfig::target_length)
      .def_readwrite("period_token_id", &RewardConfig::period_token_id)
      .def_readwrite("k3_kl", &RewardConfig::k3_kl)
      .def_property("per_token", [](const RewardConfig& c) { return c.mode == RewardMode::kPerToken; },
                    [](RewardConfig& c, bool v) { c.mode = v ? RewardMode::kPerToken : RewardMode::kScalar; })
      .def_property("device", [](const RewardConfig& c) { return c.device.ToString(); },
                    [](RewardConfig& c, py::object d) { c.device = Device::Parse(py::str(d)); });

  py::class_<RewardResult>(m, "RewardResult")
      .def(py::init<>())
      .def_readwrite("total", &RewardResult::total)
      .def_readwrite("model_scores", &RewardResult::model_scores)
      .def_readwrite("kl_penalties", &RewardResult::kl_penalties)
      .def_readwrite("rule_scores", &RewardResult::rule_scores);

  py::class_<RewardEngine>(m, "RewardEngine")
      .def(py::init<const RewardConfig&>(), py::arg("config"))
      .def("initialize", &RewardEngine::Initialize)
      .def("score_batch",
           [](RewardEngine& e, const std::vector<std::string>& resp, bool has_ref, Tensor ref) {
             RewardResult r;
             std::optional<Tensor> rr = has_ref ? std::optional<Tensor>(std::move(ref)) : std::nullopt;
             throw_if(e.ScoreBatch(resp, rr, &r));
             return r;
           },
           py::arg("responses"), py::arg("has_ref") = false, py::arg("ref_logprobs") = Tensor())
      .def("score_tokens",
           [](RewardEngine& e, const Tensor& ids, const Tensor& masks, py::object ref, py::object lp) {
             RewardResult r;
             std::optional<Tensor> refo, lpo;
             if (!ref.is_none()) refo = py::isinstance<Tensor>(ref) ? ref.cast<Tensor>() : Tensor(ref.cast<at::Tensor>());
             if (!lp.is_none()) lpo = py::isinstance<Tensor>(lp) ? lp.cast<Tensor>() : Tensor(lp.cast<at::Tensor>());
             throw_if(e.ScoreTokens(ids, masks, lpo, refo, &r));
             return r;
           },
           py::arg("token_ids"), py::arg("masks"), py::arg("ref_logprobs") = py::none(),
           py::arg("logprobs") = py::none())
      .def("hash_reward",
           [](RewardEngine& e, const at::Tensor& ids, py::object lens) {
             at::Tensor out;
             throw_if(e.HashReward(ids, lens.is_none() ? at::Tensor() : lens.cast<at::Tensor>(), &out));
             return out;
           },
           py::arg("token_ids"), py::arg("lengths") = py::none())
      .def("kl_penalty",
           [](RewardEngine& e, const at::Tensor& lp, const at::Tensor& ref, py::object mask) {
             at::Tensor out;
             throw_if(e.ComputeKLPenalty(lp, ref, mask.is_none() ? at::Tensor() : mask.cast<at::Tensor>(), &out));
             return out;
           },
           py::arg("logprobs"), py::arg("ref_logprobs"), py::arg("masks") = py::none())
      .def("update_adaptive_kl", &RewardEngine::UpdateAdaptiveKL)
      .def("update_stats", &RewardEngine::UpdateStats)
      .def("current_kl_coef", &RewardEngine::CurrentKLCoef)
      .def("running_mean", &RewardEngine::RunningMean)
      .def("running_var", &RewardEngine::RunningVar)
      .def("running_count", &RewardEngine::RunningCount);

  // ---------------- observability ----------------
  py::class_<SpanID>(m, "SpanID").def(py::init<>()).def_readwrite("id", &SpanID::id);
  py::class_<EventID>(m, "EventID").def(py::init<>()).def_readwrite("id", &EventID::id);

  py::class_<ProfilerConfig>(m, "ProfilerConfig")
      .def(py::init<>())
      .def_readwrite("enable_nvtx", &ProfilerConfig::enable_nvtx)
      .def_readwrite("enable_cuda_timing", &ProfilerConfig::enable_cuda_timing)
      .def_readwrite("enable_memory", &ProfilerConfig::enable_memory)
      .def_readwrite("enable_cpu", &ProfilerConfig::enable_cpu)
      .def_readwrite("cuda_device_id", &ProfilerConfig::cuda_device_id)
      .def_readwrite("rank", &ProfilerConfig::rank)
      .def_readwrite("export_dir", &ProfilerConfig::export_dir);

  py::class_<Span>(m, "Span")
      .def_readonly("id", &Span::id)
      .def_readonly("parent", &Span::parent)
      .def_readonly("name", &Span::name)
      .def_readonly("category", &Span::category)
      .def_readonly("device_id", &Span::device_id)
      .def_readonly("start_ns", &Span::start_ns)
      .def_readonly("end_ns", &Span::end_ns)
      .def("duration_ns", &Span::duration_ns);

  py::class_<AggregatedStats>(m, "AggregatedStats")
      .def_readonly("name", &AggregatedStats::name)
      .def_readonly("count", &AggregatedStats::count)
      .def_readonly("total_ns", &AggregatedStats::total_ns)
      .def_readonly("min_ns", &AggregatedStats::min_ns)
      .def_readonly("max_ns", &AggregatedStats::max_ns)
      .def("avg_ns", &AggregatedStats::avg_ns);

  py::class_<CommRecord>(m, "CommRecord")
      .def_readonly("name", &CommRecord::name)
      .def_readonly("bytes", &CommRecord::bytes)
      .def_readonly("ms", &CommRecord::ms)
      .def("gbps", &CommRecord::gbps);

  py::class_<Profiler::Guard>(m, "ProfilerGuard")
      .def(py::init<Profiler*, const std::string&, const std::string&, int>(), py::arg("profiler"), py::arg("name"),
           py::arg("category") = "compute", py::arg("device_id") = -1, py::keep_alive<1, 2>())
      .def("__enter__", [](Profiler::Guard& g) -> Profiler::Guard& { return g; }, py::return_value_policy::reference)
      .def("__exit__", [](Profiler::Guard& g, py::object, py::object, py::object) {
        g.End();
        return false;
      });

  py::class_<Profiler>(m, "Profiler")
      .def(py::init<const ProfilerConfig&>(), py::arg("config") = ProfilerConfig{})
      .def("enable", &Profiler::Enable)
      .def("disable", &Profiler::Disable)
      .def("is_enabled", &Profiler::IsEnabled)
      .def("begin_span", &Profiler::BeginSpan, py::arg("name"), py::arg("category") = "compute",
           py::arg("device_id") = -1)
      .def("end_span", &Profiler::EndSpan)
      .def("span",
           [](Profiler* p, const std::string& n, const std::string& c, int d) {
             return std::make_unique<Profiler::Guard>(p, n, c, d);
           },
           py::arg("name"), py::arg("category") = "compute", py::arg("device_id") = -1, py::keep_alive<0, 1>())
      .def("begin_event", &Profiler::BeginEvent, py::arg("name"), py::arg("device_id") = 0)
      .def("end_event", &Profiler::EndEvent)
      .def("mark", &Profiler::Mark)
      .def("record_comm", &Profiler::RecordComm, py::arg("name"), py::arg("bytes"), py::arg("ms"))
      .def("export_chrome_trace", &Profiler::ExportChromeTrace, py::arg("path"))
      .def("export_json", &Profiler::ExportJSON, py::arg("path"))
      .def("summary", &Profiler::Summary)
      .def("print_summary", [](const Profiler& p) { py::print(p.Summary()); })
      .def("get_all_spans", &Profiler::GetAllSpans)
      .def("get_stats", &Profiler::GetStats)
      .def("get_comm_records", &Profiler::GetCommRecords)
      .def("clear", &Profiler::Clear);

  py::class_<TensorBoardWriter>(m, "TensorBoardWriter")
      .def(py::init<const std::string&>(), py::arg("log_dir"))
      .def("add_scalar", &TensorBoardWriter::AddScalar, py::arg("tag"), py::arg("value"), py::arg("step"))
      .def("add_histogram",
           [](TensorBoardWriter& w, const std::string& tag, py::array_t<float, py::array::c_style | py::array::forcecast> v,
              int64_t step) { w.AddHistogram(tag, v.data(), static_cast<int64_t>(v.size()), step); },
           py::arg("tag"), py::arg("values"), py::arg("step"))
      .def("add_text", &TensorBoardWriter::AddText, py::arg("tag"), py::arg("text"), py::arg("step"))
      .def("flush", &TensorBoardWriter::Flush)
      .def("path", &TensorBoardWriter::path);

  m.def("crc32c", [](py::bytes b) {
    std::string s = b;
    return Crc32c(s.data(), s.size());
  });
  m.def("masked_crc32c", [](py::bytes b) {
    std::string s = b;
    return MaskedCrc32c(s.data(), s.size());
  });

  py::class_<Labels>(m, "Labels")
      .def(py::init<>())
      .def(py::init([](const std::map<std::string, std::string>& d) {
        Labels l;
        l.kv = d;
        return l;
      }))
      .def("__setitem__", [](Labels& l, const std::string& k, const std::string& v) { l.kv[k] = v; })
      .def("__getitem__", [](const Labels& l, const std::string& k) { return l.kv.at(k); });

  py::class_<PrometheusWriter>(m, "PrometheusWriter")
      .def(py::init<const std::string&>(), py::arg("path"))
      .def("write", &PrometheusWriter::Write, py::arg("name"), py::arg("value"), py::arg("labels") = Labels{})
      .def("write_counter", &PrometheusWriter::WriteCounter, py::arg("name"), py::arg("value"),
           py::arg("labels") = Labels{})
      .def("write_gauge", &PrometheusWriter::WriteGauge, py::arg("name"), py::arg("value"),
           py::arg("labels") = Labels{})
      .def("observe_histogram", &PrometheusWriter::ObserveHistogram, py::arg("name"), py::arg("value"),
           py::arg("buckets"), py::arg("labels") = Labels{})
      .def("flush", &PrometheusWriter::Flush)
      .def("render", &PrometheusWriter::Render);

  py::enum_<LogLevel>(m, "LogLevel")
      .value("DEBUG", LogLevel::kDebug)
      .value("INFO", LogLevel::kInfo)
      .value("WARNING", LogLevel::kWarning)
      .value("ERROR", LogLevel::kError)
      .value("OFF", LogLevel::kOff);
  m.def("set_log_level", &SetLogLevel);
  m.def("get_log_level", &GetLogLevel);
  m.def("log", &Log);

  // ---------------- runtime ----------------
  py::class_<CoreEngine, std::unique_ptr<CoreEngine, py::nodelete>>(m, "CoreEngine")
      .def_static("instance", &CoreEngine::Instance, py::return_value_policy::reference)
      .def("initialize", &CoreEngine::Initialize, py::arg("device_id") = 0, py::arg("streams_per_device") = 4)
      .def("shutdown", &CoreEngine::Shutdown)
      .def("synchronize", &CoreEngine::Synchronize)
      .def("is_initialized", &CoreEngine::IsInitialized)
      .def("register_module", &CoreEngine::RegisterModule)
      .def("has_module", &CoreEngine::HasModule)
      .def("list_modules", &CoreEngine::ListModules)
      .def("stream_handle", [](CoreEngine& e, int dev, int i) { return reinterpret_cast<uintptr_t>(e.GetStream(dev, i)); });

  py::class_<TensorUtils>(m, "TensorUtils")
      .def_static("fill", [](Tensor& t, float v) { return TensorUtils::Fill(&t, v); })
      .def_static("add_scalar", [](Tensor& t, float v) { return TensorUtils::AddScalar(&t, v); })
      .def_static("scale", [](Tensor& t, float v) { return TensorUtils::Scale(&t, v); })
      .def_static("add", [](const Tensor& a, const Tensor& b, Tensor& o) { return TensorUtils::Add(a, b, &o); })
      .def_static("sub", [](const Tensor& a, const Tensor& b, Tensor& o) { return TensorUtils::Sub(a, b, &o); })
      .def_static("copy", [](const Tensor& s, Tensor& d) { return TensorUtils::Copy(s, &d); })
      .def_static("same_layout", &TensorUtils::SameLayout);

  py::class_<ByteTokenizer>(m, "ByteTokenizer")
      .def(py::init<>())
      .def("encode", &ByteTokenizer::Encode, py::arg("text"), py::arg("add_bos") = false, py::arg("add_eos") = false)
      .def("decode", &ByteTokenizer::Decode, py::arg("ids"), py::arg("skip_special") = true)
      .def("vocab_size", &ByteTokenizer::vocab_size)
      .def_readonly_static("pad_id", &ByteTokenizer::kPad)
      .def_readonly_static("bos_id", &ByteTokenizer::kBos)
      .def_readonly_static("eos_id", &ByteTokenizer::kEos);

  py::class_<DatasetConfig>(m, "DatasetConfig")
      .def(py::init<>())
      .def_readwrite("data_paths", &DatasetConfig::data_paths)
      .def_readwrite("format", &DatasetConfig::format)
      .def_readwrite("tokenizer_path", &DatasetConfig::tokenizer_path)
      .def_readwrite("max_seq_length", &DatasetConfig::max_seq_length)
      .def_readwrite("truncate", &DatasetConfig::truncate)
      .def_readwrite("batch_size", &DatasetConfig::batch_size)
      .def_readwrite("num_workers", &DatasetConfig::num_workers)
      .def_readwrite("prefetch_batches", &DatasetConfig::prefetch_batches)
      .def_readwrite("shuffle", &DatasetConfig::shuffle)
      .def_readwrite("shuffle_buffer_size", &DatasetConfig::shuffle_buffer_size)
      .def_readwrite("train_split", &DatasetConfig::train_split)
      .def_readwrite("seed", &DatasetConfig::seed)
      .def_property("prefetch_device", [](const DatasetConfig& c) { return c.prefetch_device.ToString(); },
                    [](DatasetConfig& c, const std::string& d) { c.prefetch_device = Device::Parse(d); });

  py::class_<DataSample>(m, "DataSample")
      .def(py::init<>())
      .def_readwrite("prompt", &DataSample::prompt)
      .def_readwrite("chosen", &DataSample::chosen)
      .def_readwrite("rejected", &DataSample::rejected)
      .def_readwrite("source", &DataSample::source)
      .def_readwrite("reward", &DataSample::reward)
      .def_readwrite("index", &DataSample::index);

  py::class_<PreprocessedBatch>(m, "PreprocessedBatch")
      .def(py::init<>())
      .def_readwrite("input_ids", &PreprocessedBatch::input_ids)
      .def_readwrite("attention_mask", &PreprocessedBatch::attention_mask)
      .def_readwrite("labels", &PreprocessedBatch::labels)
      .def_readwrite("prompt_lens", &PreprocessedBatch::prompt_lens)
      .def_readwrite("sample_indices", &PreprocessedBatch::sample_indices);

  py::class_<Dataset>(m, "Dataset")
      .def(py::init<const DatasetConfig&>(), py::arg("config"))
      .def("initialize", &Dataset::Initialize)
      .def("shutdown", &Dataset::Shutdown)
      .def("has_next", &Dataset::HasNext)
      .def("next_batch",
           [](Dataset& d) {
             PreprocessedBatch b;
             throw_if(d.NextBatch(&b));
             return b;
           })
      .def("get_sample",
           [](const Dataset& d, size_t i) {
             DataSample s;
             throw_if(d.GetSample(i, &s));
             return s;
           })
      .def("reset", &Dataset::Reset)
      .def("seek", &Dataset::Seek)
      .def("size", &Dataset::Size)
      .def("__len__", &Dataset::Size)
      .def_static("parse_line", [](const std::string& line) {
        DataSample s;
        throw_if(Dataset::ParseLine(line, &s));
        return s;
      });

  py::class_<TcpStore>(m, "TcpStore")
      .def(py::init<const std::string&, int, bool, int>(), py::arg("host"), py::arg("port"), py::arg("is_server"),
           py::arg("timeout_ms") = 30000, py::call_guard<py::gil_scoped_release>())
      .def("set", [](TcpStore& s, const std::string& k, py::bytes v) { throw_if(s.Set(k, v)); })
      .def("get",
           [](TcpStore& s, const std::string& k, int t) {
             std::string v;
             Status st;
             {
               py::gil_scoped_release rel;
               st = s.Get(k, &v, t);
             }
             throw_if(st);
             return py::bytes(v);
           },
           py::arg("key"), py::arg("timeout_ms") = -1)
      .def("add",
           [](TcpStore& s, const std::string& k, int64_t d) {
             int64_t r = 0;
             throw_if(s.Add(k, d, &r));
             return r;
           })
      .def("wait",
           [](TcpStore& s, const std::vector<std::string>& keys, int t) {
             Status st;
             {
               py::gil_scoped_release rel;
               st = s.Wait(keys, t);
             }
             throw_if(st);
           },
           py::arg("keys"), py::arg("timeout_ms") = -1)
      .def("barrier",
           [](TcpStore& s, const std::string& n, int world, int t) {
             Status st;
             {
               py::gil_scoped_release rel;
               st = s.Barrier(n, world, t);
             }
             throw_if(st);
           },
           py::arg("name"), py::arg("world"), py::arg("timeout_ms") = -1)
      .def("port", &TcpStore::port);

  py::class_<PipelineSchedule>(m, "PipelineSchedule")
      .def_static("one_f_one_b",
                  [](int P, int s, int M) {
                    std::vector<std::pair<std::string, int>> v;
                    for (auto& o : PipelineSchedule::OneFOneB(P, s, M)) v.emplace_back(std::string(1, o.kind), o.micro_batch);
                    return v;
                  })
      .def_static("gpipe",
                  [](int P, int s, int M) {
                    std::vector<std::pair<std::string, int>> v;
                    for (auto& o : PipelineSchedule::GPipe(P, s, M)) v.emplace_back(std::string(1, o.kind), o.micro_batch);
                    return v;
                  })
      .def_static("peak_activations", [](const std::vector<std::pair<std::string, int>>& v) {
        std::vector<PipeOp> ops;
        for (auto& p : v) ops.push_back(PipeOp{p.first[0], p.second});
        return PipelineSchedule::PeakActivations(ops);
      });

  py::class_<KVBlockManager>(m, "KVBlockManager")
      .def(py::init<int, int>(), py::arg("num_blocks"), py::arg("block_size") = 16)
      .def("allocate", &KVBlockManager::Allocate)
      .def("append_token", &KVBlockManager::AppendToken)
      .def("free", &KVBlockManager::Free)
      .def("can_allocate", &KVBlockManager::CanAllocate)
      .def("block_table", &KVBlockManager::BlockTable)
      .def("seq_len", &KVBlockManager::SeqLen)
      .def("num_free", &KVBlockManager::NumFree)
      .def("num_blocks", &KVBlockManager::NumBlocks)
      .def("block_size", &KVBlockManager::BlockSize)
      .def("reset", &KVBlockManager::Reset);

  // ---------------- helpers ----------------
  // host versions of the fused policy passes and of Adam (CPU tensors)
  auto host_f32 = [](const at::Tensor& t, const char* what) {
    if (t.is_cuda() || t.scalar_type() != at::kFloat || !t.is_contiguous())
      throw std::invalid_argument(std::string(what) + ": a contiguous fp32 CPU tensor is required");
  };
  m.def("lin_gauss_act_host",
        [host_f32](const at::Tensor& x, const at::Tensor& p, at::Tensor act, at::Tensor logp, int O, int A, float stdv,
                   uint64_t seed, uint32_t counter) {
          host_f32(x, "x");
          host_f32(p, "params");
          host_f32(act, "act");
          host_f32(logp, "logp");
          const int64_t N = x.numel() / O;
          if (x.numel() != N * O || act.numel() < N * A || logp.numel() < N || p.numel() < A * O + A)
            throw std::invalid_argument("lin_gauss_act_host: shapes");
          throw_if(LinGaussActHost(x.data_ptr<float>(), p.data_ptr<float>(), act.data_ptr<float>(),
                                   logp.data_ptr<float>(), static_cast<int>(N), O, A, stdv, seed, counter));
        },
        py::arg("x"), py::arg("params"), py::arg("act"), py::arg("logp"), py::arg("O"), py::arg("A"), py::arg("std"),
        py::arg("seed"), py::arg("counter"));
  m.def("lin_gauss_grad_host",
        [host_f32](const at::Tensor& batch, const at::Tensor& p, at::Tensor g, int O, int A, float stdv, float clip,
                   float vf_coef, bool has_old) {
          host_f32(batch, "batch");
          host_f32(p, "params");
          host_f32(g, "grad");
          if (batch.dim() != 2 || p.numel() < A * O + A + O + 1 || g.numel() < A * O + A + O + 1)
            throw std::invalid_argument("lin_gauss_grad_host: shapes");
          throw_if(LinGaussGradHost(batch.data_ptr<float>(), static_cast<int>(batch.size(1)), p.data_ptr<float>(),
                                    g.data_ptr<float>(), static_cast<int>(batch.size(0)), O, A, stdv, clip, vf_coef,
                                    has_old));
        },
        py::arg("batch"), py::arg("params"), py::arg("grad"), py::arg("O"), py::arg("A"), py::arg("std"),
        py::arg("clip"), py::arg("vf_coef"), py::arg("has_old"));
  m.def("adam_host",
        [host_f32](at::Tensor p, const at::Tensor& g, at::Tensor m1, at::Tensor m2, int64_t step, float lr, float b1,
                   float b2, float eps, float wd, float grad_scale) {
          host_f32(p, "param");
          host_f32(g, "grad");
          host_f32(m1, "m");
          host_f32(m2, "v");
          const int64_t n = p.numel();
          if (g.numel() != n || m1.numel() != n || m2.numel() != n) throw std::invalid_argument("adam_host: sizes");
          AdamHost(p.data_ptr<float>(), g.data_ptr<float>(), m1.data_ptr<float>(), m2.data_ptr<float>(), n, step, lr,
                   b1, b2, eps, wd, grad_scale);
        },
        py::arg("param"), py::arg("grad"), py::arg("m"), py::arg("v"), py::arg("step"), py::arg("lr"), py::arg("b1"),
        py::arg("b2"), py::arg("eps"), py::arg("wd"), py::arg("grad_scale"));

  m.def("gae_host",
        [host_f32](const at::Tensor& r, const at::Tensor& v, const at::Tensor& d, at::Tensor adv, at::Tensor ret,
                   py::object stats, float gamma, float lam) {
          host_f32(r, "rewards");
          host_f32(v, "values");
          host_f32(adv, "adv");
          host_f32(ret, "ret");
          if (r.dim() != 2 || v.dim() != 2 || v.size(0) != r.size(0) + 1 || v.size(1) != r.size(1) ||
              d.numel() != r.numel() || d.element_size() != 1 || !d.is_contiguous() || d.is_cuda() ||
              adv.numel() != r.numel() || ret.numel() != r.numel())
            throw std::invalid_argument("gae_host: rewards / dones [T, N], values [T + 1, N], byte dones");
          double* sp = nullptr;
          at::Tensor st;
          if (!stats.is_none()) {
            st = stats.cast<at::Tensor>();
            if (st.is_cuda() || st.scalar_type() != at::kDouble || st.numel() < 2 || !st.is_contiguous())
              throw std::invalid_argument("gae_host: stats must be float64 [2] on the CPU");
            sp = st.data_ptr<double>();
          }
          throw_if(GaeHost(r.data_ptr<float>(), v.data_ptr<float>(), static_cast<const uint8_t*>(d.data_ptr()),
                           adv.data_ptr<float>(), ret.data_ptr<float>(), static_cast<int>(r.size(0)),
                           static_cast<int>(r.size(1)), gamma, lam, sp));
        },
        py::arg("rewards"), py::arg("values"), py::arg("dones"), py::arg("adv"), py::arg("ret"),
        py::arg("stats") = py::none(), py::arg("gamma") = 0.99f, py::arg("lam") = 0.95f);

  m.def("ppo_minibatch_host",
        [](const at::Tensor& flat, const at::Tensor& grad, const std::vector<int64_t>& dims_a,
           const std::vector<int64_t>& dims_c, const at::Tensor& obs, const at::Tensor& act,
           const at::Tensor& old_logp, const at::Tensor& adv, const at::Tensor& ret, const at::Tensor& idx, float clip,
           float vf_coef, float ent_coef, const at::Tensor& stats) {
          if (flat.is_cuda() || obs.is_cuda()) throw std::invalid_argument("ppo_minibatch_host: CPU tensors");
          throw_if(PpoCategoricalMinibatchHost(flat, grad, dims_a, dims_c, obs, act, old_logp, adv, ret, idx, clip,
                                               vf_coef, ent_coef, stats));
        },
        py::arg("flat"), py::arg("grad"), py::arg("dims_actor"), py::arg("dims_critic"), py::arg("obs"),
        py::arg("act"), py::arg("old_logp"), py::arg("adv"), py::arg("ret"), py::arg("idx"), py::arg("clip"),
        py::arg("vf_coef"), py::arg("ent_coef"), py::arg("stats"));

  m.def("ppo_update_host",
        [](const at::Tensor& flat, const at::Tensor& grad, const at::Tensor& m1, const at::Tensor& m2, int64_t step,
           const std::vector<int64_t>& dims_a, const std::vector<int64_t>& dims_c, const at::Tensor& obs,
           const at::Tensor& act, const at::Tensor& old_logp, const at::Tensor& adv, const at::Tensor& ret,
           const at::Tensor& perms, int64_t minibatch, float clip, float vf_coef, float ent_coef, float lr, float b1,
           float b2, float eps, float wd, const at::Tensor& stats) {
          if (flat.is_cuda() || obs.is_cuda()) throw std::invalid_argument("ppo_update_host: CPU tensors");
          Status st;
          int64_t last;
          {
            py::gil_scoped_release release;
            last = PpoCategoricalUpdateHost(flat, grad, m1, m2, step, dims_a, dims_c, obs, act, old_logp, adv, ret,
                                            perms, minibatch, clip, vf_coef, ent_coef, lr, b1, b2, eps, wd, stats,
                                            &st);
          }
          throw_if(st);
          return last;
        },
        py::arg("flat"), py::arg("grad"), py::arg("m"), py::arg("v"), py::arg("step"), py::arg("dims_actor"),
        py::arg("dims_critic"), py::arg("obs"), py::arg("act"), py::arg("old_logp"), py::arg("adv"), py::arg("ret"),
        py::arg("perms"), py::arg("minibatch"), py::arg("clip"), py::arg("vf_coef"), py::arg("ent_coef"),
        py::arg("lr"), py::arg("b1"), py::arg("b2"), py::arg("eps"), py::arg("wd"), py::arg("stats"));

  m.def("ppo_cartpole_rollout_host",
        [](GPUEnvironment& env, const at::Tensor& flat, const std::vector<int64_t>& dims_a,
           const std::vector<int64_t>& dims_c, const at::Tensor& obs_buf, const at::Tensor& act_buf,
           const at::Tensor& logp_buf, const at::Tensor& val_buf, const at::Tensor& rew_buf, const at::Tensor& done_buf,
           uint64_t seed, uint64_t counter) {
          Status st;
          {
            py::gil_scoped_release release;
            st = PpoCartPoleRolloutHost(&env, flat, dims_a, dims_c, obs_buf, act_buf, logp_buf, val_buf, rew_buf,
                                        done_buf, seed, counter);
          }
          throw_if(st);
        },
        "The CPU PPO rollout on CartPole (T = obs_buf.shape[0] steps) in one call: policy forward, sampling, "
        "environment step, buffers.",
        py::arg("env"), py::arg("flat"), py::arg("dims_actor"), py::arg("dims_critic"), py::arg("obs_buf"),
        py::arg("act_buf"), py::arg("logp_buf"), py::arg("val_buf"), py::arg("rew_buf"), py::arg("done_buf"),
        py::arg("seed"), py::arg("counter"));

  m.def("get_version", []() { return std::string("1.0.0"); });
  m.def("get_device_count", &GetCudaDeviceCount);
  m.def("get_memory_info",
        [](int id) {
          auto i = GetCudaMemoryInfo(id);
          py::dict d;
          d["total"] = static_cast<long long>(i.total);
          d["free"] = static_cast<long long>(i.free);
          d["used"] = static_cast<long long>(i.used());
          d["utilization"] = i.utilization();
          return d;
        },
        py::arg("device_id") = 0);
#if TURBOL_CUDA
  m.def("built_for", []() { return std::string("sm_100a"); });
#else
  m.def("built_for", []() { return std::string("cpu"); });
#endif

#if TURBOL_CUDA
  py::module_ ops = m.def_submodule("ops", "raw sm_100a kernel launchers on torch tensors");
  register_kernel_ops(ops);
  register_llm_ops(ops);
  register_comm_ops(ops);
  py::module_ dist = m.def_submodule("dist", "C++ distributed runtime: NcclCommunicator, DistributedTrainer, "
                                               "PipelineTrainer (turbol/distributed.hpp)");
  register_dist(dist);
#endif
}
