// NCCL communicators, the data-parallel facade and the 1F1B pipeline driver
// of the C++ API (declarations and the parity notes in turbol/distributed.hpp).
#include "turbol/distributed.hpp"

#include <c10/cuda/CUDAGuard.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <thread>

namespace turbol {
namespace distributed {

namespace {

using Clock = std::chrono::steady_clock;

bool ToNccl(DataType t, ncclDataType_t* out) {
  switch (t) {
    case DataType::kFloat32: *out = ncclFloat32; return true;
    case DataType::kFloat16: *out = ncclFloat16; return true;
    case DataType::kBFloat16: *out = ncclBfloat16; return true;
    case DataType::kInt32: *out = ncclInt32; return true;
    case DataType::kInt64: *out = ncclInt64; return true;
    case DataType::kInt8: *out = ncclInt8; return true;
    case DataType::kUInt8: *out = ncclUint8; return true;
    case DataType::kBool: *out = ncclUint8; return true;
    default: return false;
  }
}

std::string Hex(const void* p, size_t n) {
  static const char* d = "0123456789abcdef";
  std::string s;
  const auto* b = static_cast<const unsigned char*>(p);
  for (size_t i = 0; i < n; ++i) {
    s.push_back(d[b[i] >> 4]);
    s.push_back(d[b[i] & 15]);
  }
  return s;
}

bool Unhex(const std::string& s, void* p, size_t n) {
  if (s.size() != 2 * n) return false;
  auto v = [](char c) { return c >= 'a' ? c - 'a' + 10 : c - '0'; };
  auto* b = static_cast<unsigned char*>(p);
  for (size_t i = 0; i < n; ++i) b[i] = static_cast<unsigned char>(v(s[2 * i]) << 4 | v(s[2 * i + 1]));
  return true;
}

// The communicator runs in NCCL's non-blocking mode: every call may return
// ncclInProgress, and completion is polled with a deadline, so a missing peer
// shows up as kTimeout (and an aborted communicator) instead of a hang.
Status Settle(ncclComm_t comm, ncclResult_t r, const char* what, double timeout_s) {
  const auto t0 = Clock::now();
  while (r == ncclInProgress) {
    if (std::chrono::duration<double>(Clock::now() - t0).count() > timeout_s) {
      ncclCommAbort(comm);
      return Status::Timeout(std::string(what) + ": NCCL did not complete in time (communicator aborted)");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
    ncclCommGetAsyncError(comm, &r);
  }
  if (r != ncclSuccess) return Status::InternalError(std::string(what) + ": " + ncclGetErrorString(r));
  return Status::Ok();
}

}  // namespace

// ============================================================ NcclCommunicator
NcclCommunicator& NcclCommunicator::Instance() {
  static NcclCommunicator inst;
  return inst;
}

NcclCommunicator::NcclCommunicator() = default;

NcclCommunicator::~NcclCommunicator() {
  if (initialized_) Shutdown();
}

Status NcclCommunicator::Check(int r, const char* what) {
  return Settle(static_cast<ncclComm_t>(comm_), static_cast<ncclResult_t>(r), what, 300.0);
}

cudaStream_t NcclCommunicator::StreamOr(cudaStream_t s) const { return s ? s : CurrentStream(device_); }

Status NcclCommunicator::Initialize(int rank, int world_size, int device_id, const std::string& master_addr,
                                    int master_port, double timeout_s, const std::string& key) {
  if (initialized_) return Status::AlreadyExists("NcclCommunicator already initialized");
  if (world_size < 1 || rank < 0 || rank >= world_size)
    return Status::InvalidArgument("NcclCommunicator: rank " + std::to_string(rank) + " of world " +
                                   std::to_string(world_size));
  if (device_id < 0 || device_id >= GetCudaDeviceCount())
    return Status::InvalidArgument("NcclCommunicator: no CUDA device " + std::to_string(device_id));
  rank_ = rank;
  world_size_ = world_size;
  device_ = device_id;
  c10::cuda::CUDAGuard guard(device_);
  ncclUniqueId id;
  const int ms = static_cast<int>(timeout_s * 1000);
  try {
    store_ = std::make_unique<TcpStore>(master_addr, master_port, rank == 0, ms);
  } catch (const std::exception& e) {
    return Status::Unavailable(std::string("NcclCommunicator bootstrap: ") + e.what());
  }
  if (rank == 0) {
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return Status::InternalError(std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
    TURBOL_RETURN_IF_ERROR(store_->Set(key, Hex(&id, sizeof(id))));
  } else {
    std::string v;
    TURBOL_RETURN_IF_ERROR(store_->Get(key, &v, ms));
    if (!Unhex(v, &id, sizeof(id))) return Status::InternalError("NcclCommunicator: malformed unique id");
  }
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclComm_t comm = nullptr;
  ncclResult_t r = ncclCommInitRankConfig(&comm, world_size, id, rank, &cfg);
  comm_ = comm;
  if (r != ncclSuccess && r != ncclInProgress)
    return Status::InternalError(std::string("ncclCommInitRankConfig: ") + ncclGetErrorString(r));
  Status st = Settle(comm, r, "ncclCommInitRankConfig", timeout_s);
  if (!st.ok()) {
    comm_ = nullptr;
    return st;
  }
  initialized_ = true;
  // every rank is in: rank 0 may drop its store once all have read the id
  return store_->Barrier(key + "/ready", world_size, ms);
}

Status NcclCommunicator::Shutdown() {
  if (!initialized_) return Status::Ok();
  c10::cuda::CUDAGuard guard(device_);
  ncclResult_t r = ncclCommFinalize(static_cast<ncclComm_t>(comm_));
  Status st = Settle(static_cast<ncclComm_t>(comm_), r, "ncclCommFinalize", 60.0);
  if (st.ok()) ncclCommDestroy(static_cast<ncclComm_t>(comm_));
  comm_ = nullptr;
  initialized_ = false;
  store_.reset();
  return st;
}

Status NcclCommunicator::Abort() {
  if (comm_) ncclCommAbort(static_cast<ncclComm_t>(comm_));
  comm_ = nullptr;
  initialized_ = false;
  store_.reset();
  return Status::Ok();
}

#define TURBOL_NCCL_READY()                                                               \
  if (!initialized_) return Status::InvalidArgument("NcclCommunicator not initialized"); \
  ncclDataType_t nt;                                                                      \
  if (!ToNccl(dtype, &nt)) return Status::InvalidArgument("NcclCommunicator: unsupported dtype");

Status NcclCommunicator::AllReduce(const void* send, void* recv, size_t count, bool is_mean, DataType dtype,
                                   cudaStream_t stream) {
  TURBOL_NCCL_READY();
  return Check(ncclAllReduce(send, recv, count, nt, is_mean ? ncclAvg : ncclSum, static_cast<ncclComm_t>(comm_),
                             StreamOr(stream)),
               "ncclAllReduce");
}

Status NcclCommunicator::AllGather(const void* send, void* recv, size_t count, DataType dtype, cudaStream_t stream) {
  TURBOL_NCCL_READY();
  return Check(ncclAllGather(send, recv, count, nt, static_cast<ncclComm_t>(comm_), StreamOr(stream)),
               "ncclAllGather");
}

Status NcclCommunicator::ReduceScatter(const void* send, void* recv, size_t count, bool is_mean, DataType dtype,
                                       cudaStream_t stream) {
  TURBOL_NCCL_READY();
  return Check(ncclReduceScatter(send, recv, count, nt, is_mean ? ncclAvg : ncclSum, static_cast<ncclComm_t>(comm_),
                                 StreamOr(stream)),
               "ncclReduceScatter");
}

Status NcclCommunicator::Broadcast(const void* send, void* recv, size_t count, int root, DataType dtype,
                                   cudaStream_t stream) {
  TURBOL_NCCL_READY();
  if (root < 0 || root >= world_size_) return Status::InvalidArgument("Broadcast: bad root");
  return Check(ncclBroadcast(send, recv, count, nt, root, static_cast<ncclComm_t>(comm_), StreamOr(stream)),
               "ncclBroadcast");
}

Status NcclCommunicator::Send(const void* data, size_t count, int peer, DataType dtype, cudaStream_t stream) {
  TURBOL_NCCL_READY();
  return Check(ncclSend(data, count, nt, peer, static_cast<ncclComm_t>(comm_), StreamOr(stream)), "ncclSend");
}

Status NcclCommunicator::Recv(void* data, size_t count, int peer, DataType dtype, cudaStream_t stream) {
  TURBOL_NCCL_READY();
  return Check(ncclRecv(data, count, nt, peer, static_cast<ncclComm_t>(comm_), StreamOr(stream)), "ncclRecv");
}
#undef TURBOL_NCCL_READY

Status NcclCommunicator::GroupStart() {
  if (!initialized_) return Status::InvalidArgument("NcclCommunicator not initialized");
  ncclResult_t r = ncclGroupStart();
  return r == ncclSuccess ? Status::Ok() : Status::InternalError(std::string("ncclGroupStart: ") + ncclGetErrorString(r));
}

Status NcclCommunicator::GroupEnd() {
  if (!initialized_) return Status::InvalidArgument("NcclCommunicator not initialized");
  return Check(ncclGroupEnd(), "ncclGroupEnd");
}

Status NcclCommunicator::Barrier() {
  if (!initialized_) return Status::InvalidArgument("NcclCommunicator not initialized");
  c10::cuda::CUDAGuard guard(device_);
  at::Tensor one = at::ones({1}, at::TensorOptions().dtype(at::kFloat).device(at::kCUDA, device_));
  TURBOL_RETURN_IF_ERROR(AllReduce(one.data_ptr(), one.data_ptr(), 1, false, DataType::kFloat32, nullptr));
  const float got = one.item<float>();  // synchronizes
  if (got != static_cast<float>(world_size_)) return Status::InternalError("Barrier: wrong participant count");
  return Status::Ok();
}

Status NcclCommunicator::AllReduce(Tensor* t, const std::string& op) {
  if (t == nullptr || !t->is_cuda()) return Status::InvalidArgument("AllReduce: a CUDA tensor is required");
  if (op != "sum" && op != "mean") return Status::InvalidArgument("AllReduce: op must be \"sum\" or \"mean\"");
  return AllReduce(t->data(), t->data(), static_cast<size_t>(t->numel()), op == "mean", t->dtype(), nullptr);
}

Status NcclCommunicator::Broadcast(Tensor* t, int root) {
  if (t == nullptr || !t->is_cuda()) return Status::InvalidArgument("Broadcast: a CUDA tensor is required");
  return Broadcast(t->data(), t->data(), static_cast<size_t>(t->numel()), root, t->dtype(), nullptr);
}

Status NcclCommunicator::AllGather(const Tensor& in, Tensor* out) {
  if (out == nullptr || !in.is_cuda() || !out->is_cuda() || out->numel() != in.numel() * world_size_ ||
      out->dtype() != in.dtype())
    return Status::InvalidArgument("AllGather: out must be a CUDA tensor of world_size x the input");
  return AllGather(in.data(), out->data(), static_cast<size_t>(in.numel()), in.dtype(), nullptr);
}

// ============================================================ DistributedTrainer
DistributedTrainer::DistributedTrainer(const DistributedConfig& config) : config_(config) {}

DistributedTrainer::~DistributedTrainer() {
  if (initialized_) Shutdown();
}

Status DistributedTrainer::Initialize() {
  if (initialized_) return Status::Ok();
  if (config_.world_size < 1 || config_.rank < 0 || config_.rank >= config_.world_size)
    return Status::InvalidArgument("DistributedTrainer: bad rank / world size");
  if (config_.world_size > 1) {
    if (!config_.use_nccl) return Status::Unimplemented("DistributedTrainer: world_size > 1 needs use_nccl");
    const int n = GetCudaDeviceCount();
    if (n < 1) return Status::Unavailable("DistributedTrainer: no CUDA device");
    const int dev = config_.device_id >= 0 ? config_.device_id : config_.rank % n;
    comm_ = std::make_unique<NcclCommunicator>();
    TURBOL_RETURN_IF_ERROR(comm_->Initialize(config_.rank, config_.world_size, dev, config_.master_addr,
                                             config_.master_port, config_.timeout_s));
  }
  initialized_ = true;
  return Status::Ok();
}

Status DistributedTrainer::Shutdown() {
  Status st = Status::Ok();
  if (comm_) st = comm_->Shutdown();
  comm_.reset();
  initialized_ = false;
  return st;
}

Status DistributedTrainer::AllReduce(Tensor* tensor, const std::string& op) {
  if (!initialized_) return Status::InvalidArgument("DistributedTrainer not initialized");
  if (op != "sum" && op != "mean") return Status::InvalidArgument("AllReduce: op must be \"sum\" or \"mean\"");
  if (config_.world_size == 1) return Status::Ok();  // a group of one: nothing to reduce
  return comm_->AllReduce(tensor, op);
}

Status DistributedTrainer::Broadcast(Tensor* tensor, int root_rank) {
  if (!initialized_) return Status::InvalidArgument("DistributedTrainer not initialized");
  if (root_rank < 0 || root_rank >= config_.world_size) return Status::InvalidArgument("Broadcast: bad root");
  if (config_.world_size == 1) return Status::Ok();
  return comm_->Broadcast(tensor, root_rank);
}

Status DistributedTrainer::Barrier() {
  if (!initialized_) return Status::InvalidArgument("DistributedTrainer not initialized");
  if (config_.world_size == 1) return Status::Ok();
  return comm_->Barrier();
}

// ============================================================ PipelineTrainer
PipelineTrainer::PipelineTrainer(const PipelineConfig& config) : config_(config) {}
PipelineTrainer::~PipelineTrainer() = default;

Status PipelineTrainer::Initialize(NcclCommunicator* comm, StageFunctions fns, at::ScalarType act_dtype) {
  const int S = config_.num_pipeline_stages, s = config_.stage_id;
  if (S < 1 || s < 0 || s >= S || config_.num_microbatches < 1 || config_.hidden_size < 1)
    return Status::InvalidArgument("PipelineTrainer: stages, stage_id, micro-batches and hidden_size");
  if (S > 1 && (comm == nullptr || !comm->is_initialized() || comm->world_size() != S || comm->rank() != s))
    return Status::InvalidArgument("PipelineTrainer: the communicator must span the stages (rank == stage_id)");
  if (!fns.forward || !fns.backward || (s == 0 && !fns.input) || (s == S - 1 && !fns.loss))
    return Status::InvalidArgument("PipelineTrainer: stage functions missing");
  if (config_.activation_checkpointing && !fns.recompute)
    return Status::InvalidArgument("PipelineTrainer: activation_checkpointing needs a recompute function");
  comm_ = comm;
  fns_ = std::move(fns);
  dtype_ = act_dtype;
  initialized_ = true;
  return Status::Ok();
}

Status PipelineTrainer::Shutdown() {
  initialized_ = false;
  fns_ = StageFunctions();
  return Status::Ok();
}

at::Tensor PipelineTrainer::NewActivation() const {
  const int64_t rows = static_cast<int64_t>(config_.microbatch_batch_sz) * config_.microbatch_seq_len;
  return at::empty({rows, config_.hidden_size}, at::TensorOptions().dtype(dtype_).device(at::kCUDA, comm_->device()));
}

Status PipelineTrainer::SendForward(const at::Tensor& t, int dst_stage) {
  return comm_->Send(t.data_ptr(), static_cast<size_t>(t.numel()), dst_stage, FromTorch(t.scalar_type()));
}
Status PipelineTrainer::RecvForward(at::Tensor* t, int src_stage) {
  return comm_->Recv(t->data_ptr(), static_cast<size_t>(t->numel()), src_stage, FromTorch(t->scalar_type()));
}
Status PipelineTrainer::SendBackward(const at::Tensor& t, int dst_stage) { return SendForward(t, dst_stage); }
Status PipelineTrainer::RecvBackward(at::Tensor* t, int src_stage) { return RecvForward(t, src_stage); }

Status PipelineTrainer::TrainingStep(float* out_avg_loss) {
  if (!initialized_) return Status::InvalidArgument("PipelineTrainer not initialized");
  const int S = config_.num_pipeline_stages, s = config_.stage_id, M = config_.num_microbatches;
  const bool first = s == 0, last = s == S - 1;
  const int prev = s - 1, next = s + 1;
  last_order_.clear();
  std::vector<at::Tensor> x_in(M), dx_out(M);
  float loss_sum = 0.f;
  // A send to one neighbour and a receive from one (or both) are issued as
  // one NCCL group, so two stages that exchange in opposite directions at the
  // same time never wait on each other's stream.
  auto exchange = [&](const at::Tensor* send_next, const at::Tensor* send_prev, at::Tensor* recv_next,
                      at::Tensor* recv_prev) -> Status {
    if (!send_next && !send_prev && !recv_next && !recv_prev) return Status::Ok();
    TURBOL_RETURN_IF_ERROR(comm_->GroupStart());
    Status st = Status::Ok();
    if (send_next && st.ok()) st = SendForward(*send_next, next);
    if (send_prev && st.ok()) st = SendBackward(*send_prev, prev);
    if (recv_prev && st.ok()) st = RecvForward(recv_prev, prev);
    if (recv_next && st.ok()) st = RecvBackward(recv_next, next);
    Status end = comm_->GroupEnd();
    return st.ok() ? end : st;
  };
  auto fwd = [&](int i, const at::Tensor& xin) -> at::Tensor {
    last_order_.push_back("F" + std::to_string(i));
    x_in[i] = xin;
    at::Tensor out = fns_.forward(i, xin);
    if (last) {
      auto lg = fns_.loss(i, out);
      loss_sum += lg.first;
      dx_out[i] = lg.second;
    }
    return out;
  };
  auto bwd = [&](int i, const at::Tensor& dout) -> at::Tensor {
    last_order_.push_back("B" + std::to_string(i));
    if (config_.activation_checkpointing) fns_.recompute(i, x_in[i]);
    at::Tensor d = fns_.backward(i, dout);
    x_in[i] = at::Tensor();
    return d;
  };
  const int warm = std::min(config_.num_warmup_microbatches >= 0 ? config_.num_warmup_microbatches : S - s - 1, M);
  const int remaining = M - warm;
  int fi = 0, bi = 0;
  for (int k = 0; k < warm; ++k) {  // warm-up forwards
    at::Tensor xin = first ? fns_.input(fi) : NewActivation();
    if (!first) TURBOL_RETURN_IF_ERROR(exchange(nullptr, nullptr, nullptr, &xin));
    at::Tensor out = fwd(fi, xin);
    if (!last) TURBOL_RETURN_IF_ERROR(exchange(&out, nullptr, nullptr, nullptr));
    ++fi;
  }
  at::Tensor xin;
  if (remaining > 0) {
    xin = first ? fns_.input(fi) : NewActivation();
    if (!first) TURBOL_RETURN_IF_ERROR(exchange(nullptr, nullptr, nullptr, &xin));
  }
  for (int k = 0; k < remaining; ++k) {  // steady state: one forward, one backward
    at::Tensor out = fwd(fi, xin);
    ++fi;
    at::Tensor dout;
    if (last) {
      dout = dx_out[fi - 1];
    } else {
      dout = NewActivation();
      TURBOL_RETURN_IF_ERROR(exchange(&out, nullptr, &dout, nullptr));
    }
    at::Tensor din = bwd(bi, dout);
    ++bi;
    const bool last_iter = k == remaining - 1;
    if (last_iter) {
      if (!first) TURBOL_RETURN_IF_ERROR(exchange(nullptr, &din, nullptr, nullptr));
    } else if (first) {
      xin = fns_.input(fi);
    } else {
      xin = NewActivation();
      TURBOL_RETURN_IF_ERROR(exchange(nullptr, &din, nullptr, &xin));
    }
  }
  for (int k = 0; k < warm; ++k) {  // cool-down backwards
    at::Tensor dout = last ? dx_out[bi] : NewActivation();
    if (!last) TURBOL_RETURN_IF_ERROR(exchange(nullptr, nullptr, &dout, nullptr));
    at::Tensor din = bwd(bi, dout);
    if (!first) TURBOL_RETURN_IF_ERROR(exchange(nullptr, &din, nullptr, nullptr));
    ++bi;
  }
  ++current_step_;
  if (out_avg_loss) *out_avg_loss = last ? loss_sum / static_cast<float>(M) : 0.f;
  return Status::Ok();
}

Status PipelineTrainer::Forward(std::vector<at::Tensor>* outputs) {
  if (!initialized_) return Status::InvalidArgument("PipelineTrainer not initialized");
  const int S = config_.num_pipeline_stages, s = config_.stage_id, M = config_.num_microbatches;
  if (outputs) outputs->clear();
  for (int i = 0; i < M; ++i) {
    at::Tensor xin = s == 0 ? fns_.input(i) : NewActivation();
    if (s > 0) TURBOL_RETURN_IF_ERROR(RecvForward(&xin, s - 1));
    at::Tensor out = fns_.forward(i, xin);
    if (s < S - 1) {
      TURBOL_RETURN_IF_ERROR(SendForward(out, s + 1));
    } else if (outputs) {
      outputs->push_back(out);
    }
  }
  return Status::Ok();
}

}  // namespace distributed
}  // namespace turbol
