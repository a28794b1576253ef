// Distributed runtime of the C++ API: NCCL communicators, the data-parallel
// facade and a 1F1B pipeline driver (one process per GPU).
//
// Parity with the reference's C++ headers:
//   DistributedConfig / DistributedTrainer  turbol_vllm/include/turbol/distributed/distributed_trainer.hpp:9-34
//   NcclCommunicator                        turbol_vllm/include/turbol/distributed/nccl_communicator.hpp:11-41
//   PipelineConfig / PipelineTrainer        turbol_vllm/include/turbol/distributed/pipeline_trainer.hpp:32-112
// Same class and method names; the behaviour is the working version of what
// those headers describe:
//   * bootstrap over the native TcpStore at master_addr:master_port (the
//     reference writes the NCCL id to a fixed /tmp file and ignores the port),
//     with a deadline: init is non-blocking NCCL (ncclCommInitRankConfig,
//     blocking = 0) polled until ready, aborted with kTimeout when late;
//   * each rank drives its own GPU (device_id, default rank % visible devices;
//     the reference uses device 0 on every rank);
//   * "mean" is NCCL's device-side average (the reference scales a device
//     pointer on the host), any dtype of the Tensor, the caller's stream;
//   * Barrier is a one-element all-reduce (the reference calls a function
//     NCCL does not have);
//   * PipelineTrainer runs the 1F1B schedule of PipelineSchedule over NCCL
//     send/recv with caller-supplied stage functions, optionally recomputing
//     activations (the reference's TrainingStep is a serial stub).
// Built only in the CUDA build (the CPU-only build has no NCCL).
#pragma once

#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "turbol/common.hpp"
#include "turbol/runtime.hpp"

namespace turbol {
namespace distributed {

enum class ParallelStrategy { kDataParallel, kModelParallel, kPipelineParallel };

struct DistributedConfig {
  ParallelStrategy strategy = ParallelStrategy::kDataParallel;
  int world_size = 1;
  int rank = 0;
  std::string master_addr = "127.0.0.1";
  int master_port = 29500;
  bool use_nccl = true;
  int device_id = -1;        // -1: rank % visible devices
  double timeout_s = 120.0;  // bootstrap and NCCL init deadline
};

class NcclCommunicator {
 public:
  // The process-wide world communicator (the reference's singleton).
  static NcclCommunicator& Instance();
  NcclCommunicator();
  ~NcclCommunicator();
  NcclCommunicator(const NcclCommunicator&) = delete;
  NcclCommunicator& operator=(const NcclCommunicator&) = delete;

  // Rank 0 creates the unique id and publishes it under `key` in the store at
  // master_addr:master_port (rank 0 hosts the store); all ranks then join.
  Status Initialize(int rank, int world_size, int device_id = 0, const std::string& master_addr = "127.0.0.1",
                    int master_port = 29500, double timeout_s = 120.0, const std::string& key = "turbol/nccl_id");
  Status Shutdown();
  Status Abort();

  // Raw buffers (float32 unless a dtype is given), on `stream` (null: the
  // current torch stream of the device).
  Status AllReduce(const void* send, void* recv, size_t count, bool is_mean = false,
                   DataType dtype = DataType::kFloat32, cudaStream_t stream = nullptr);
  Status AllGather(const void* send, void* recv, size_t count, DataType dtype = DataType::kFloat32,
                   cudaStream_t stream = nullptr);
  Status ReduceScatter(const void* send, void* recv, size_t count, bool is_mean = false,
                       DataType dtype = DataType::kFloat32, cudaStream_t stream = nullptr);
  Status Broadcast(const void* send, void* recv, size_t count, int root = 0, DataType dtype = DataType::kFloat32,
                   cudaStream_t stream = nullptr);
  Status Send(const void* data, size_t count, int peer, DataType dtype = DataType::kFloat32,
              cudaStream_t stream = nullptr);
  Status Recv(void* data, size_t count, int peer, DataType dtype = DataType::kFloat32, cudaStream_t stream = nullptr);
  Status Barrier();
  // Brackets sends / receives that must be posted together (NCCL group).
  Status GroupStart();
  Status GroupEnd();

  // Tensor forms (CUDA tensors of this communicator's device).
  Status AllReduce(Tensor* t, const std::string& op = "sum");
  Status Broadcast(Tensor* t, int root = 0);
  Status AllGather(const Tensor& in, Tensor* out);

  int rank() const { return rank_; }
  int world_size() const { return world_size_; }
  int device() const { return device_; }
  bool is_initialized() const { return initialized_; }

 private:
  Status Check(int nccl_result, const char* what);
  cudaStream_t StreamOr(cudaStream_t s) const;
  int rank_ = 0, world_size_ = 0, device_ = 0;
  bool initialized_ = false;
  void* comm_ = nullptr;  // ncclComm_t
  std::unique_ptr<TcpStore> store_;
};

class DistributedTrainer {
 public:
  explicit DistributedTrainer(const DistributedConfig& config = DistributedConfig());
  ~DistributedTrainer();

  Status Initialize();
  Status Shutdown();
  Status AllReduce(Tensor* tensor, const std::string& op = "sum");
  Status Broadcast(Tensor* tensor, int root_rank = 0);
  Status Barrier();

  int GetRank() const { return config_.rank; }
  int GetWorldSize() const { return config_.world_size; }
  NcclCommunicator* communicator() { return comm_.get(); }

 private:
  DistributedConfig config_;
  bool initialized_ = false;
  std::unique_ptr<NcclCommunicator> comm_;
};

struct PipelineConfig {
  int num_pipeline_stages = 1;
  int num_microbatches = 8;
  int stage_id = 0;
  int num_warmup_microbatches = -1;  // -1: the 1F1B warm-up, num_stages - stage_id - 1
  int microbatch_seq_len = 512;
  int microbatch_batch_sz = 1;
  int hidden_size = 0;  // activation width exchanged between stages
  int max_cache_seq_len = 8192;
  bool activation_checkpointing = false;  // keep stage inputs only; recompute in backward
  int checkpoint_every_n_layers = 1;
  Device device = Device::CUDA(0);
};

// What a stage computes.  forward(mb, x_in) -> x_out; backward(mb, dx_out)
// -> dx_in (weight gradients accumulate inside the caller's model); on the
// first stage `input(mb)` gives x_in, on the last stage `loss(mb, x_out)`
// returns (loss value, dx_out).  Activations are bf16 or fp32 CUDA tensors of
// [microbatch_batch_sz * microbatch_seq_len, hidden_size].
struct StageFunctions {
  std::function<at::Tensor(int)> input;
  std::function<at::Tensor(int, const at::Tensor&)> forward;
  std::function<std::pair<float, at::Tensor>(int, const at::Tensor&)> loss;
  std::function<at::Tensor(int, const at::Tensor&)> backward;
  // optional: forward again before backward when activation_checkpointing is set
  std::function<void(int, const at::Tensor&)> recompute;
};

class PipelineTrainer {
 public:
  explicit PipelineTrainer(const PipelineConfig& config);
  ~PipelineTrainer();

  // comm: the pipeline's communicator (stage s = its rank s).
  Status Initialize(NcclCommunicator* comm, StageFunctions fns, at::ScalarType act_dtype = at::kBFloat16);
  Status Shutdown();
  // One step over all micro-batches in 1F1B order.  The mean loss over the
  // micro-batches lands in *out_avg_loss on the last stage (0 elsewhere).
  Status TrainingStep(float* out_avg_loss);
  // Forward only (evaluation): the last stage's outputs per micro-batch.
  Status Forward(std::vector<at::Tensor>* outputs);

  Status SendForward(const at::Tensor& t, int dst_stage);
  Status RecvForward(at::Tensor* t, int src_stage);
  Status SendBackward(const at::Tensor& t, int dst_stage);
  Status RecvBackward(at::Tensor* t, int src_stage);

  const PipelineConfig& config() const { return config_; }
  int CurrentStep() const { return current_step_; }
  // The op order of the last TrainingStep ("F0", "B0", ...).
  const std::vector<std::string>& LastOrder() const { return last_order_; }

 private:
  at::Tensor NewActivation() const;
  PipelineConfig config_;
  NcclCommunicator* comm_ = nullptr;
  StageFunctions fns_;
  at::ScalarType dtype_ = at::kBFloat16;
  bool initialized_ = false;
  int current_step_ = 0;
  std::vector<std::string> last_order_;
};

}  // namespace distributed
}  // namespace turbol
