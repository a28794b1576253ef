// Runtime services of the host core:
//   CoreEngine      module registry + per-device stream pool (reference
//                   turbol_vllm/include/turbol/core/core_engine.hpp:6-21 is an
//                   empty singleton)
//   TensorUtils     f32 elementwise ops (reference utils/tensor_utils.hpp:11-30)
//   ByteTokenizer   UTF-8 byte-level tokenizer (ids 0..255 = bytes, then
//                   pad/bos/eos), the tokenizer the reference's Dataset stubs out
//   Dataset         JSONL prompt/chosen/rejected loader with byte offsets,
//                   seeded shuffling and real tokenization (reference
//                   dataset/dataset.hpp:29-125, whose Tokenize is a stub)
//   TcpStore        rendezvous key/value store over TCP with deadlines on every
//                   wait (replaces the reference's /tmp file bootstrap,
//                   src/distributed/nccl_communicator.cpp:14-67)
//   PipelineSchedule 1F1B / GPipe op order per stage (the reference's
//                   PipelineTrainer runs micro-batches serially through a stub)
//   KVBlockManager  paged-KV block allocator for the rollout engine
#pragma once

#include <atomic>
#include <condition_variable>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "turbol/common.hpp"

namespace turbol {

class CoreEngine {
 public:
  static CoreEngine& Instance();
  Status Initialize(int device_id = 0, int streams_per_device = 4);
  Status Shutdown();
  bool IsInitialized() const { return initialized_; }
  Status Synchronize();
  void RegisterModule(const std::string& name) {
    std::lock_guard<std::mutex> g(mu_);
    modules_[name] = true;
  }
  bool HasModule(const std::string& name) const {
    std::lock_guard<std::mutex> g(mu_);
    return modules_.count(name) != 0;
  }
  std::vector<std::string> ListModules() const;
  // Round-robin stream from the pool of `device_id` (high priority when asked).
  cudaStream_t GetStream(int device_id, int index);
  int device_id() const { return device_id_; }

 private:
  CoreEngine() = default;
  bool initialized_ = false;
  int device_id_ = 0;
  std::map<std::string, bool> modules_;
  std::map<int, std::vector<cudaStream_t>> streams_;
  mutable std::mutex mu_;
};

class TensorUtils {
 public:
  static Status Fill(Tensor* t, float v);
  static Status AddScalar(Tensor* t, float v);
  static Status Scale(Tensor* t, float v);
  static Status Add(const Tensor& a, const Tensor& b, Tensor* out);
  static Status Sub(const Tensor& a, const Tensor& b, Tensor* out);
  static Status Copy(const Tensor& src, Tensor* dst);
  static bool SameLayout(const Tensor& a, const Tensor& b);
};

class ByteTokenizer {
 public:
  static constexpr int kPad = 256, kBos = 257, kEos = 258, kVocab = 259;
  std::vector<int> Encode(const std::string& s, bool add_bos = false, bool add_eos = false) const;
  std::string Decode(const std::vector<int>& ids, bool skip_special = true) const;
  int vocab_size() const { return kVocab; }
};

struct DatasetConfig {
  std::vector<std::string> data_paths;
  std::string format = "jsonl";
  std::string tokenizer_path;
  int max_seq_length = 2048;
  bool truncate = true;
  int batch_size = 8;
  int num_workers = 4;
  int prefetch_batches = 2;
  bool shuffle = true;
  int shuffle_buffer_size = 10000;
  float train_split = 0.98f;
  uint64_t seed = 0;
  Device prefetch_device = Device::CPU();
};

struct DataSample {
  std::string prompt, chosen, rejected, source;
  float reward = 0.f;
  int64_t index = 0;
};

struct PreprocessedBatch {
  Tensor input_ids, attention_mask, labels, prompt_lens;
  std::vector<int64_t> sample_indices;
};

class Dataset {
 public:
  explicit Dataset(const DatasetConfig& cfg) : cfg_(cfg) {}
  Status Initialize();
  Status Shutdown();
  bool HasNext() const { return cursor_ < order_.size(); }
  Status NextBatch(PreprocessedBatch* batch);
  Status GetSample(size_t i, DataSample* out) const;
  void Reset();
  Status Seek(size_t index);
  size_t Size() const { return entries_.size(); }
  const DatasetConfig& config() const { return cfg_; }
  // Parses one JSONL line (exposed for tests).
  static Status ParseLine(const std::string& line, DataSample* out);

 private:
  struct Entry {
    size_t file, offset;
  };
  DatasetConfig cfg_;
  ByteTokenizer tok_;
  std::vector<Entry> entries_;
  std::vector<size_t> order_;
  size_t cursor_ = 0;
  uint64_t epoch_ = 0;
  bool initialized_ = false;
};

// ---------------------------------------------------------------------------
class TcpStore {
 public:
  // Rank 0 (is_server) listens on `port` (0 = pick one, see port()); every rank
  // connects to host:port within timeout_ms.
  TcpStore(const std::string& host, int port, bool is_server, int timeout_ms = 30000);
  ~TcpStore();
  TcpStore(const TcpStore&) = delete;
  TcpStore& operator=(const TcpStore&) = delete;

  Status Set(const std::string& key, const std::string& value);
  // Blocks until the key exists or timeout_ms passes (kTimeout).
  Status Get(const std::string& key, std::string* value, int timeout_ms = -1);
  Status Add(const std::string& key, int64_t delta, int64_t* result);
  Status Wait(const std::vector<std::string>& keys, int timeout_ms = -1);
  // All `world` participants call Barrier(name); kTimeout if someone is missing.
  Status Barrier(const std::string& name, int world, int timeout_ms = -1);
  int port() const { return port_; }

 private:
  Status Request(char op, const std::string& key, const std::string& val, int timeout_ms, std::string* reply);
  void ServeLoop();
  void ServeClient(int fd);
  std::string host_;
  int port_;
  bool server_;
  int timeout_ms_;
  int listen_fd_ = -1, fd_ = -1;
  std::atomic<bool> stop_{false};
  std::thread accept_thread_;
  std::vector<std::thread> client_threads_;
  std::mutex data_mu_, req_mu_;
  std::condition_variable data_cv_;
  std::unordered_map<std::string, std::string> data_;
};

// ---------------------------------------------------------------------------
struct PipeOp {
  char kind;  // 'F' forward, 'B' backward
  int micro_batch;
};

class PipelineSchedule {
 public:
  static std::vector<PipeOp> OneFOneB(int num_stages, int stage, int num_micro_batches);
  static std::vector<PipeOp> GPipe(int num_stages, int stage, int num_micro_batches);
  // Peak number of in-flight micro-batch activations a stage holds.
  static int PeakActivations(const std::vector<PipeOp>& ops);
};

// ---------------------------------------------------------------------------
class KVBlockManager {
 public:
  KVBlockManager(int num_blocks, int block_size);
  // Reserves blocks for `num_tokens` tokens of a new sequence.
  Status Allocate(int64_t seq_id, int num_tokens);
  // Makes room for one more token; allocates a block at block boundaries.
  Status AppendToken(int64_t seq_id);
  Status Free(int64_t seq_id);
  bool CanAllocate(int num_tokens) const { return BlocksFor(num_tokens) <= static_cast<int>(free_.size()); }
  std::vector<int> BlockTable(int64_t seq_id) const;
  int SeqLen(int64_t seq_id) const;
  int NumFree() const { return static_cast<int>(free_.size()); }
  int NumBlocks() const { return num_blocks_; }
  int BlockSize() const { return block_size_; }
  int BlocksFor(int tokens) const { return (tokens + block_size_ - 1) / block_size_; }
  void Reset();

 private:
  struct Seq {
    std::vector<int> blocks;
    int len = 0;
  };
  int num_blocks_, block_size_;
  std::vector<int> free_;
  std::unordered_map<int64_t, Seq> seqs_;
};

}  // namespace turbol
